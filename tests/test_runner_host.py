"""The runner contract and the CudaRunner's process logic, on CPU: data
contracts and their wire form (kernelverify/runners/spec.py, result.py),
specialize, and hang / crash / lost-context / compile-death / no-device
handling against a scripted fake worker (the reference tests the same paths
with /usr/bin/false and a spinning Metal kernel, tests/test_metal_runner.py:
502-543; a spinning GPU kernel is never run on a shared GPU, so the hang here
is a sleeping host process)."""

from __future__ import annotations

import numpy as np
import pytest

from kernelverify_b200.runners import (Binding, BindingKind, CudaRunner, KernelSpec, LaunchMode,
                                       LaunchSpec, RunCase, RunResult, RunStatus, SpecError,
                                       Timing, specialize)
from kernelverify_b200.runners.spec import resolve_extent

SRC = 'extern "C" __global__ void k(float* out) {}'


def spec(name="s"):
    return KernelSpec(source=SRC, entry_point="k", name=name,
                      bindings=(Binding(BindingKind.INPUT, "x"), Binding(BindingKind.OUTPUT),
                                Binding(BindingKind.SCALAR, "n", "uint32")),
                      launch=LaunchSpec(grid=("n", 1, 1), threadgroup=(32, 1, 1)))


def case(label="", n=4, fill=1):
    return RunCase(inputs={"x": np.zeros(n, np.float32)}, params={"n": n, "fill": fill},
                   output_shapes=[((n,), "float32")], label=label)


def test_extents():
    assert resolve_extent(3, {}, "g") == 3
    assert resolve_extent("n", {"n": 5}, "g") == 5
    assert resolve_extent(["a", 2, ["b"]], {"a": 3, "b": 4}, "g") == 24
    for bad in (True, [], "missing", 0, 1.5):
        with pytest.raises(SpecError):
            resolve_extent(bad, {"n": 1}, "g")


def test_spec_validation():
    with pytest.raises(SpecError):
        Binding(BindingKind.SCALAR, "")
    with pytest.raises(SpecError):
        Binding(BindingKind.SCALAR, "n", "float64")
    with pytest.raises(SpecError):
        Binding(BindingKind.INPUT)
    with pytest.raises(SpecError):
        KernelSpec(source=" ", entry_point="k", bindings=(Binding(BindingKind.OUTPUT),))
    with pytest.raises(SpecError):
        KernelSpec(source=SRC, entry_point="k", bindings=(Binding(BindingKind.INPUT, "x"),))
    with pytest.raises(SpecError):
        KernelSpec(source=SRC, entry_point="k",
                   bindings=(Binding(BindingKind.OUTPUT, index=1), Binding(BindingKind.OUTPUT)))
    with pytest.raises(SpecError):
        LaunchSpec(grid=(1, 1))
    with pytest.raises(SpecError):
        RunCase(inputs={}, output_shapes=[((0,), "float32")])
    with pytest.raises(SpecError):
        RunCase(inputs={}, output_shapes=[((1,), "float64")])
    with pytest.raises(SpecError):
        case().validate_against(KernelSpec(source=SRC, entry_point="k", bindings=(
            Binding(BindingKind.INPUT, "y"), Binding(BindingKind.OUTPUT))))


def test_wire_forms_round_trip():
    s = spec()
    assert KernelSpec.from_json(s.to_json()) == s
    c = case("lbl")
    back = RunCase.from_json(c.to_json())
    assert back.label == "lbl" and np.array_equal(back.inputs["x"], c.inputs["x"])
    r = RunResult(status=RunStatus.OK, outputs=[np.arange(3, dtype=np.float16)],
                  timing=Timing((1.0, 2.0), (3.0,), 1), label="z")
    rb = RunResult.from_json(r.to_json())
    assert rb.ok and rb.timing.gpu_best == 1.0 and rb.timing.gpu_spread == 2.0
    assert np.array_equal(rb.outputs[0], r.outputs[0])
    assert LaunchSpec.from_json(LaunchSpec(mode=LaunchMode.THREADGROUPS).to_json()).mode \
        is LaunchMode.THREADGROUPS


def test_specialize():
    t = KernelSpec(source="// $BITS $DH", entry_point="k_$BITS", name="n-$DH",
                   bindings=(Binding(BindingKind.OUTPUT),))
    s = specialize(t, {"BITS": 4, "DH": 128})
    assert s.source == "// 4 128" and s.entry_point == "k_4" and s.name == "n-128"
    with pytest.raises(SpecError, match="do not supply"):
        specialize(t, {"BITS": 4})
    with pytest.raises(SpecError, match="appear nowhere"):
        specialize(t, {"BITS": 4, "DH": 1, "BTIS": 2})


def fake(**kw):
    return CudaRunner(worker_module="tests.fake_worker", case_timeout=1.5, startup_timeout=30, **kw)


def test_batch_runs_and_reports_compile_options():
    [batch] = fake().run_candidate([(spec(), [case("a", fill=2), case("b")])])
    assert batch.all_ok and batch.device.name == "fake"
    assert np.array_equal(batch[0].outputs[0], np.full(4, 2.0, np.float32))
    assert batch.compile_options == {"math_mode": "safe"}


def test_hang_costs_one_case_and_resumes():
    [batch] = fake().run_candidate([(spec(), [case("a"), case("hang"), case("c")])])
    assert [r.status for r in batch] == [RunStatus.OK, RunStatus.TIMEOUT, RunStatus.OK]


def test_crash_costs_one_case_and_resumes():
    [batch] = fake().run_candidate([(spec(), [case("crash"), case("b"), case("crash"), case("d")])])
    assert [r.status for r in batch] == [RunStatus.CRASH, RunStatus.OK, RunStatus.CRASH, RunStatus.OK]


def test_lost_context_restarts_without_blaming_the_next_case():
    [batch] = fake().run_candidate([(spec(), [case("sticky"), case("b"), case("c")])])
    assert [r.status for r in batch] == [RunStatus.LAUNCH_ERROR, RunStatus.OK, RunStatus.OK]


def test_death_while_compiling_fails_that_spec_only():
    out = fake().run_candidate([(spec("die-compiling"), [case("a"), case("b")]),
                                (spec("fine"), [case("c")])])
    assert [r.status for r in out[0]] == [RunStatus.CRASH, RunStatus.CRASH]
    assert out[1].all_ok


def test_invalid_spec_is_caught_before_a_process():
    bad = RunCase(inputs={}, params={"n": 4}, output_shapes=[((4,), "float32")])
    out = fake().run_candidate([(spec(), [bad]), (spec(), [case("ok")])])
    assert out[0][0].status is RunStatus.INVALID_SPEC and out[1].all_ok


def test_no_device_is_unsupported_for_every_case():
    r = fake(worker_env={"FAKE_NO_DEVICE": "1"})
    [batch] = r.run_candidate([(spec(), [case(), case()])])
    assert [x.status for x in batch] == [RunStatus.UNSUPPORTED] * 2
    assert r.probe() is None


def test_a_worker_that_cannot_start_is_a_crash():
    r = CudaRunner(python="/usr/bin/false", startup_timeout=10)
    [batch] = r.run_candidate([(spec(), [case()])])
    assert batch[0].status is RunStatus.CRASH


def test_probe_finds_the_fake_device():
    assert fake().probe().name == "fake"


def test_real_worker_without_a_gpu_reports_unsupported():
    r = CudaRunner(worker_env={"KVQ_FORCE_NO_GPU": "1"}, startup_timeout=120)
    [batch] = r.run_candidate([(spec(), [case()])])
    assert batch[0].status is RunStatus.UNSUPPORTED


def test_ragged_kernel_spec_adds_seq_lens_after_new_v():
    """The raw door keeps the reference's bindings in order; the ragged form
    inserts one int32 input, seq_lens, before the output."""
    from kernelverify_b200.pack.kv_attention import kernel_spec
    from kernelverify_b200.runners import BindingKind, specialize
    plain = specialize(kernel_spec(), {"T": "half", "BITS": 4, "DH": 128})
    ragged = specialize(kernel_spec(ragged=True), {"T": "half", "BITS": 4, "DH": 128})
    names = lambda spec: [b.name for b in spec.bindings if b.kind is BindingKind.INPUT]
    assert names(plain) == ["q", "k_wq", "k_scales", "k_biases", "v_wq", "v_scales", "v_biases",
                            "new_k", "new_v"]
    assert names(ragged) == names(plain) + ["seq_lens"]
    assert ragged.output_count() == plain.output_count() == 1
    scalars = lambda spec: [b.name for b in spec.bindings if b.kind is BindingKind.SCALAR]
    assert scalars(ragged) == scalars(plain) == ["n_heads", "t_cached", "n_kv_heads", "t_stride"]
