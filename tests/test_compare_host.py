"""Interleaved A/B (kernelverify_b200.runners.compare) against the scripted
fake worker's stream mode, on CPU: the speedup is reference best over
candidate best, a round whose reference arm spreads past the limit is
rejected and voids `ok`, and an arm that fails, crashes or hangs aborts the
comparison with its reason (the reference's compare.py semantics)."""

from __future__ import annotations

import math

import numpy as np

from kernelverify_b200.runners import (Binding, BindingKind, CudaRunner, KernelSpec, LaunchSpec,
                                       RunCase)
from kernelverify_b200.runners.compare import compare

SRC = 'extern "C" __global__ void k(float* out) {}'


def spec(name):
    return KernelSpec(source=SRC, entry_point="k", name=name,
                      bindings=(Binding(BindingKind.INPUT, "x"), Binding(BindingKind.OUTPUT),
                                Binding(BindingKind.SCALAR, "n", "uint32")),
                      launch=LaunchSpec(grid=("n", 1, 1), threadgroup=(32, 1, 1)))


def case(label="c", n=4):
    return RunCase(inputs={"x": np.zeros(n, np.float32)}, params={"n": n},
                   output_shapes=[((n,), "float32")], label=label)


def fake(**kw):
    return CudaRunner(worker_module="tests.fake_worker", case_timeout=1.5, startup_timeout=30,
                      **kw)


def test_speedup_is_reference_best_over_candidate_best():
    rep = compare(spec("slow"), spec("fast"), [case("a"), case("b")], rounds=3, runner=fake())
    assert rep.ok and not rep.failure and rep.rejected_rounds == 0
    assert [c.label for c in rep.cases] == ["a", "b"]
    for c in rep.cases:
        assert len(c.samples) == 3 and math.isclose(c.speedup, 2.0)


def test_a_noisy_reference_arm_rejects_rounds_and_voids_ok():
    rep = compare(spec("noisy"), spec("fast"), [case("a")], rounds=4, runner=fake())
    c = rep.cases[0]
    assert not rep.ok and rep.rejected_rounds == 2 and len(c.accepted) == 2
    assert math.isclose(c.speedup, 1.0) and "REJECTED" in rep.summary()


def test_a_failing_or_dying_arm_aborts():
    rep = compare(spec("fast"), spec("fast"), [case("a"), case("fail")], rounds=2, runner=fake())
    assert not rep.ok and "failed case 'fail'" in rep.failure
    rep = compare(spec("fast"), spec("slow"), [case("crash")], rounds=1, runner=fake())
    assert not rep.ok and "died" in rep.failure
    rep = compare(spec("fast"), spec("die-compiling"), [case("a")], rounds=1, runner=fake())
    assert not rep.ok and "before compiling" in rep.failure


def test_a_hung_arm_times_out():
    rep = compare(spec("fast"), spec("fast"), [case("hang")], rounds=1, runner=fake())
    assert not rep.ok and "timed out" in rep.failure


def test_cases_are_validated_before_any_worker_starts():
    bad = RunCase(inputs={"y": np.zeros(4, np.float32)}, params={"n": 4},
                  output_shapes=[((4,), "float32")], label="bad")
    rep = compare(spec("fast"), spec("fast"), [bad], runner=fake(python="/nonexistent"))
    assert not rep.ok and "arm A" in rep.failure
