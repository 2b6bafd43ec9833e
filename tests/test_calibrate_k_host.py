"""The K-calibration harness (oracle/calibrate_k.py) on a few cases: every
held-out implementation is a correct implementation (inside the shipped
tolerance on its own), the gates read what the rule says, and a planted wrong
implementation is exhibited as a soundness violation rather than absorbed."""

from __future__ import annotations

import numpy as np

from oracle import calibrate_k as ck
from oracle import cases, kv


def _case(bits=4, dtype="float32", t=300, group=64):
    q, kc, vc, nk, nv = cases.make_case(2, 4, t, 128, seed=17, dtype=dtype)
    return kv.kv_inputs(q, kc, vc, nk, nv, bits, group)


def test_held_out_implementations_are_correct():
    for bits, dtype, group in ((4, "float32", 64), (8, "float16", 64), (3, "float32", 32),
                               (2, "float16", 128)):
        x = _case(bits, dtype, group=group)
        ref, tol = kv.reference_and_tolerance(x, dtype)
        for name, fn in ck.HELD_OUT.items():
            err = kv.max_abs_error(fn(x), ref)
            assert err <= tol, (name, bits, dtype, err, tol)


def test_k_required_reads_the_rule():
    assert ck.k_required(base=1.0, floor_e=0.1, floor_c=0.9) == 0.0
    assert ck.k_required(base=0.1, floor_e=0.2, floor_c=0.5) == 2.5
    assert ck.k_required(base=0.0, floor_e=0.0, floor_c=0.5) == float("inf")


def test_draws_are_disjoint_in_seed_and_cover_the_extension_widths():
    specs = ck.draws()
    cal = [s for s in specs if s.draw == "calibration"]
    ind = [s for s in specs if s.draw == "independent"]
    ext = [s for s in specs if s.draw == "extension"]
    assert len(cal) == len(ind) == 400
    assert not {s.seed for s in cal} & {s.seed for s in ind}
    assert {dict(s.dims)["BITS"] for s in ext} == set(ck.EXTENSION_BITS)
    assert {s.group for s in ext} == {64, 32, 128}


def test_summary_on_a_small_sample():
    rows = [ck.measure(s) for s in ck.draws(limit=3)]
    summary = ck.summarize(rows)
    assert summary["cases"] == {"calibration": 3, "independent": 3, "extension": 3}
    assert set(summary["G2"]) == {str(k) for k in ck.K_GRID}
    assert "decision" in summary and ck.render(summary).startswith("# kv_attention K")


def test_a_wrong_implementation_is_exhibited(monkeypatch):
    """A planted held-out implementation with fp16 scores (a contract
    violation) must drive K_required past the shipped K on some case."""
    def fp16_scores(x):
        q, kd, vd, nk, nv, scale = ck._operands(x)
        s = (np.einsum("bhd,htd->bht", q, kd) * scale).astype(np.float16).astype(np.float32)
        s_new = np.sum(q * nk, axis=-1) * scale
        allv = np.concatenate([s, s_new[..., None]], axis=-1)
        p = np.exp(allv - allv.max(axis=-1, keepdims=True))
        p /= p.sum(axis=-1, keepdims=True)
        o = np.einsum("bht,htd->bhd", p[..., :-1], vd) + p[..., -1:] * nv
        return o.astype(x["q"].dtype)

    monkeypatch.setitem(ck.HELD_OUT, "planted-fp16-scores", fp16_scores)
    specs = [s for s in ck.draws() if s.draw == "calibration" and s.dtype == "float32"][:24]
    summary = ck.summarize([ck.measure(s) for s in specs])
    assert summary["k_required_by_impl"]["planted-fp16-scores"] > ck.K_SHIPPED
    assert not summary["G1_sound_at_shipped_K"]


def test_device_form_fits_fp16_steps_only():
    """The emulated tensor-core arithmetic sits well inside the tolerance of
    fp16 steps (the only steps those kernels serve) in both precisions, and
    outside it at fp32 -- why fp32 caches run the CUDA-core kernel."""
    for bits, group in ((4, 64), (8, 64), (3, 32)):
        x16 = _case(bits, "float16", group=group)
        ref, tol = kv.reference_and_tolerance(x16, "float16")
        for parts in (3, 2):
            assert kv.max_abs_error(ck.device_form(x16, parts), ref) <= 0.5 * tol, (bits, parts)
    x32 = _case(2, "float32", group=128)
    ref, tol = kv.reference_and_tolerance(x32, "float32")
    assert kv.max_abs_error(ck.device_form(x32, 3), ref) > tol
