"""The CUDA mutation battery's seam source (tests/seams/kvq_seams.cu), built
for the host: the same functions the sm_100a kernel runs reproduce the
reference's recorded battery verdicts -- the control passes, each of the
seven faults is detected exactly where the reference's numpy port is -- so a
machine without a GPU checks the source's arithmetic. No device call is made.

A stride through the 400 cases checks in-process; one test walks all 400 x 8
verdicts over a spawned pool (176/259/259/132/372/339/366 detections, every
control passing); the GPU test runs the device build against the host build."""

from __future__ import annotations

import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

from oracle import battery, faults, kv
from tests import seams

GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def bg():
    return json.loads((GOLDEN / "battery_golden.json").read_text())


@pytest.mark.parametrize("index", list(range(0, 400, 23)))
def test_host_build_reproduces_the_reference_verdicts(bg, index):
    rec = bg["cases"][index]
    case = battery.case_space()[index]
    inputs = battery.case_inputs(case)
    ref = kv.kv_reference(inputs)
    tol = kv.kv_tolerance(case.dtype, inputs, ref)
    assert battery.corpus_oracle_passes(seams.run_host(inputs, {}), ref, tol) == rec["control"]
    for params in faults.KV_FAULTS:
        detected = not battery.corpus_oracle_passes(seams.run_host(inputs, params), ref, tol)
        assert detected == rec["detected"][faults.fault_name(params)], params


def test_the_two_half_accumulations_are_one_computation():
    """numpy's float16 reduce over the position axis of the port's
    [B, H, T, DH] products is a running sum per dim, bit for bit its float16
    accumulate; the seam source computes both faults that way."""
    rng = np.random.default_rng(3)
    c = (rng.standard_normal((2, 3, 300, 64)) * 0.2).astype(np.float16)
    assert np.array_equal(np.add.reduce(c, axis=2, dtype=np.float16),
                          np.add.accumulate(c, axis=2, dtype=np.float16)[:, :, -1])
    inputs = battery.case_inputs(battery.case_space()[5])
    a = seams.run_host(inputs, {"accum_dtype": "float16"})
    b = seams.run_host(inputs, {"accum_dtype": "float16-seq"})
    assert np.array_equal(a.view(np.uint8), b.view(np.uint8))


def test_every_catalogue_entry_has_a_fault_bit():
    bits = {seams.fault_bit(p) for p in faults.KV_FAULTS}
    assert len(bits) == len(faults.KV_FAULTS) and 0 not in bits


@pytest.mark.parametrize("over", [dict(bits=5), dict(t_cached=8193), dict(group=48),
                                  dict(n_kv_heads=3), dict(fault=3), dict(dtype=2)])
def test_arguments_outside_the_seam_kernel_are_refused(over):
    """Refused before any pointer is read (host mode, dummy buffers)."""
    buf = np.zeros(64, dtype=np.float32)
    p = buf.ctypes.data
    a = dict(fault=0, dtype=0, b_rows=1, n_heads=4, n_kv_heads=2, t_cached=16, head_dim=64,
             bits=4, group=64)
    a.update(over)
    rc = seams.lib().kvq_seams_decode(0, a["fault"], a["dtype"], *([p] * 10), a["b_rows"],
                                      a["n_heads"], a["n_kv_heads"], a["t_cached"],
                                      a["head_dim"], a["bits"], a["group"], ctypes.c_void_p())
    assert rc == -1


def _case_verdicts(index: int):
    """(control verdict, {fault: detected}) of the seam source's host build on
    one battery case (run in a spawned worker)."""
    case = battery.case_space()[index]
    inputs = battery.case_inputs(case)
    ref = kv.kv_reference(inputs)
    tol = kv.kv_tolerance(case.dtype, inputs, ref)
    control = battery.corpus_oracle_passes(seams.run_host(inputs, {}), ref, tol)
    detected = {faults.fault_name(p): not battery.corpus_oracle_passes(seams.run_host(inputs, p),
                                                                       ref, tol)
                for p in faults.KV_FAULTS}
    return index, control, detected


def test_host_build_reproduces_every_recorded_verdict(bg):
    """All 400 cases x (control + 7 faults), spread over the host's cores:
    every verdict equals the reference's recorded one, so the detection
    counts are 176/259/259/132/372/339/366 of 400."""
    import multiprocessing as mp
    import os
    seams.build()
    with mp.get_context("spawn").Pool(min(8, os.cpu_count() or 1)) as pool:
        rows = pool.map(_case_verdicts, range(400), chunksize=10)
    counts = {name: 0 for name in bg["counts"]}
    for index, control, detected in rows:
        rec = bg["cases"][index]
        assert control == rec["control"], index
        assert detected == rec["detected"], index
        for name, d in detected.items():
            counts[name] += d
    assert counts == bg["counts"]
