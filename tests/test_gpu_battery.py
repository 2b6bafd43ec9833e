"""All 400 cases of the reference's kv battery through the CUDA path.

The battery's control is the correct kernel: it must pass the shipped oracle
(fp64 reference, floored tolerance, the corpus validator's shape and
finiteness checks) on every case, fp16 and fp32, every input mode
(kernelverify/battery/core.py:253-329, the control check at :312-319).
"""

from __future__ import annotations

import pytest

from oracle import battery, kv
from tests.kvq_cases import run_decode

pytestmark = pytest.mark.gpu


def test_cuda_control_passes_all_400_battery_cases(native):
    failures = []
    space = battery.case_space()
    assert len(space) == 400
    for case in space:
        inputs = battery.case_inputs(case)
        ref = kv.kv_reference(inputs)
        tol = kv.kv_tolerance(case.dtype, inputs, ref)
        bits = int(inputs["bits"][0])
        out = run_decode(inputs["q"], inputs["k_cache"], inputs["v_cache"], inputs["new_k"],
                         inputs["new_v"], bits)
        if not battery.corpus_oracle_passes(out, ref, tol):
            failures.append((case, kv.max_abs_error(out, ref), tol))
    assert not failures, f"{len(failures)} battery cases fail, first: {failures[:3]}"
