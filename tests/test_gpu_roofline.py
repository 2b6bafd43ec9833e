"""The roofline probes on the B200: read-stream and copy bandwidth over a
buffer above L2 and the fp32 FMA rate land in physically plausible ranges
(well inside the spec ceilings, far above anything a broken probe reports)."""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def test_device_ceilings_are_plausible(native):
    from kernelverify_b200 import roofline
    res = roofline.measure(gib=0.5, repeats=3, warmup=2)
    assert 2000 < res["read_gbs"] < 1.2 * roofline.SPEC["hbm_gbs_dgx"], res
    assert 2000 < res["copy_gbs"] < 1.2 * roofline.SPEC["hbm_gbs_dgx"], res
    assert 10 < res["fp32_tflops"] < 1.1 * roofline.SPEC["fp32_tflops"], res
