"""The roofline probe library on a machine without a GPU: it builds, exports
its probes, refuses bad arguments before any launch, and the host triad runs
on the CPU cores."""

from __future__ import annotations

import ctypes

from kernelverify_b200 import roofline


def test_probe_library_builds_and_exports():
    h = roofline.lib()
    for name in ("kvq_probe_blocks", "kvq_probe_read", "kvq_probe_copy", "kvq_probe_fma",
                 "kvq_probe_host_triad"):
        assert hasattr(h, name)


def test_bad_arguments_are_refused_before_a_launch():
    h = roofline.lib()
    assert h.kvq_probe_read(None, 1 << 20, None, 4, None) == -1
    assert h.kvq_probe_read(4096, 17, 4096, 4, None) == -1          # not a multiple of 16
    assert h.kvq_probe_copy(4096, None, 1 << 20, 4, None) == -1
    assert h.kvq_probe_fma(None, 4, 10, None) == -1
    g = ctypes.c_double()
    assert h.kvq_probe_host_triad(0, 1, 1, ctypes.byref(g)) == -1


def test_host_triad_measures_the_cpu():
    res = roofline.host_triad(n=1 << 20, reps=2, threads=2)
    assert res["host_triad_gbs"] > 0 and res["host_threads"] == 2


def test_spec_table():
    assert roofline.SPEC["sms"] == 148 and 70 < roofline.SPEC["fp32_tflops"] < 80
