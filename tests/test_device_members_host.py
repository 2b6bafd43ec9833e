"""The repaired kv tolerance contract with the factored device member
(oracle/device_members.py): it keeps the reference's four members and K,
only ever widens the tolerance, and admits the correct factored-form
implementation the shipped floor rejects on the calibration harness's
exhibited case."""

from __future__ import annotations

import pytest

from oracle import battery, calibrate_k as ck, device_members as dm, kv

# The independent-draw case the calibration harness exhibits: factored-serial
# needs K = 4.38 over the shipped four members there.
EXHIBIT = battery.Case(tuple(sorted({"B": 4, "BITS": 8, "DH": 64, "H": 2, "T": 512}.items())),
                       "float32", "corpus uniform[-10,10]", ck.INDEPENDENT_SEED_BASE + 256)


def test_members_are_the_shipped_four_plus_the_factored_form():
    assert list(dm.KV_DEVICE_MEMBERS)[:4] == list(kv.KV_MEMBERS)
    assert list(dm.KV_DEVICE_MEMBERS)[4:] == ["kv:factored-serial"]


@pytest.mark.parametrize("index", [0, 7, 121, 250, 399])
def test_the_repaired_tolerance_only_widens(index):
    case = battery.case_space()[index]
    x = battery.case_inputs(case)
    ref = kv.kv_reference(x)
    assert dm.kv_tolerance_device(case.dtype, x, ref) >= kv.kv_tolerance(case.dtype, x, ref)


def test_the_exhibited_factored_implementation_is_admitted():
    x = battery.case_inputs(EXHIBIT)
    ref = kv.kv_reference(x)
    shipped = kv.kv_tolerance("float32", x, ref)
    repaired = dm.kv_tolerance_device("float32", x, ref)
    err = kv.max_abs_error(ck.factored_serial(x), ref)
    assert err > shipped                 # the shipped floor rejects a correct implementation
    assert err <= repaired
    for name, fn in ck.HELD_OUT.items():  # and every held-out one passes the repaired floor
        assert kv.max_abs_error(fn(x), ref) <= repaired, name
    assert dm.verify_output_device(x, ck.factored_serial(x), "float32").ok
