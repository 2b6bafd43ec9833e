"""The B200 pack gate's host side (tests/gate.py): the reference's six gate
cases regenerate with their seeds, and the CLI parses. No device call."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import cases
from tests import gate


def test_the_six_gate_cases():
    got = gate.verify_cases()
    assert [g[0] for g in got] == [f"B={b} H={h} T={t} DH={d} {bits}-bit"
                                   for (b, h, t, d) in cases.VERIFY_SHAPES
                                   for bits in cases.VERIFY_BITS]
    label, bits, (b, h, t, d), arrays = got[0]
    again = cases.make_case(b, h, t, d, seed=t + bits)
    assert all(np.array_equal(x, y) for x, y in zip(arrays, again))


def test_cli_parses():
    with pytest.raises(SystemExit) as e:
        gate.main(["--help"])
    assert e.value.code == 0
