"""The B200 pack gate (tests/gate.py): the six gate cases verify through the
isolated runner, the stock arm passes the same oracle, the device quantizer's
artefacts equal the canonical ones; one timing row runs end to end."""

from __future__ import annotations

import pytest

pytestmark = pytest.mark.gpu


def test_gate_verifies(native):
    from tests import gate
    assert gate.verify()


def test_a_timing_row_runs(native):
    from tests import gate
    row, spread, agree = gate.time_row(1, 8, 128, 128, 4, rounds=2)
    assert agree and spread >= 1.0
    if row is not None:
        ours, stock = row
        assert ours > 0 and stock > 0
