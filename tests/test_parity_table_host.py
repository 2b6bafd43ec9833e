"""The parity table of the certified cases (tests/parity_table.py) on one
committed certificate: the protocol's inputs regenerate on the CPU, the
recomputed tolerances equal the recorded ones bit for bit (the certificates'
protocol-bound claim, for the host half of the verdict), and each case's
max-rel error is below fp16's unit roundoff."""

from __future__ import annotations

from pathlib import Path

from tests import parity_table

CERTS = Path(__file__).resolve().parents[1] / "certificates"


def test_certified_cases_reproduce_their_tolerances_and_stay_under_an_fp16_rounding():
    table = parity_table.rows(CERTS, "kv_attn_decode-BITS4-DH128-float16.certificate.json")
    assert len(table) == 4
    for r in table:
        assert r["how"].startswith("recomputed") and "differs" not in r["how"], r
        assert r["passed"] and r["err"] <= r["tol"]
        assert r["rel"] < 2.0 ** -11, r
