"""The certificate data model, audit and rendering on the CPU: a certificate
that reads stronger than its evidence is refused (a failing case, C1 missing,
the fast precision, no byte-bound hashes, no chip)."""

from __future__ import annotations

import json

from kernelverify_b200 import certificate as C


def _cert(**kw):
    base = dict(bits=4, head_dim=128, dtype="float16", policy="p", seed_protocol="s",
                cases=[C.CaseEvidence("a", True, 1e-5, 1e-3, "00", "tensor-core"),
                       C.CaseEvidence("b", True, 2e-5, 1e-3, "11", "CUDA-core")],
                clauses=C.contract_clauses("contract"), translation_unit="ab" * 32,
                library="cd" * 32, flags=["-O3"], chip="NVIDIA B200",
                toolchain={"torch": "x"}, budget=2)
    base.update(kw)
    return C.Certificate(**base)


def test_an_honest_certificate_has_no_complaints():
    cert = _cert()
    assert C.audit(cert) == []
    doc = json.loads(cert.dumps())
    assert doc["kernel"] == "kv_attn_decode-BITS4-DH128-float16"
    assert doc["protocol_bound"]["all_passed"] is True
    assert {c["clause"] for c in doc["attestation"]["clauses"]} == {"C1", "C4", "C5"}
    assert "Audit complaints" not in C.render_markdown(cert)


def test_the_audit_refuses_what_the_evidence_does_not_carry():
    failing = _cert(cases=[C.CaseEvidence("a", False, 1.0, 1e-3, "00", "k")])
    assert any("failed" in p for p in C.audit(failing))
    fast = _cert(clauses=C.contract_clauses("fast"), precision="fast")
    complaints = C.audit(fast)
    assert any("C1" in p for p in complaints) and any("precision" in p for p in complaints)
    assert any("byte-bound" in p for p in C.audit(_cert(library="")))
    assert any("chip" in p for p in C.audit(_cert(chip="")))
    assert any("budget" in p for p in C.audit(_cert(budget=5)))
    assert "Audit complaints" in C.render_markdown(fast)


def test_the_translation_unit_hash_covers_the_sources():
    h = C.translation_unit_sha256()
    assert len(h) == 64 and h == C.translation_unit_sha256()
    assert any(f.startswith("-gencode") or "sm_100a" in f for f in C.build_flags())


def test_committed_certificates_are_complete_and_honest():
    """Every specialization (bits 2/3/4/6/8 x head_dim 64/128, fp16) has a
    committed certificate that passed every case, attests C1/C4/C5 at the
    contract precision, carries both byte-bound hashes and binds to a chip."""
    from pathlib import Path
    root = Path(__file__).resolve().parents[1] / "certificates"
    names = {f"kv_attn_decode-BITS{b}-DH{d}-float16" for b in (2, 3, 4, 6, 8) for d in (64, 128)}
    found = {p.name[:-len(".certificate.json")] for p in root.glob("*.certificate.json")}
    assert found == names
    for name in names:
        doc = json.loads((root / f"{name}.certificate.json").read_text())
        assert doc["kernel"] == name
        pb, bb = doc["protocol_bound"], doc["byte_bound"]
        assert pb["all_passed"] and pb["cases_passed"] == pb["cases_run"] > 0
        assert bb["precision"] == "contract"
        assert len(bb["translation_unit_sha256"]) == 64 and len(bb["library_sha256"]) == 64
        assert {c["clause"] for c in doc["attestation"]["clauses"]} >= {"C1", "C4", "C5"}
        assert "B200" in doc["validity"]["binding_on"]["chip_generation"]
        assert (root / f"{name}.md").exists()


def test_case_evidence_states_max_abs_and_max_rel():
    """A case judged with its reference magnitude carries max-rel beside
    max-abs in the advisory block; one without it carries max-abs only."""
    cert = _cert(cases=[C.CaseEvidence("a", True, 6e-5, 6e-4, "00", "tensor-core", ref_max=0.15),
                        C.CaseEvidence("b", True, 2e-5, 1e-3, "11", "CUDA-core")])
    a, b = json.loads(cert.dumps())["advisory"]["cases"]
    assert a["err"] == 6e-5 and abs(a["max_rel_err"] - 4e-4) < 1e-12 and a["ref_max_abs"] == 0.15
    assert "max_rel_err" not in b


def test_verdicts_carry_the_reference_magnitude():
    import numpy as np
    from oracle import kv
    ref = np.array([[0.5, -2.0]])
    v = kv.judge(ref + 1e-3, ref, 1e-2)
    assert v.ok and v.ref_max == 2.0 and abs(v.rel - 5e-4) < 1e-12
