"""Certificates emitted on the B200 for two specializations: every protocol
case passes, the audit raises nothing, and the files say what was verified."""

from __future__ import annotations

import json

import pytest

pytestmark = pytest.mark.gpu


def test_emit_two_specializations(native, tmp_path):
    from tests import certify
    written, refused = certify.emit(tmp_path, [4, 8], [128])
    assert refused == []
    assert [c.kernel_name for c in written] == ["kv_attn_decode-BITS4-DH128-float16",
                                                "kv_attn_decode-BITS8-DH128-float16"]
    doc = json.loads((tmp_path / "kv_attn_decode-BITS4-DH128-float16.certificate.json").read_text())
    assert doc["protocol_bound"]["all_passed"] and doc["protocol_bound"]["cases_run"] == 4
    assert "B200" in doc["validity"]["binding_on"]["chip_generation"]
    kernels = {c["kernel"] for c in doc["advisory"]["cases"]}
    # max-abs and max-rel versus fp64 on fp16 outputs, both stated per case
    assert all(0 < c["max_rel_err"] < 2.0 ** -11 for c in doc["advisory"]["cases"])
    assert any("tensor-core" in k for k in kernels)
    assert (tmp_path / "MANIFEST.md").exists()
