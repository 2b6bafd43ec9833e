"""The CUDA path against the oracle, on a B200.

Dequantization and the device quantizer must be bit-exact to the reference's
numpy (pinned through tests/golden/quant_golden.npz). Attention outputs must
pass the reference's own verdict -- fp64 reference, tolerance
max(4*eps*max|ref|, 4*ensemble floor) -- which the tests never restate; the
gate cases are judged against the reference's own fp64 outputs and
tolerances from tests/golden/gate_golden.npz.
"""

from __future__ import annotations

import json
from pathlib import Path

import numpy as np
import pytest

from oracle import cases, kv, quant
from tests.kvq_cases import judge_gqa, judge_per_sequence, pack, run_decode, to_dev

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def kva(native):
    from kernelverify_b200.pack import kv_attention
    return kv_attention


@pytest.fixture(scope="module")
def qg():
    return np.load(GOLDEN / "quant_golden.npz")


@pytest.mark.parametrize("dtype", ["float16", "float32"])
@pytest.mark.parametrize("bits", [2, 3, 4, 6, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_device_dequant_bit_exact(kva, qg, dtype, bits, group):
    key = f"{dtype}_b{bits}_g{group}"
    words, scales, biases = (to_dev(qg[f"{n}_{key}"]) for n in ("words", "scales", "biases"))
    out = kva.dequant(words, scales, biases, bits).cpu().numpy()
    assert np.array_equal(out.view(np.uint32), qg[f"deq_{key}"].view(np.uint32))


@pytest.mark.parametrize("dtype", ["float16", "float32"])
@pytest.mark.parametrize("bits", [2, 3, 4, 6, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_device_quantizer_bit_exact(kva, qg, dtype, bits, group):
    key = f"{dtype}_b{bits}_g{group}"
    words, scales, biases = kva.quantize(to_dev(qg[f"w_{dtype}"]), bits, group)
    assert np.array_equal(words.cpu().numpy().view(np.uint32), qg[f"words_{key}"])
    assert np.array_equal(scales.cpu().numpy().view(np.uint8), qg[f"scales_{key}"].view(np.uint8))
    assert np.array_equal(biases.cpu().numpy().view(np.uint8), qg[f"biases_{key}"].view(np.uint8))


def test_device_quantizer_bit_exact_at_scale(kva):
    """A large N(0,1) cache with outliers, every width: the device artefact is
    the oracle's, byte for byte."""
    rng = np.random.default_rng(5)
    w = rng.standard_normal((4096, 128)).astype(np.float32)
    w[rng.random(w.shape) < 0.01] *= 20
    w = w.astype(np.float16)
    for bits in (2, 3, 4, 6, 8):
        for group in (32, 64, 128):
            dw, ds, db = kva.quantize(to_dev(w), bits, group)
            codes, s, b = quant.canonical_quantize(w, bits, group)
            assert np.array_equal(dw.cpu().numpy().view(np.uint32), quant.pack_codes(codes, bits))
            assert np.array_equal(ds.cpu().numpy().view(np.uint16), s.view(np.uint16))
            assert np.array_equal(db.cpu().numpy().view(np.uint16), b.view(np.uint16))


def _gate():
    z = np.load(GOLDEN / "gate_golden.npz")
    return z, json.loads(bytes(z["meta_json"]).decode())


def _gate_inputs(spec):
    b, h, t, dh = spec["shape"]
    q, kc, vc, nk, nv = cases.make_case(b, h, t, dh, seed=spec["seed"], dtype=spec["dtype"])
    if spec.get("dominate"):
        nk = (q.astype(np.float32) * 60.0).astype(np.float16)
    hkv = spec.get("hkv", h)
    if hkv != h:
        kc, vc, nk, nv = kc[:hkv], vc[:hkv], nk[:, :hkv], nv[:, :hkv]
    return q, kc, vc, nk, nv


@pytest.mark.parametrize("index", range(24))
def test_gate_and_unit_cases_against_reference_outputs(kva, index):
    """The six gate cases (bench/pack_kv_attention.py:65-66) and the
    reference's kv unit-test cases, judged against the reference's own fp64
    output and tolerance."""
    z, meta = _gate()
    spec = meta[index]
    q, kc, vc, nk, nv = _gate_inputs(spec)
    g = spec.get("group", 64)
    out = run_decode(q, kc, vc, nk, nv, spec["bits"], g)
    assert out.dtype == np.dtype(spec["dtype"])
    v = kv.judge(out, z[f"ref_{index}"], spec["tol"])
    assert v.ok, f"{spec['label']}: {v}"
    if spec.get("dominate"):   # tests/test_pack_kv_attention.py:116-117
        assert float(np.max(np.abs(out - nv.astype(np.float64)))) < 0.05


def test_batch_rows_are_independent(kva):
    """Each batch row reproduces its own B=1 answer exactly
    (tests/test_pack_kv_attention.py:120-130)."""
    b, h, t, dh = 4, 2, 96, 64
    q, kc, vc, nk, nv = cases.make_case(b, h, t, dh, seed=11)
    full = run_decode(q, kc, vc, nk, nv, 4)
    for row in range(b):
        one = run_decode(q[row:row + 1], kc, vc, nk[row:row + 1], nv[row:row + 1], 4)
        assert np.array_equal(full[row:row + 1], one)


def test_padded_cache_reads_only_the_logical_prefix(kva):
    """Rows past the logical length hold garbage; any read past t_cached, or a
    stride confusion between heads, fails the oracle
    (tests/test_pack_kv_attention.py:143-173)."""
    b, h, t, t_pad, dh, bits = 1, 4, 300, 512, 128, 8
    q, kc, vc, nk, nv = cases.make_case(b, h, t, dh, seed=23)
    rng = np.random.default_rng(99)
    junk_k = rng.standard_normal((h, t_pad - t, dh)).astype(np.float16) * 50
    junk_v = rng.standard_normal((h, t_pad - t, dh)).astype(np.float16) * 50
    k_art = pack(np.concatenate([kc, junk_k], axis=1), bits)
    v_art = pack(np.concatenate([vc, junk_v], axis=1), bits)
    out = run_decode(q, None, None, nk, nv, bits, t_cached=t, k_art=k_art, v_art=v_art)
    v = kv.verify_output(kv.kv_inputs(q, kc, vc, nk, nv, bits), out)
    assert v.ok, v


def test_empty_cache_returns_the_new_entry(kva):
    """T=0: the softmax has one entry, p_new = 1, so out == new_v exactly."""
    b, h, dh, bits = 2, 4, 128, 4
    q, kc, vc, nk, nv = cases.make_case(b, h, 8, dh, seed=4)
    k_art, v_art = pack(kc, bits), pack(vc, bits)
    out = run_decode(q, None, None, nk, nv, bits, t_cached=0, k_art=k_art, v_art=v_art)
    assert np.array_equal(out, nv)


@pytest.mark.parametrize("t", [1023, 1024, 1025, 5000, 20000])
def test_lengths_past_the_reference_capacity(kva, t):
    """The reference kernel stops at T = 1024 (kernelverify/pack/kv_attention.py:77);
    the split-T kernel serves any length, across tile and split boundaries."""
    q, kc, vc, nk, nv = cases.make_case(1, 4, t, 128, seed=t)
    out = run_decode(q, kc, vc, nk, nv, 4)
    v = kv.verify_output(kv.kv_inputs(q, kc, vc, nk, nv, 4), out)
    assert v.ok, v


@pytest.mark.parametrize("bits,group", [(2, 128), (3, 32), (4, 64), (6, 32), (8, 128), (3, 128)])
@pytest.mark.parametrize("dh", [64, 128])
def test_widths_groups_and_head_dims(kva, bits, group, dh):
    if dh % group:
        pytest.skip("group does not divide head_dim")
    q, kc, vc, nk, nv = cases.make_case(2, 4, 700, dh, seed=bits * 7 + group + dh)
    out = run_decode(q, kc, vc, nk, nv, bits, group)
    v = kv.verify_output(kv.kv_inputs(q, kc, vc, nk, nv, bits, group), out)
    assert v.ok, v


@pytest.mark.parametrize("h,hkv", [(8, 2), (28, 4), (32, 8), (64, 8), (12, 1), (24, 2), (6, 2)])
def test_gqa_ratios(kva, h, hkv):
    """GQA r = 4, 7, 4, 8, 12 (two head tiles), 12, 3 against the tiled oracle."""
    q, kc, vc, nk, nv = cases.make_case(2, h, 600, 128, seed=h * 100 + hkv)
    kc, vc, nk, nv = kc[:hkv], vc[:hkv], nk[:, :hkv], nv[:, :hkv]
    out = run_decode(q, kc, vc, nk, nv, 4)
    v = judge_gqa(q, kc, vc, nk, nv, 4, out)
    assert v.ok, v


def test_fp32_gqa_group32(kva):
    q, kc, vc, nk, nv = cases.make_case(2, 8, 333, 128, seed=9, dtype="float32")
    kc, vc, nk, nv = kc[:2], vc[:2], nk[:, :2], nv[:, :2]
    out = run_decode(q, kc, vc, nk, nv, 4, 32)
    assert out.dtype == np.float32
    v = judge_gqa(q, kc, vc, nk, nv, 4, out, 32, "float32")
    assert v.ok, v


def test_per_sequence_and_ragged_caches(kva):
    """One cache per sequence, ragged logical lengths in a padded buffer,
    each sequence judged as its own case."""
    rng = np.random.default_rng(77)
    b, h, hkv, dh, t_pad, bits = 5, 28, 4, 128, 1500, 8
    lens = np.array([1, 345, 1024, 1500, 777], dtype=np.int32)
    q = rng.standard_normal((b, h, dh)).astype(np.float16)
    kc = rng.standard_normal((b, hkv, t_pad, dh)).astype(np.float16)
    vc = rng.standard_normal((b, hkv, t_pad, dh)).astype(np.float16)
    nk = rng.standard_normal((b, hkv, dh)).astype(np.float16)
    nv = rng.standard_normal((b, hkv, dh)).astype(np.float16)
    out = run_decode(q, kc, vc, nk, nv, bits, t_cached=int(lens.max()), seq_lens=lens)
    for v in judge_per_sequence(q, kc, vc, nk, nv, bits, out, lens):
        assert v.ok, v


def test_t_split_shards_merge_to_the_single_pass(kva):
    """Positions split into 3 unequal ranges, the new entry in the last one,
    merged by log-sum-exp: the oracle passes it and it sits within fp32
    rounding of the single-pass step."""
    import torch
    q, kc, vc, nk, nv = cases.make_case(2, 8, 3000, 128, seed=12)
    kc, vc, nk, nv = kc[:2], vc[:2], nk[:, :2], nv[:, :2]
    bits = 4
    args = [to_dev(x) for x in (q, *pack(kc, bits), *pack(vc, bits), nk, nv)]
    bounds = [(0, 700), (700, 2100), (2100, 3000)]
    parts = [kva.decode_partial(*args, bits=bits, t_begin=lo, t_end=hi,
                                has_new_entry=(i == len(bounds) - 1))
             for i, (lo, hi) in enumerate(bounds)]
    po = torch.stack([p[0] for p in parts])
    pm = torch.stack([p[1] for p in parts])
    pl = torch.stack([p[2] for p in parts])
    merged = kva.lse_merge(po, pm, pl, torch.float16).cpu().numpy()
    single = kva.decode(*args, bits=bits).cpu().numpy()
    v = judge_gqa(q, kc, vc, nk, nv, bits, merged)
    assert v.ok, v
    assert np.max(np.abs(merged.astype(np.float64) - single)) <= 2 * 9.77e-4 * np.max(np.abs(single))


def test_door_spelling_matches_the_reference(kva):
    """build(torch) in the MLX door's call shape (kernelverify/pack/kv_attention.py:369-393)."""
    import torch
    kernel = kva.build(torch)
    b, h, t, dh, bits = 1, 8, 512, 128, 4
    q, kc, vc, nk, nv = cases.make_case(b, h, t, dh, seed=t + bits)
    ins = [to_dev(x) for x in (q, *pack(kc, bits), *pack(vc, bits), nk, nv)]
    [out] = kernel(inputs=ins, t_cached=t, output_shapes=[(b, h, dh)],
                   output_dtypes=[torch.float16],
                   template=[("T", torch.float16), ("BITS", bits), ("DH", dh)])
    v = kv.verify_output(kv.kv_inputs(q, kc, vc, nk, nv, bits), out.cpu().numpy())
    assert v.ok, v


def test_invalid_arguments_raise_before_launch(kva):
    import torch
    from kernelverify_b200._native import KvqError
    q, kc, vc, nk, nv = cases.make_case(1, 4, 64, 128, seed=1)
    ins = [to_dev(x) for x in (q, *pack(kc, 4), *pack(vc, 4), nk, nv)]
    with pytest.raises(ValueError):
        kva.decode(*ins, bits=5)
    with pytest.raises(ValueError, match="exceeds"):
        kva.decode(*ins, bits=4, t_cached=65)
    a = kva._args(*ins, bits=4)
    a.group_size = 48
    lib = kva._native.lib()
    out = torch.empty_like(ins[0])
    status = lib.kvq_decode(a, out.data_ptr(), None, 0, None)
    assert status == -1 and b"group_size" in lib.kvq_last_error()
    with pytest.raises(KvqError):
        kva._native.check(status)
