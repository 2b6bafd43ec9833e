"""The byte-code tensor-core kernel (fp16, head_dim 128, 2-, 3-, 6- and 8-bit
codes at groups 32, 64 and 128, 8-row-aligned geometry) against the oracle and against the
CUDA-core kernel on the same inputs, in both precisions: GQA ratios up to 8
(config 4's 28/4 among them), lengths that end mid-stage, ragged per-sequence
caches, T-range shards and outlier caches. Each case first checks that the
library planned the tensor-core kernel, so the comparison is never the
CUDA-core kernel with itself."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import cases
from tests.kvq_cases import judge_gqa, judge_per_sequence, pack, run_decode, to_dev
from tests.test_gpu_paths import close, run_with

pytestmark = pytest.mark.gpu

WIDTHS = (2, 3, 6, 8)
GROUPS = (32, 64, 128)


def planned(q, kc, vc, nk, nv, BITS, t_cached=None, seq_lens=None, k_art=None, v_art=None,
            group=64):
    from kernelverify_b200.pack import kv_attention as kva
    kw, ks, kb = k_art if k_art is not None else pack(kc, BITS, group)
    vw, vs, vb = v_art if v_art is not None else pack(vc, BITS, group)
    args = [to_dev(x) for x in (q, kw, ks, kb, vw, vs, vb, nk, nv)]
    sl = to_dev(np.asarray(seq_lens, dtype=np.int32)) if seq_lens is not None else None
    return kva.plan_kernel(*args, bits=BITS, t_cached=t_cached, seq_lens=sl)


def three(fn):
    """(tensor-core, its fast precision, CUDA-core) outputs of one call."""
    return run_with(None, fn), run_with(None, fn, "fast"), run_with("generic", fn)


@pytest.mark.parametrize("group", GROUPS)
@pytest.mark.parametrize("BITS", WIDTHS)
@pytest.mark.parametrize("h,hkv", [(8, 8), (8, 4), (8, 2), (32, 8), (28, 4), (64, 8), (6, 2)])
def test_byte_kernel_gqa(native, h, hkv, BITS, group):
    t = 1000
    q, kc, vc, nk, nv = cases.make_case(2, h, t, 128, seed=h * 11 + hkv + group)
    kc, vc, nk, nv = kc[:hkv], vc[:hkv], nk[:, :hkv], nv[:, :hkv]
    assert planned(q, kc, vc, nk, nv, BITS, group=group) == "tensor-core"
    tc, fast, gen = three(lambda: run_decode(q, kc, vc, nk, nv, BITS, group))
    for out in (tc, fast, gen):
        v = judge_gqa(q, kc, vc, nk, nv, BITS, out, group)
        assert v.ok, v
    assert close(tc, gen) and close(fast, gen)


LENGTHS = [(t, 64) for t in (1, 7, 8, 63, 64, 65, 129, 4096, 9000)] + \
    [(t, g) for g in (32, 128) for t in (1, 65, 4096)]


@pytest.mark.parametrize("BITS", WIDTHS)
@pytest.mark.parametrize("t,group", LENGTHS)
def test_byte_kernel_lengths(native, t, group, BITS):
    q, kc, vc, nk, nv = cases.make_case(1, 8, max(t, 8), 128, seed=2000 + t)
    kc, vc = kc[:2, :t], vc[:2, :t]
    nk, nv = nk[:, :2], nv[:, :2]
    t_pad = -(-t // 8) * 8
    rng = np.random.default_rng(t)
    junk = rng.standard_normal((2, t_pad - t, 128)).astype(np.float16) * 30
    k_art = pack(np.concatenate([kc, junk], axis=1), BITS, group)
    v_art = pack(np.concatenate([vc, junk], axis=1), BITS, group)
    assert planned(q, None, None, nk, nv, BITS, t_cached=t, k_art=k_art,
                   v_art=v_art) == "tensor-core"
    tc, fast, gen = three(lambda: run_decode(q, None, None, nk, nv, BITS, group, t_cached=t,
                                             k_art=k_art, v_art=v_art))
    for out in (tc, fast, gen):
        v = judge_gqa(q, kc, vc, nk, nv, BITS, out, group)
        assert v.ok, (t, v)
    assert close(tc, gen) and close(fast, gen)


@pytest.mark.parametrize("group", GROUPS)
@pytest.mark.parametrize("BITS", WIDTHS)
def test_byte_kernel_ragged_per_sequence(native, BITS, group):
    """Config 4's form: one cache per sequence, device lengths, GQA 7."""
    rng = np.random.default_rng(18)
    b, h, hkv, t_pad = 5, 28, 4, 2048
    lens = np.array([1, 300, 2048, 777, 64], dtype=np.int32)
    q = rng.standard_normal((b, h, 128)).astype(np.float16)
    kc = rng.standard_normal((b, hkv, t_pad, 128)).astype(np.float16)
    vc = rng.standard_normal((b, hkv, t_pad, 128)).astype(np.float16)
    nk = rng.standard_normal((b, hkv, 128)).astype(np.float16)
    nv = rng.standard_normal((b, hkv, 128)).astype(np.float16)
    assert planned(q, kc, vc, nk, nv, BITS, t_cached=int(lens.max()), seq_lens=lens,
                   group=group) == "tensor-core"
    tc, fast, gen = three(lambda: run_decode(q, kc, vc, nk, nv, BITS, group,
                                             t_cached=int(lens.max()), seq_lens=lens))
    for out in (tc, fast, gen):
        for v in judge_per_sequence(q, kc, vc, nk, nv, BITS, out, lens, group):
            assert v.ok, v
    assert close(tc, gen) and close(fast, gen)


@pytest.mark.parametrize("group", GROUPS)
@pytest.mark.parametrize("BITS", WIDTHS)
def test_byte_kernel_t_split_shards(native, BITS, group):
    import torch
    from kernelverify_b200.pack import kv_attention as kva
    q, kc, vc, nk, nv = cases.make_case(1, 64, 4096, 128, seed=5)
    kc, vc, nk, nv = kc[:8], vc[:8], nk[:, :8], nv[:, :8]
    args = [to_dev(x) for x in (q, *pack(kc, BITS, group), *pack(vc, BITS, group), nk, nv)]
    bounds = [(0, 1024), (1024, 2048), (2048, 3072), (3072, 4096)]
    parts = [kva.decode_partial(*args, bits=BITS, t_begin=a, t_end=z, has_new_entry=(i == 3))
             for i, (a, z) in enumerate(bounds)]
    merged = kva.lse_merge(torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts]),
                           torch.stack([p[2] for p in parts]), torch.float16).cpu().numpy()
    v = judge_gqa(q, kc, vc, nk, nv, BITS, merged, group)
    assert v.ok, v


@pytest.mark.parametrize("group", GROUPS)
@pytest.mark.parametrize("BITS", WIDTHS)
def test_byte_kernel_outlier_caches(native, BITS, group):
    rng = np.random.default_rng(44)
    q, nk, nv = (rng.standard_normal(s).astype(np.float16)
                 for s in ((2, 32, 128), (2, 8, 128), (2, 8, 128)))
    raw = rng.standard_normal((2, 2, 8, 1536, 128)).astype(np.float32)
    raw[rng.random(raw.shape) < 0.01] *= 20
    raw = raw.astype(np.float16)
    kc, vc = raw[0], raw[1]
    assert planned(q, kc, vc, nk, nv, BITS, group=group) == "tensor-core"
    tc, fast, gen = three(lambda: run_decode(q, kc, vc, nk, nv, BITS, group))
    for out in (tc, fast, gen):
        for v in judge_per_sequence(q, kc, vc, nk, nv, BITS, out, group=group):
            assert v.ok, v
    assert close(tc, gen) and close(fast, gen)
