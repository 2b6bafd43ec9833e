"""The tensor-core kernels (fp16, 4-bit, head_dim 128, 8-row-aligned geometry)
and the CUDA-core kernel on the same inputs: each passes the oracle, and they
agree with each other to 2e-3 of the output's max magnitude (the tensor-core
kernels carry the V-side weights to 2^-23 relative by default, 2^-16 with
KVQ_PRECISION=fast). KVQ_KERNEL=generic forces the CUDA-core kernel for a
call, KVQ_KERNEL=umma the tcgen05 kernel (group 64; other groups keep the
register-fragment kernel)."""

from __future__ import annotations

import os

import numpy as np
import pytest

from oracle import cases
from tests.kvq_cases import judge_gqa, judge_per_sequence, pack, run_decode, to_dev

pytestmark = pytest.mark.gpu


def run_with(kernel, fn, precision=None):
    if kernel is not None:
        os.environ["KVQ_KERNEL"] = kernel
    if precision is not None:
        os.environ["KVQ_PRECISION"] = precision
    try:
        return fn()
    finally:
        os.environ.pop("KVQ_KERNEL", None)
        os.environ.pop("KVQ_PRECISION", None)


def kernels(fn):
    """(default tensor-core, tcgen05, CUDA-core) outputs of the same call; the
    default kernel's fast precision is checked against the oracle here too."""
    fast = run_with(None, fn, "fast")
    return run_with(None, fn), run_with("umma", fn), run_with("generic", fn), fast


def close(a, b, rel=2e-3):
    scale = max(1e-6, float(np.max(np.abs(b.astype(np.float64)))))
    return float(np.max(np.abs(a.astype(np.float64) - b))) <= rel * scale


@pytest.mark.parametrize("h,hkv", [(8, 8), (8, 4), (8, 2), (32, 8), (28, 4), (64, 8), (6, 2)])
@pytest.mark.parametrize("group", [32, 64, 128])
def test_tensor_core_path_gqa_and_groups(native, h, hkv, group):
    t = 1000   # not a multiple of the 64-position stage: the tail is masked
    q, kc, vc, nk, nv = cases.make_case(2, h, t, 128, seed=h * 7 + hkv + group)
    kc, vc, nk, nv = kc[:hkv], vc[:hkv], nk[:, :hkv], nv[:, :hkv]
    mma, umma, gen, fast = kernels(lambda: run_decode(q, kc, vc, nk, nv, 4, group))
    for out in (mma, umma, gen, fast):
        v = judge_gqa(q, kc, vc, nk, nv, 4, out, group)
        assert v.ok, v
    assert close(mma, gen) and close(umma, gen) and close(fast, gen)


@pytest.mark.parametrize("t", [1, 7, 8, 63, 64, 65, 129, 4096, 9000])
def test_tensor_core_path_lengths(native, t):
    q, kc, vc, nk, nv = cases.make_case(1, 8, max(t, 8), 128, seed=1000 + t)
    kc, vc = kc[:, :t], vc[:, :t]
    kc, vc, nk, nv = kc[:2], vc[:2], nk[:, :2], nv[:, :2]
    t_pad = -(-t // 8) * 8
    rng = np.random.default_rng(t)
    junk = rng.standard_normal((2, t_pad - t, 128)).astype(np.float16) * 30
    k_art = pack(np.concatenate([kc, junk], axis=1), 4)
    v_art = pack(np.concatenate([vc, junk], axis=1), 4)
    mma, umma, gen, fast = kernels(lambda: run_decode(q, None, None, nk, nv, 4, t_cached=t, k_art=k_art,
                                                 v_art=v_art))
    for out in (mma, umma, gen, fast):
        v = judge_gqa(q, kc, vc, nk, nv, 4, out)
        assert v.ok, (t, v)
    assert close(mma, gen) and close(umma, gen) and close(fast, gen)


def test_tensor_core_path_per_sequence_ragged(native):
    rng = np.random.default_rng(8)
    b, h, hkv, t_pad = 6, 32, 8, 2048
    lens = np.array([1, 100, 2048, 777, 1024, 64], dtype=np.int32)
    q = rng.standard_normal((b, h, 128)).astype(np.float16)
    kc = rng.standard_normal((b, hkv, t_pad, 128)).astype(np.float16)
    vc = rng.standard_normal((b, hkv, t_pad, 128)).astype(np.float16)
    nk = rng.standard_normal((b, hkv, 128)).astype(np.float16)
    nv = rng.standard_normal((b, hkv, 128)).astype(np.float16)
    mma, umma, gen, fast = kernels(lambda: run_decode(q, kc, vc, nk, nv, 4, t_cached=int(lens.max()),
                                                 seq_lens=lens))
    for out in (mma, umma, gen, fast):
        for v in judge_per_sequence(q, kc, vc, nk, nv, 4, out, lens):
            assert v.ok, v
    assert close(mma, gen) and close(umma, gen) and close(fast, gen)


@pytest.mark.parametrize("kernel", [None, "umma"])
def test_tensor_core_path_t_split_shards(native, kernel):
    """Shards starting at multiples of 8 run on the tensor-core kernels."""
    import torch
    from kernelverify_b200.pack import kv_attention as kva
    q, kc, vc, nk, nv = cases.make_case(1, 64, 4096, 128, seed=3)
    kc, vc, nk, nv = kc[:8], vc[:8], nk[:, :8], nv[:, :8]
    args = [to_dev(x) for x in (q, *pack(kc, 4), *pack(vc, 4), nk, nv)]
    bounds = [(0, 1024), (1024, 2048), (2048, 3072), (3072, 4096)]
    parts = run_with(kernel, lambda: [
        kva.decode_partial(*args, bits=4, t_begin=a, t_end=z, has_new_entry=(i == 3))
        for i, (a, z) in enumerate(bounds)])
    merged = kva.lse_merge(torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts]),
                           torch.stack([p[2] for p in parts]), torch.float16).cpu().numpy()
    v = judge_gqa(q, kc, vc, nk, nv, 4, merged)
    assert v.ok, v


def test_outlier_caches(native):
    """1% of cache entries x20 (config 3's distribution): wide scale/bias ranges."""
    rng = np.random.default_rng(33)
    q, nk, nv = (rng.standard_normal(s).astype(np.float16) for s in ((2, 32, 128), (2, 8, 128), (2, 8, 128)))
    raw = rng.standard_normal((2, 2, 8, 1536, 128)).astype(np.float32)
    raw[rng.random(raw.shape) < 0.01] *= 20
    raw = raw.astype(np.float16)
    kc, vc = raw[0], raw[1]
    mma, umma, gen, fast = kernels(lambda: run_decode(q, kc, vc, nk, nv, 4))
    for out in (mma, umma, gen, fast):
        for v in judge_per_sequence(q, kc, vc, nk, nv, 4, out):
            assert v.ok, v
