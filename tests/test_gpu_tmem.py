"""The warp-specialised tensor-memory kernel (KVQ_KERNEL=tmem; fp16, 4-bit,
head_dim 128, group 64) against the oracle, across tile boundaries, GQA
ratios, ragged and T-split steps, item counts above and below one per SM, and
against the CUDA-core kernel on the same inputs."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import cases
from tests.kvq_cases import judge_gqa, judge_per_sequence, pack, run_decode, to_dev
from tests.test_gpu_paths import close, run_with

pytestmark = pytest.mark.gpu


def tmem_and_generic(fn):
    return run_with("tmem", fn), run_with("generic", fn)


def test_plan_names_the_kernel(native):
    from kernelverify_b200.pack import kv_attention as kva
    q, kc, vc, nk, nv = cases.make_case(1, 8, 256, 128, seed=2)
    kc, vc, nk, nv = kc[:2], vc[:2], nk[:, :2], nv[:, :2]
    args = [to_dev(x) for x in (q, *pack(kc, 4), *pack(vc, 4), nk, nv)]
    assert run_with("tmem", lambda: kva.plan_kernel(*args, bits=4)) == "tcgen05"


@pytest.mark.parametrize("t", [1, 7, 8, 63, 127, 128, 129, 255, 256, 1000, 4096, 9000])
def test_lengths(native, t):
    q, kc, vc, nk, nv = cases.make_case(1, 8, max(t, 8), 128, seed=2000 + t)
    kc, vc = kc[:, :t], vc[:, :t]
    kc, vc, nk, nv = kc[:2], vc[:2], nk[:, :2], nv[:, :2]
    t_pad = -(-t // 8) * 8
    rng = np.random.default_rng(t)
    junk = rng.standard_normal((2, t_pad - t, 128)).astype(np.float16) * 30
    k_art = pack(np.concatenate([kc, junk], axis=1), 4)
    v_art = pack(np.concatenate([vc, junk], axis=1), 4)
    ours, gen = tmem_and_generic(lambda: run_decode(q, None, None, nk, nv, 4, t_cached=t, k_art=k_art,
                                                    v_art=v_art))
    v = judge_gqa(q, kc, vc, nk, nv, 4, ours)
    assert v.ok, (t, v)
    assert close(ours, gen)


@pytest.mark.parametrize("b,h,hkv,t", [(2, 8, 8, 700), (2, 8, 2, 1000), (3, 32, 8, 640),
                                        (1, 64, 8, 3000), (2, 12, 1, 500), (2, 6, 2, 384),
                                        (2, 28, 4, 1024)])
def test_gqa_ratios_and_head_tiles(native, b, h, hkv, t):
    q, kc, vc, nk, nv = cases.make_case(b, h, t, 128, seed=h * 31 + hkv + t)
    kc, vc, nk, nv = kc[:hkv], vc[:hkv], nk[:, :hkv], nv[:, :hkv]
    ours, gen = tmem_and_generic(lambda: run_decode(q, kc, vc, nk, nv, 4))
    v = judge_gqa(q, kc, vc, nk, nv, 4, ours)
    assert v.ok, v
    assert close(ours, gen)


def test_many_items_per_cta(native):
    """More work items than SMs: each persistent CTA walks several items,
    across item, Q-operand and tensor-memory buffer parities."""
    rng = np.random.default_rng(12)
    b, h, hkv, t = 40, 32, 8, 1200
    q = rng.standard_normal((b, h, 128)).astype(np.float16)
    kc = rng.standard_normal((b, hkv, t, 128)).astype(np.float16)
    vc = rng.standard_normal((b, hkv, t, 128)).astype(np.float16)
    nk = rng.standard_normal((b, hkv, 128)).astype(np.float16)
    nv = rng.standard_normal((b, hkv, 128)).astype(np.float16)
    ours, gen = tmem_and_generic(lambda: run_decode(q, kc, vc, nk, nv, 4))
    for v in judge_per_sequence(q, kc, vc, nk, nv, 4, ours, rows=[0, 13, 39]):
        assert v.ok, v
    assert close(ours, gen)


def test_per_sequence_ragged(native):
    rng = np.random.default_rng(9)
    b, h, hkv, t_pad = 7, 32, 8, 2048
    lens = np.array([0, 1, 100, 2048, 777, 1024, 129], dtype=np.int32)
    q = rng.standard_normal((b, h, 128)).astype(np.float16)
    kc = rng.standard_normal((b, hkv, t_pad, 128)).astype(np.float16)
    vc = rng.standard_normal((b, hkv, t_pad, 128)).astype(np.float16)
    nk = rng.standard_normal((b, hkv, 128)).astype(np.float16)
    nv = rng.standard_normal((b, hkv, 128)).astype(np.float16)
    ours, gen = tmem_and_generic(lambda: run_decode(q, kc, vc, nk, nv, 4, t_cached=int(lens.max()),
                                                    seq_lens=lens))
    # a zero-length row's softmax has only the step's own entry: out == new_v
    # exactly (the oracle's serial members need at least one position)
    r = h // hkv
    assert np.array_equal(ours[0], np.repeat(nv[0], r, axis=0))
    for v in judge_per_sequence(q, kc, vc, nk, nv, 4, ours, lens, rows=range(1, b)):
        assert v.ok, v
    assert close(ours, gen)


def test_t_split_shards(native):
    import torch
    from kernelverify_b200.pack import kv_attention as kva
    q, kc, vc, nk, nv = cases.make_case(1, 64, 4096, 128, seed=5)
    kc, vc, nk, nv = kc[:8], vc[:8], nk[:, :8], nv[:, :8]
    args = [to_dev(x) for x in (q, *pack(kc, 4), *pack(vc, 4), nk, nv)]
    bounds = [(0, 1000), (1000, 2048), (2048, 3072), (3072, 4096)]
    parts = run_with("tmem", lambda: [
        kva.decode_partial(*args, bits=4, t_begin=a, t_end=z, has_new_entry=(i == 3))
        for i, (a, z) in enumerate(bounds)])
    merged = kva.lse_merge(torch.stack([p[0] for p in parts]), torch.stack([p[1] for p in parts]),
                           torch.stack([p[2] for p in parts]), torch.float16).cpu().numpy()
    v = judge_gqa(q, kc, vc, nk, nv, 4, merged)
    assert v.ok, v


def test_outliers_and_large_q(native):
    """1 % of cache entries x20, and q scaled x40: wide scale/bias ranges and
    score magnitudes that move the softmax reference point often."""
    rng = np.random.default_rng(34)
    q = (rng.standard_normal((2, 32, 128)) * 40).astype(np.float16)
    nk, nv = (rng.standard_normal((2, 8, 128)).astype(np.float16) for _ in range(2))
    raw = rng.standard_normal((2, 2, 8, 1536, 128)).astype(np.float32)
    raw[rng.random(raw.shape) < 0.01] *= 20
    raw = raw.astype(np.float16)
    kc, vc = raw[0], raw[1]
    ours, gen = tmem_and_generic(lambda: run_decode(q, kc, vc, nk, nv, 4))
    for v in judge_per_sequence(q, kc, vc, nk, nv, 4, ours):
        assert v.ok, v


def test_repeat_calls_are_identical(native):
    """No state leaks between launches: the same step twice, bit for bit."""
    q, kc, vc, nk, nv = cases.make_case(4, 32, 2000, 128, seed=77)
    kc, vc, nk, nv = kc[:8], vc[:8], nk[:, :8], nv[:, :8]
    a = run_with("tmem", lambda: run_decode(q, kc, vc, nk, nv, 4))
    b = run_with("tmem", lambda: run_decode(q, kc, vc, nk, nv, 4))
    assert np.array_equal(a, b)
