"""Seeded case makers: the gate's `make_case` and the BASELINE configs.

Test infrastructure (see oracle/__init__.py).
"""

from __future__ import annotations

import numpy as np

# bench/pack_kv_attention.py:65-66 -- (B, H, T, DH) x bits, the 6 gate cases
VERIFY_SHAPES = [(1, 8, 512, 128), (4, 2, 64, 64), (1, 4, 300, 128)]
VERIFY_BITS = (4, 8)


def make_case(b, h, t, dh, seed, dtype="float16"):
    """q and new_k at peak 0.6, caches and new_v N(0,1), one generator in the
    reference's draw order (bench/pack_kv_attention.py:75-88)."""
    rng = np.random.default_rng(seed)

    def peaked(shape):
        a = rng.standard_normal(shape).astype(np.float32)
        return (a * (0.6 / float(np.max(np.abs(a))))).astype(dtype)

    q, new_k = peaked((b, h, dh)), peaked((b, h, dh))
    k_cache = rng.standard_normal((h, t, dh)).astype(dtype)
    v_cache = rng.standard_normal((h, t, dh)).astype(dtype)
    new_v = rng.standard_normal((b, h, dh)).astype(dtype)
    return q, k_cache, v_cache, new_k, new_v


# BASELINE.json configs, as plain parameters (inputs are seeded synthetic
# draws with the configs' shapes and distributions; the reference measures on
# no public dataset for this path).
CONFIGS = {
    1: dict(name="cpu-oracle", B=1, H=8, HKV=2, DH=128, T=2048, bits=4, group=64),
    2: dict(name="llama3-8b-decode", B=32, H=32, HKV=8, DH=128, T=8192, bits=4, group=64),
    3: dict(name="bits-group-sweep", B=16, H=32, HKV=8, DH=128, T=16384,
            bits=(2, 3, 4, 6, 8), group=(32, 64, 128), outliers=0.01),
    4: dict(name="ragged-8bit", B=64, H=28, HKV=4, DH=128, T=(256, 32768), bits=8, group=64),
    5: dict(name="long-context-tsplit", B=1, H=64, HKV=8, DH=128, T=131072, bits=4, group=64),
}


def ragged_lengths(b: int = 64, lo: int = 256, hi: int = 32768, seed: int = 0) -> np.ndarray:
    """Per-sequence cached lengths of config 4, inclusive U[lo, hi]
    (seed 0: sum 1,077,211, min 345, max 32678)."""
    return np.random.default_rng(seed).integers(lo, hi, b, endpoint=True)


def draw_sequence(rng, h, hkv, t, dh, dtype="float16", outliers: float = 0.0):
    """One sequence's raw step inputs: q [1,H,DH] and new_k/new_v [1,HKV,DH]
    N(0,1) fp16, caches [HKV,T,DH] N(0,1) drawn fp32 and cast to the storage
    dtype before quantizing; with `outliers`, that fraction of cache entries
    (seeded mask) is scaled x20."""
    q = rng.standard_normal((1, h, dh)).astype(dtype)
    k = rng.standard_normal((hkv, t, dh)).astype(np.float32)
    v = rng.standard_normal((hkv, t, dh)).astype(np.float32)
    if outliers:
        k = np.where(rng.random(k.shape) < outliers, k * 20.0, k)
        v = np.where(rng.random(v.shape) < outliers, v * 20.0, v)
    new_k = rng.standard_normal((1, hkv, dh)).astype(dtype)
    new_v = rng.standard_normal((1, hkv, dh)).astype(dtype)
    return q, k.astype(dtype), v.astype(dtype), new_k, new_v
