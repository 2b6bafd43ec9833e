"""MLX-affine quantization artefacts: quantize, pack, unpack, dequantize.

Test infrastructure (see oracle/__init__.py). Each function restates one step
of the reference and cites where that step lives.
"""

from __future__ import annotations

import numpy as np

_TINY_STEP = np.float32(1e-7)
_HALF = np.float32(0.5)


def round_half_away(x: np.ndarray) -> np.ndarray:
    """fp32 round-half-away-from-zero: sign(x) * floor(|x| + 0.5), the add at
    fp32 (kernelverify/schemas/quant_contract.py:55-57)."""
    return np.sign(x) * np.floor(np.abs(x) + _HALF)


def canonical_quantize(w: np.ndarray, bits: int, group_size: int = 64):
    """(codes int32 [rows, cols], scales [rows, cols/g], biases [rows, cols/g]).

    The MLX-affine quantizer as the reference states it
    (kernelverify/schemas/quant_contract.py:60-104), every step in fp32:

    1. per group: lo = min(w), hi = max(max(w), 0)              (:85-86)
    2. step = max((hi - lo) / (2^bits - 1), 1e-7)                 (:88)
    3. the dominant edge decides the sign: when |lo| > |hi| the
       step stays positive and the edge is lo, else the step is
       negated and the edge is hi                                  (:89-91)
    4. n = round_half_away(edge / step); when n != 0 the step is
       snapped to edge / n and the bias is the edge, else bias 0   (:92-95)
    5. codes = min(round_half_away((w - bias) / step), 2^bits - 1) (:97-98)
    6. scales and biases are stored in w's dtype (fp16 caches give
       fp16 scales, fp32 caches fp32 scales)                       (:99-104)
    """
    rows, cols = w.shape
    if cols % group_size:
        raise ValueError(f"row length {cols} is not a multiple of group {group_size}")
    top = np.float32((1 << bits) - 1)
    grp = w.astype(np.float32).reshape(rows, cols // group_size, group_size)
    lo = grp.min(axis=2)
    hi = np.maximum(grp.max(axis=2), np.float32(0.0))

    step = np.maximum((hi - lo) / top, _TINY_STEP)
    low_side = np.abs(lo) > np.abs(hi)
    step = np.where(low_side, step, -step).astype(np.float32)
    edge = np.where(low_side, lo, hi).astype(np.float32)
    n_edge = round_half_away((edge / step).astype(np.float32))
    degenerate = n_edge == 0.0
    safe_n = np.where(degenerate, np.float32(1.0), n_edge)
    step = np.where(degenerate, step, (edge / safe_n).astype(np.float32))
    bias = np.where(degenerate, np.float32(0.0), edge)

    codes = round_half_away(((grp - bias[:, :, None]) / step[:, :, None]).astype(np.float32))
    codes = np.minimum(codes, top).astype(np.int32).reshape(rows, cols)
    return codes, step.astype(w.dtype), bias.astype(w.dtype)


def pack_codes(codes: np.ndarray, bits: int) -> np.ndarray:
    """uint32 words [rows, cols*bits/32]: one contiguous little-endian bit
    stream per row, code i at stream bit i*bits, lowest code in the lowest
    bits (kernelverify/pack/wide_qmv.py:185-201). 3- and 6-bit codes straddle
    word boundaries."""
    rows, cols = codes.shape
    total = cols * bits
    if total % 32:
        raise ValueError(f"{cols} codes of {bits} bits do not fill whole words")
    n_words = total // 32
    words = np.zeros((rows, n_words + 1), dtype=np.uint64)
    c = codes.astype(np.uint64)
    for i in range(cols):
        bit = i * bits
        w, sh = bit >> 5, bit & 31
        words[:, w] |= (c[:, i] << np.uint64(sh)) & np.uint64(0xFFFFFFFF)
        if sh + bits > 32:
            words[:, w + 1] |= c[:, i] >> np.uint64(32 - sh)
    return words[:, :n_words].astype(np.uint32)


def unpack_codes(words: np.ndarray, bits: int, cols: int) -> np.ndarray:
    """Inverse of `pack_codes`: int32 codes [rows, cols]."""
    rows = words.shape[0]
    w64 = np.concatenate([words.astype(np.uint64),
                          np.zeros((rows, 1), dtype=np.uint64)], axis=1)
    mask = np.uint64((1 << bits) - 1)
    out = np.empty((rows, cols), dtype=np.int32)
    for i in range(cols):
        bit = i * bits
        w, sh = bit >> 5, bit & 31
        window = w64[:, w] | (w64[:, w + 1] << np.uint64(32))
        out[:, i] = ((window >> np.uint64(sh)) & mask).astype(np.int32)
    return out


def dequantize(codes: np.ndarray, scales: np.ndarray, biases: np.ndarray,
               group_size: int = 64, dtype=np.float64) -> np.ndarray:
    """scale * code + bias per group at `dtype`: a rounded multiply followed
    by a rounded add, never a fused multiply-add
    (kernelverify/schemas/quant_contract.py:107-113)."""
    rows, cols = codes.shape
    grp = codes.reshape(rows, cols // group_size, group_size).astype(dtype)
    out = scales.astype(dtype)[:, :, None] * grp + biases.astype(dtype)[:, :, None]
    return out.reshape(rows, cols)


def quantize_cache(cache: np.ndarray, bits: int, group_size: int = 64):
    """Packed artefact triplet for an (H, T, DH) cache, quantized as the (H*T,
    DH) reshape (kernelverify/pack/kv_attention.py:270-283; the group size is a
    parameter here where the reference fixes 64). Returns
    (words [H, T, DH*bits/32] uint32, scales [H, T, DH/g], biases [H, T, DH/g])."""
    h, t, dh = cache.shape
    codes, scales, biases = canonical_quantize(cache.reshape(h * t, dh), bits, group_size)
    words = pack_codes(codes, bits).reshape(h, t, dh * bits // 32)
    g = dh // group_size
    return words, scales.reshape(h, t, g), biases.reshape(h, t, g)
