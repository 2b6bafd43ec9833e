"""The fp32 numpy port of the operator with its seven fault seams.

Test infrastructure (see oracle/__init__.py). `kv_attention(inputs)` is the
battery's control (the correct port); each catalogue entry switches on one
seam (kernelverify/reference/native_kernels.py:168-221,
kernelverify/mutation/catalogue.py:153-166).
"""

from __future__ import annotations

import functools

import numpy as np

from oracle.kv import cache_dequant, group_of


def scales_rotated(codes, scales, biases):
    """Every group reads its neighbour's scale and bias
    (kernelverify/schemas/quant_contract.py:253-256)."""
    return codes, np.roll(scales, 1, axis=1), np.roll(biases, 1, axis=1)


def bias_dropped(codes, scales, biases):
    """The affine bias is discarded (kernelverify/schemas/quant_contract.py:265-267)."""
    return codes, scales, np.zeros_like(biases)


def kv_attention(inputs, *, scores_dtype="float32", accum_dtype="float32",
                 k_scales_rotated=False, v_bias_dropped=False,
                 new_entry_skipped=False, dhead_scale_dropped=False):
    """One decode step at fp32 over the canonical artefacts, with seams
    (kernelverify/reference/native_kernels.py:168-221)."""
    bits, g = int(inputs["bits"][0]), group_of(inputs)
    kd = cache_dequant(inputs["k_cache"], bits, g, scales_rotated if k_scales_rotated else None)
    vd = cache_dequant(inputs["v_cache"], bits, g, bias_dropped if v_bias_dropped else None)
    return attend_dequantized(inputs["q"], kd, vd, inputs["new_k"], inputs["new_v"],
                              scores_dtype=scores_dtype, accum_dtype=accum_dtype,
                              new_entry_skipped=new_entry_skipped,
                              dhead_scale_dropped=dhead_scale_dropped)


def attend_dequantized(q, kd, vd, new_k, new_v, *, scores_dtype="float32", accum_dtype="float32",
                       new_entry_skipped=False, dhead_scale_dropped=False):
    """The port's attention arithmetic over already dequantized fp32 caches
    kd/vd [H, T, DH] (kernelverify/reference/native_kernels.py:178-221): the
    part of a step that remains once the artefacts are decoded."""
    dh = q.shape[-1]
    qf = q.astype(np.float32)
    scale = 1.0 if dhead_scale_dropped else 1.0 / np.sqrt(np.float32(dh))
    scores = np.einsum("bhd,htd->bht", qf, kd) * scale
    s_new = np.sum(qf * new_k.astype(np.float32), axis=-1) * scale
    if not new_entry_skipped:
        scores = np.concatenate([scores, s_new[..., None]], axis=-1)
    if scores_dtype != "float32":
        scores = scores.astype(scores_dtype).astype(np.float32)

    probs = np.exp(scores - scores.max(axis=-1, keepdims=True))
    probs /= probs.sum(axis=-1, keepdims=True)
    pc = probs[..., : kd.shape[1]]
    if accum_dtype in ("float16", "float16-seq"):
        contrib = pc.astype(np.float16)[..., None] * vd.astype(np.float16)[None, ...]
        if accum_dtype == "float16-seq":
            out = np.add.accumulate(contrib, axis=2, dtype=np.float16)[:, :, -1]
        else:
            out = np.add.reduce(contrib, axis=2, dtype=np.float16)
        out = out.astype(np.float32)
    else:
        out = np.einsum("bht,htd->bhd", pc, vd)
    if not new_entry_skipped:
        out = out + probs[..., -1][..., None] * new_v.astype(np.float32)
    return out.astype(q.dtype)


# (name, seam keywords) -- the reference's Mutation.name is "kernel[k=v]"
# (kernelverify/mutation/catalogue.py:43-46,153-166).
KV_FAULTS = [
    {"scores_dtype": "float16"},
    {"accum_dtype": "float16"},
    {"accum_dtype": "float16-seq"},
    {"k_scales_rotated": True},
    {"v_bias_dropped": True},
    {"new_entry_skipped": True},
    {"dhead_scale_dropped": True},
]


def fault_name(params: dict) -> str:
    args = ", ".join(f"{k}={v}" for k, v in params.items())
    return f"kv_attention[{args}]"


def faulty(params: dict):
    return functools.partial(kv_attention, **params)
