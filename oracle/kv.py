"""fp64 reference, fp32 ensemble, floored tolerance and judge for kv decode.

Test infrastructure (see oracle/__init__.py). An `inputs` dict has the
reference's native-op form (kernelverify/pack/verify.py:84-95): RAW float
caches `k_cache`/`v_cache` [H, T, DH] (the oracle quantizes them itself, so a
surface cannot hand it an artefact that disagrees with the one it packed),
`q`/`new_k`/`new_v` [B, H, DH] and `bits` (an int32 array of one element).
`group_size` is an optional extra key (default 64, the reference's fixed
group); groups other than 64 are the one extension the reference's functions
do not take as a parameter (its dequant hard-codes 64 at
kernelverify/reference/native_kernels.py:162).
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from oracle.quant import canonical_quantize, dequantize

# kernelverify/schemas/native_ops.py:42,45
K_QUANT = 4.0
EPS = {"float16": 9.77e-4, "float32": 1.19e-7}


def base_tol(dtype: str, ref: np.ndarray) -> float:
    """4 * eps(dtype) * max|ref| (kernelverify/schemas/native_ops.py:48-50)."""
    scale = float(np.max(np.abs(ref))) if ref.size else 0.0
    return 4.0 * EPS[dtype] * scale


def max_abs_error(candidate, ref) -> float:
    """fp64 max |candidate - ref|, 0 on empty (kernelverify/tolerance/floor.py:76-82)."""
    diff = np.abs(np.asarray(candidate).astype(np.float64) - np.asarray(ref).astype(np.float64))
    return float(np.max(diff)) if diff.size else 0.0


def floored_tolerance(base: float, k: float, member_outputs, ref) -> float:
    """max(base, k * worst member error) (kernelverify/tolerance/floor.py:85-89)."""
    return max(base, k * max(max_abs_error(out, ref) for out in member_outputs))


def group_of(inputs: dict) -> int:
    return int(inputs.get("group_size", 64))


def cache_dequant(cache: np.ndarray, bits: int, group_size: int = 64,
                  fault=None) -> np.ndarray:
    """Quantize an (H, T, DH) cache as its (H*T, DH) reshape and dequantize at
    fp32 (kernelverify/reference/native_kernels.py:153-165). `fault`, when
    given, corrupts the artefact (codes, scales, biases) before dequant."""
    h, t, dh = cache.shape
    codes, scales, biases = canonical_quantize(cache.reshape(h * t, dh), bits, group_size)
    if fault is not None:
        codes, scales, biases = fault(codes, scales, biases)
    return dequantize(codes, scales, biases, group_size, np.float32).reshape(h, t, dh)


# Two-slot identity memo: the reference and the four members dequantize the
# same two caches per case (kernelverify/schemas/native_ops.py:298-311).
_memo: dict = {}


def dequant64(cache: np.ndarray, bits: int, group_size: int = 64) -> np.ndarray:
    key = (id(cache), int(bits), int(group_size))
    hit = _memo.get(key)
    if hit is not None and hit[0] is cache:
        return hit[1]
    if len(_memo) >= 2:
        _memo.clear()
    value = cache_dequant(cache, bits, group_size).astype(np.float64)
    _memo[key] = (cache, value)
    return value


def kv_reference(inputs: dict) -> np.ndarray:
    """fp64 truth [B, H, DH] (kernelverify/schemas/native_ops.py:314-329):
    cached K/V are the artefacts' dequantized values, the step's own new entry
    enters at full precision, scores * 1/sqrt(DH), max-shifted softmax over
    T+1, then the combine."""
    q = inputs["q"].astype(np.float64)
    bits, g = int(inputs["bits"][0]), group_of(inputs)
    kd = dequant64(inputs["k_cache"], bits, g)
    vd = dequant64(inputs["v_cache"], bits, g)
    scale = 1.0 / np.sqrt(float(q.shape[-1]))
    scores = np.einsum("bhd,htd->bht", q, kd) * scale
    s_new = np.sum(q * inputs["new_k"].astype(np.float64), axis=-1) * scale
    scores = np.concatenate([scores, s_new[..., None]], axis=-1)
    probs = np.exp(scores - scores.max(axis=-1, keepdims=True))
    probs /= probs.sum(axis=-1, keepdims=True)
    out = np.einsum("bht,htd->bhd", probs[..., :-1], vd)
    return out + probs[..., -1][..., None] * inputs["new_v"].astype(np.float64)


def kv_member(inputs: dict, *, scores_order: str = "pairwise",
              combine_order: str = "pairwise") -> np.ndarray:
    """One legitimate fp32 implementation; the two knobs pick the reduction
    order of the scores and of the combine
    (kernelverify/schemas/native_ops.py:332-359)."""
    q = inputs["q"].astype(np.float32)
    bits, g = int(inputs["bits"][0]), group_of(inputs)
    kd = dequant64(inputs["k_cache"], bits, g).astype(np.float32)
    vd = dequant64(inputs["v_cache"], bits, g).astype(np.float32)
    scale = np.float32(1.0 / np.sqrt(float(q.shape[-1])))
    if scores_order == "serial":
        prods = q[:, :, None, :] * kd[None, :, :, :]
        scores = np.add.accumulate(prods, axis=-1, dtype=np.float32)[..., -1] * scale
    else:
        scores = np.einsum("bhd,htd->bht", q, kd) * scale
    s_new = np.sum(q * inputs["new_k"].astype(np.float32), axis=-1) * scale
    scores = np.concatenate([scores, s_new[..., None]], axis=-1)
    probs = np.exp(scores - scores.max(axis=-1, keepdims=True))
    probs /= probs.sum(axis=-1, keepdims=True)
    pc = probs[..., :-1]
    if combine_order in ("serial", "reversed"):
        contrib = pc[..., None] * vd[None, ...]
        if combine_order == "reversed":
            contrib = contrib[:, :, ::-1, :]
        out = np.add.accumulate(contrib, axis=2, dtype=np.float32)[:, :, -1]
    else:
        out = np.einsum("bht,htd->bhd", pc, vd)
    out = out + probs[..., -1][..., None] * inputs["new_v"].astype(np.float32)
    return out.astype(inputs["q"].dtype)


# kernelverify/schemas/native_ops.py:362-367 (labels are part of the identity)
KV_MEMBERS = {
    "kv:pairwise-pairwise": dict(scores_order="pairwise", combine_order="pairwise"),
    "kv:serial-scores": dict(scores_order="serial", combine_order="pairwise"),
    "kv:serial-combine": dict(scores_order="pairwise", combine_order="serial"),
    "kv:reversed-combine": dict(scores_order="pairwise", combine_order="reversed"),
}


def kv_tolerance(dtype: str, inputs: dict, ref: np.ndarray) -> float:
    """max(4*eps(dtype)*max|ref|, K_QUANT * worst member error); K_QUANT = 4.0
    is borrowed from the quantized-matmul calibration, never calibrated over
    KV_MEMBERS (kernelverify/schemas/native_ops.py:376-394)."""
    return floored_tolerance(base_tol(dtype, ref), K_QUANT,
                             (kv_member(inputs, **kw) for kw in KV_MEMBERS.values()), ref)


@dataclass(frozen=True)
class Verdict:
    ok: bool
    err: float
    tol: float
    ref_max: float = 0.0     # max|ref|: err / ref_max is the max-rel error

    @property
    def rel(self) -> float:
        """max |candidate - ref| / max|ref| (0 when the reference is all zero)."""
        return self.err / self.ref_max if self.ref_max > 0 else 0.0

    def __str__(self) -> str:
        return (f"err {self.err:9.3e}  rel {self.rel:9.3e}  tol {self.tol:9.3e}  "
                f"{'pass' if self.ok else 'FAIL'}")


def kv_inputs(q, k_cache, v_cache, new_k, new_v, bits: int, group_size: int = 64) -> dict:
    """Native-op inputs from RAW caches (kernelverify/pack/verify.py:84-95)."""
    inputs = {"q": q, "k_cache": k_cache, "v_cache": v_cache, "new_k": new_k,
              "new_v": new_v, "bits": np.array([bits], dtype=np.int32)}
    if group_size != 64:
        inputs["group_size"] = group_size
    return inputs


def reference_and_tolerance(inputs: dict, dtype: str = "float16"):
    """(fp64 reference, tolerance) for one case (kernelverify/pack/verify.py:98-105)."""
    ref = kv_reference(inputs)
    return ref, float(kv_tolerance(dtype, inputs, ref))


def judge(candidate, ref: np.ndarray, tol: float) -> Verdict:
    """Max-abs error at fp64 against tol (kernelverify/pack/verify.py:108-111)."""
    err = max_abs_error(candidate, ref)
    ref_max = float(np.max(np.abs(ref))) if np.size(ref) else 0.0
    return Verdict(ok=err <= tol, err=err, tol=tol, ref_max=ref_max)


def verify_output(inputs: dict, candidate, dtype: str = "float16") -> Verdict:
    """One-step gate (kernelverify/pack/verify.py:114-118)."""
    ref, tol = reference_and_tolerance(inputs, dtype)
    return judge(candidate, ref, tol)


def max_rel_error(candidate, ref) -> float:
    """max |candidate - ref| / max|ref| -- the relative figure reported beside
    max-abs for fp16 outputs (not part of the reference's verdict)."""
    scale = float(np.max(np.abs(ref))) if np.size(ref) else 0.0
    return max_abs_error(candidate, ref) / scale if scale else 0.0


# ---------------------------------------------------------------------------
# GQA, per-sequence and ragged cases, judged through the shared-cache oracle.
# ---------------------------------------------------------------------------
def gqa_tiled_inputs(q, k_cache, v_cache, new_k, new_v, bits, group_size=64) -> dict:
    """The reference has no GQA form: tile each cache head and new_k/new_v row
    r = H/HKV times along the head axis (contiguous-block mapping h -> h // r,
    kernelverify/pack/kv_attention.py:99-103). Quantization is per row, so the
    tiled case's artefact is the untiled one repeated and the answer is exact
    (the reference's own argument, tests/test_pack_kv_attention.py:176-205)."""
    r = q.shape[1] // k_cache.shape[0]
    return kv_inputs(q, np.repeat(k_cache, r, axis=0), np.repeat(v_cache, r, axis=0),
                     np.repeat(new_k, r, axis=1), np.repeat(new_v, r, axis=1),
                     bits, group_size)
