"""The 400-case kv_attention battery: schema, input modes, augment, validator.

Test infrastructure (see oracle/__init__.py). Reproduces the reference's case
space and inputs bit for bit so the CUDA path is judged on exactly the cases
the reference's mutation battery scores.
"""

from __future__ import annotations

import itertools
from dataclasses import dataclass

import numpy as np

# kernelverify/schemas/native_ops.py:258-280
KV_ATTENTION_META = {
    "op_schema": {
        "inputs": [
            {"name": "q", "dims": ["B", "H", "DH"]},
            {"name": "k_cache", "dims": ["H", "T", "DH"]},
            {"name": "v_cache", "dims": ["H", "T", "DH"]},
            {"name": "new_k", "dims": ["B", "H", "DH"]},
            {"name": "new_v", "dims": ["B", "H", "DH"]},
        ],
        "dims": [
            {"name": "B", "candidates": [1, 4]},
            {"name": "H", "candidates": [2, 8]},
            {"name": "T", "candidates": [64, 512]},
            {"name": "DH", "candidates": [64, 128]},
            {"name": "BITS", "candidates": [4, 8]},
        ],
    },
    "dtypes": ["float32", "float16"],
    "tolerances": {"float32": 1e-3, "float16": 1e-2},
}

QUERY_SCALE = 0.6          # kernelverify/schemas/native_ops.py:282
SWEEP_SEED = 1234          # kernelverify/battery/core.py:76
BENCHMARK_SEEDS = 8        # kernelverify/battery/core.py:75

# bench/measure_escape.py:67-70; kernelverify/battery/core.py:95-98
DISTRIBUTIONS = {
    "corpus uniform[-10,10]": (-10.0, 10.0),
    "unit-scale uniform[-1,1]": (-1.0, 1.0),
}
CORPUS_MODE = "corpus uniform[-10,10]"
IID_MODES = ("corpus uniform[-10,10]", "unit-scale uniform[-1,1]")
INPUT_MODES = IID_MODES + ("opposed signs", "near zero", "constant rows")
_NP = {"float16": np.float16, "float32": np.float32}


@dataclass(frozen=True)
class Case:
    dims: tuple          # sorted (name, value) pairs
    dtype: str
    distribution: str
    seed: int

    @property
    def dim_map(self) -> dict:
        return dict(self.dims)


def all_dims(meta: dict):
    """Every schema combination (bench/measure_escape.py:199-203)."""
    names = [d["name"] for d in meta["op_schema"]["dims"]]
    for combo in itertools.product(*[d["candidates"] for d in meta["op_schema"]["dims"]]):
        yield dict(zip(names, combo))


def benchmark_dims(meta: dict) -> dict:
    """Largest power-of-two candidate per dim (bench/measure_escape.py:184-196)."""
    chosen = {}
    for dim in meta["op_schema"]["dims"]:
        cands = sorted(dim["candidates"])
        pows = [c for c in cands if c >= 2 and (c & (c - 1)) == 0]
        chosen[dim["name"]] = pows[-1] if pows else cands[-1]
    return chosen


def case_space(meta: dict = KV_ATTENTION_META) -> list:
    """Schema sweep at SWEEP_SEED plus BENCHMARK_SEEDS draws at the benchmark
    shape, every dtype and mode, deduplicated and sorted
    (kernelverify/battery/core.py:140-160)."""
    cases = []
    for dims in all_dims(meta):
        key = tuple(sorted(dims.items()))
        for dtype in meta["dtypes"]:
            for mode in INPUT_MODES:
                cases.append(Case(key, dtype, mode, SWEEP_SEED))
    bench_key = tuple(sorted(benchmark_dims(meta).items()))
    for dtype in meta["dtypes"]:
        for mode in INPUT_MODES:
            for seed in range(BENCHMARK_SEEDS):
                cases.append(Case(bench_key, dtype, mode, seed))
    return sorted(set(cases), key=lambda c: (c.dims, c.dtype, c.distribution, c.seed))


def make_inputs(meta, dims, dtype, seed, distribution) -> dict:
    """Uniform draws per schema input, in schema order, from one generator
    (bench/measure_escape.py:83-94)."""
    low, high = DISTRIBUTIONS[distribution]
    rng = np.random.default_rng(seed)
    out = {}
    for spec in meta["op_schema"]["inputs"]:
        shape = [dims[d] for d in spec["dims"]]
        data = rng.random(int(np.prod(shape))) * (high - low) + low
        out[spec["name"]] = data.reshape(shape).astype(_NP[dtype])
    return out


def make_mode_inputs(meta, dims, dtype, seed, mode) -> dict:
    """The five input modes (kernelverify/battery/core.py:104-122)."""
    if mode in IID_MODES:
        return make_inputs(meta, dims, dtype, seed, mode)
    base = make_inputs(meta, dims, dtype, seed, CORPUS_MODE)
    if mode == "opposed signs":
        return {name: (np.abs(a) if i % 2 == 0 else -np.abs(a)).astype(a.dtype)
                for i, (name, a) in enumerate(base.items())}
    if mode == "near zero":
        return {name: (a * np.float32(1e-3)).astype(a.dtype) for name, a in base.items()}
    if mode == "constant rows":
        return {name: np.ascontiguousarray(np.broadcast_to(a[..., :1], a.shape)).astype(a.dtype)
                for name, a in base.items()}
    raise ValueError(f"unknown input mode: {mode}")


def rescaled(arr: np.ndarray, target_peak: float) -> np.ndarray:
    """Scale to a peak magnitude, all-zero left alone
    (kernelverify/schemas/native_ops.py:138-142)."""
    peak = float(np.max(np.abs(arr.astype(np.float32)))) if arr.size else 0.0
    if peak == 0.0:
        return arr
    return (arr.astype(np.float32) * (target_peak / peak)).astype(arr.dtype)


def kv_augment(case: Case, inputs: dict) -> dict:
    """bits from the case; q and new_k rescaled to QUERY_SCALE
    (kernelverify/schemas/native_ops.py:286-290)."""
    inputs["bits"] = np.array([case.dim_map["BITS"]], dtype=np.int32)
    inputs["q"] = rescaled(inputs["q"], QUERY_SCALE)
    inputs["new_k"] = rescaled(inputs["new_k"], QUERY_SCALE)
    return inputs


def case_inputs(case: Case) -> dict:
    """The augmented native-op inputs of one battery case."""
    inputs = make_mode_inputs(KV_ATTENTION_META, case.dim_map, case.dtype,
                              case.seed, case.distribution)
    return kv_augment(case, inputs)


def corpus_oracle_passes(candidate, ref, tol: float) -> bool:
    """Shape, finiteness, then max-abs <= tol (bench/measure_escape.py:166-174)."""
    if candidate.shape != ref.shape:
        return False
    a = candidate.astype(np.float64)
    if not np.all(np.isfinite(a)):
        return False
    return bool(np.all(np.abs(a - ref.astype(np.float64)) <= tol))
