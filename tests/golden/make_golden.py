"""Generate the golden fixtures that pin oracle/ to the reference itself.

Run in a container where the kernelverify reference tree is present:

    python tests/golden/make_golden.py --reference <path to kernelverify>

It imports the reference's own numpy code (quantizer, packing, fp64 kv
reference, tolerance, fault seams, battery) and writes:

* quant_golden.npz  -- canonical artefacts (packed words, scales, biases) and
  fp32 dequantized values for bits {2,3,4,6,8} x group {32,64,128} x storage
  dtype {fp16, fp32}, over rows built to hit the quantizer's edge rules.
* gate_golden.npz   -- fp64 reference outputs and tolerances of the six gate
  cases and of the reference's kv unit-test cases (fp32 dtype, every width,
  GQA by tiling, padded cache, T=1, new-entry dominance) plus group-32/128
  cases, with sha256 fingerprints of the inputs they were computed on.
* battery_golden.json -- for each of the 400 kv battery cases: input
  fingerprints, reference fingerprint, tolerance, the control verdict and the
  seven fault verdicts.

Nothing at run time reads the reference: tests compare oracle/ against these
files only.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def sha(a: np.ndarray) -> str:
    a = np.ascontiguousarray(a)
    h = hashlib.sha256()
    h.update(str(a.dtype).encode() + str(a.shape).encode())
    h.update(a.tobytes())
    return h.hexdigest()[:24]


def edge_rows(rng, dtype):
    """16 x 128 rows that exercise every branch of the quantizer."""
    rows = [rng.standard_normal(128) for _ in range(8)]
    rows.append(np.zeros(128))                               # degenerate: step 1e-7, bias 0
    rows.append(-np.abs(rng.standard_normal(128)) - 0.1)     # all negative: hi clamps to 0
    rows.append(np.full(128, 0.75))                          # constant positive
    rows.append(np.full(128, -1.25))                         # constant negative
    rows.append(rng.standard_normal(128) * 1e-9)             # below the 1e-7 step floor
    r = rng.standard_normal(128)
    r[rng.random(128) < 0.05] *= 20.0                        # outliers
    rows.append(r)
    rows.append(np.abs(rng.standard_normal(128)))            # all positive
    rows.append(rng.uniform(-10, 10, 128))                   # corpus range
    return np.stack(rows).astype(dtype)


def quant_golden(ref_mods):
    qc = ref_mods["quant_contract"]
    pack_codes = ref_mods["wide_qmv"].pack_codes
    rng = np.random.default_rng(2024)
    out = {}
    for dtype in ("float16", "float32"):
        w = edge_rows(rng, dtype)
        out[f"w_{dtype}"] = w
        for bits in (2, 3, 4, 6, 8):
            for g in (32, 64, 128):
                art = qc.canonical_quantize(w, qc.QuantContract(bits=bits, group_size=g))
                key = f"{dtype}_b{bits}_g{g}"
                out[f"words_{key}"] = pack_codes(art.q, bits)
                out[f"scales_{key}"] = art.scales
                out[f"biases_{key}"] = art.biases
                out[f"deq_{key}"] = qc.dequantize(art, np.float32)
    np.savez_compressed(HERE / "quant_golden.npz", **out)
    print(f"quant_golden.npz: {len(out)} arrays")


def gate_cases():
    """(label, builder) pairs; builders return (inputs-kwargs, dtype, extra)."""
    from oracle.cases import VERIFY_BITS, VERIFY_SHAPES, make_case

    cases = []
    for b, h, t, dh in VERIFY_SHAPES:                     # bench/pack_kv_attention.py:158-161
        for bits in VERIFY_BITS:
            cases.append((f"gate B={b} H={h} T={t} DH={dh} {bits}-bit",
                          dict(shape=(b, h, t, dh), seed=t + bits, bits=bits, dtype="float16")))
    for bits in (4, 8):                                   # tests/test_pack_kv_attention.py:82-91
        cases.append((f"fp32 dtype {bits}-bit",
                      dict(shape=(2, 4, 256, 128), seed=17 + bits, bits=bits, dtype="float32")))
    for bits in (2, 3, 4, 6, 8):                          # :94-102 (+6, which the build supports)
        cases.append((f"width {bits}-bit",
                      dict(shape=(1, 4, 128, 64), seed=40 + bits, bits=bits, dtype="float16")))
    cases.append(("single cached position",               # :133-140
                  dict(shape=(1, 2, 1, 64), seed=3, bits=4, dtype="float16")))
    cases.append(("new entry dominates",                  # :105-117
                  dict(shape=(2, 4, 128, 64), seed=5, bits=8, dtype="float16", dominate=True)))
    cases.append(("gqa 8:2 tiled",                        # :176-205
                  dict(shape=(1, 8, 128, 64), seed=31, bits=8, dtype="float16", hkv=2)))
    cases.append(("padded cache logical prefix",          # :143-173 (oracle side is unpadded)
                  dict(shape=(1, 4, 300, 128), seed=23, bits=8, dtype="float16")))
    for g in (32, 128):                                   # group extension
        for bits in (3, 4, 6):
            cases.append((f"group {g} {bits}-bit",
                          dict(shape=(2, 4, 96, 128), seed=70 + g + bits, bits=bits,
                               dtype="float16", group=g)))
    cases.append(("gqa 4:1 fp32 group 32",
                  dict(shape=(2, 8, 200, 128), seed=91, bits=4, dtype="float32", hkv=2, group=32)))
    return cases, make_case


def build_gate_inputs(spec, make_case):
    b, h, t, dh = spec["shape"]
    q, kc, vc, nk, nv = make_case(b, h, t, dh, seed=spec["seed"], dtype=spec["dtype"])
    if spec.get("dominate"):
        nk = (q.astype(np.float32) * 60.0).astype(np.float16)
    hkv = spec.get("hkv", h)
    if hkv != h:
        kc, vc, nk, nv = kc[:hkv], vc[:hkv], nk[:, :hkv], nv[:, :hkv]
    return q, kc, vc, nk, nv


def gate_golden(ref_mods):
    native_ops = ref_mods["native_ops"]
    nk_mod = ref_mods["native_kernels"]
    qc = ref_mods["quant_contract"]
    cases, make_case = gate_cases()
    real_dequant = nk_mod._cache_dequant
    out, meta = {}, []
    for i, (label, spec) in enumerate(cases):
        q, kc, vc, nk, nv = build_gate_inputs(spec, make_case)
        g = spec.get("group", 64)
        r = q.shape[1] // kc.shape[0]
        tile = (lambda a, ax: np.repeat(a, r, axis=ax)) if r > 1 else (lambda a, ax: a)
        inputs = {"q": q, "k_cache": tile(kc, 0), "v_cache": tile(vc, 0),
                  "new_k": tile(nk, 1), "new_v": tile(nv, 1),
                  "bits": np.array([spec["bits"]], dtype=np.int32)}

        # The reference's dequant fixes group 64; for the group extension the
        # same function is re-pointed at the reference's own quantizer and
        # dequantizer with the case's group.
        def grouped(cache, bits, fault=None, _g=g):
            hh, tt, dd = cache.shape
            art = qc.canonical_quantize(cache.reshape(hh * tt, dd),
                                        qc.QuantContract(bits=bits, group_size=_g))
            if fault is not None:
                art = fault(art)
            return qc.dequantize(art, np.float32).reshape(hh, tt, dd)

        nk_mod._cache_dequant = grouped if g != 64 else real_dequant
        native_ops._kv_dequant_memo.clear()
        try:
            op = native_ops.NATIVE_OPS["kv_attention"]
            ref = op.reference(inputs)

            class _C:
                dtype = spec["dtype"]
            tol = float(op.tolerance(_C, inputs, ref))
        finally:
            nk_mod._cache_dequant = real_dequant
            native_ops._kv_dequant_memo.clear()
        out[f"ref_{i}"] = ref
        meta.append({"label": label, **{k: v for k, v in spec.items()},
                     "tol": tol,
                     "input_sha": {n: sha(a) for n, a in
                                   zip(("q", "k_cache", "v_cache", "new_k", "new_v"),
                                       (q, kc, vc, nk, nv))}})
    out["meta_json"] = np.frombuffer(json.dumps(meta).encode(), dtype=np.uint8)
    np.savez_compressed(HERE / "gate_golden.npz", **out)
    print(f"gate_golden.npz: {len(meta)} cases")


def battery_golden(ref_mods):
    core = ref_mods["battery_core"]
    cat = ref_mods["catalogue"]
    native_ops = ref_mods["native_ops"]
    kernels = ref_mods["kernels"]
    me = ref_mods["measure_escape"]
    op = native_ops.NATIVE_OPS["kv_attention"]
    faults = [m for m in cat.CATALOGUE if m.kernel == "kv_attention"]
    records = []
    counts = {m.name: 0 for m in faults}
    for case in core.case_space(op.meta):
        inputs = core.make_mode_inputs(op.meta, case.dim_map, case.dtype, case.seed,
                                       case.distribution)
        inputs = op.augment(case, inputs)
        ref = op.reference(inputs)
        tol = float(op.tolerance(case, inputs, ref))
        control = bool(me.corpus_oracle_passes(kernels.KERNELS["kv_attention"](inputs), ref, tol))
        det = {}
        for m in faults:
            det[m.name] = not me.corpus_oracle_passes(m.build()(inputs), ref, tol)
            counts[m.name] += det[m.name]
        records.append({
            "dims": [list(p) for p in case.dims], "dtype": case.dtype,
            "distribution": case.distribution, "seed": case.seed,
            "input_sha": {n: sha(a) for n, a in inputs.items()},
            "ref_sha": sha(ref), "tol": tol, "control": control, "detected": det,
        })
    (HERE / "battery_golden.json").write_text(json.dumps(
        {"faults": [m.name for m in faults], "counts": counts, "cases": records}))
    print("battery_golden.json:", counts)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True)
    ap.add_argument("--only", choices=["quant", "gate", "battery"], default=None)
    args = ap.parse_args()
    sys.dont_write_bytecode = True  # the reference tree is read-only
    sys.path[:0] = [str(REPO), args.reference, str(Path(args.reference) / "bench")]
    import importlib
    names = {
        "quant_contract": "kernelverify.schemas.quant_contract",
        "wide_qmv": "kernelverify.pack.wide_qmv",
        "native_ops": "kernelverify.schemas.native_ops",
        "native_kernels": "kernelverify.reference.native_kernels",
        "kernels": "kernelverify.reference.kernels",
        "catalogue": "kernelverify.mutation.catalogue",
        "battery_core": "kernelverify.battery.core",
        "measure_escape": "measure_escape",
    }
    mods = {k: importlib.import_module(v) for k, v in names.items()}
    if args.only in (None, "quant"):
        quant_golden(mods)
    if args.only in (None, "gate"):
        gate_golden(mods)
    if args.only in (None, "battery"):
        battery_golden(mods)


if __name__ == "__main__":
    main()
