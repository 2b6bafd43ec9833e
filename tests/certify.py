"""Emit certificates for the library's kv_attn_decode specializations (test
infrastructure: it judges with the oracle). Needs a CUDA device.

    python tests/certify.py --out certificates [--bits 4 8] [--dh 64 128]

KVQ_HARNESS_COMMIT names the commit of this tree when it is not a git checkout
(a copy on a GPU host).

Protocol per (bits, head_dim), fp16: the reference's three gate shapes
(bench/pack_kv_attention.py:65-66) restricted to that head_dim, seeded
t + bits (pack_kv_attention.py:161), plus two extension cases that exercise
what the reference gate cannot: grouped queries (32 query / 8 cache heads,
per-sequence caches) and a cache past the reference's T <= 1024 capacity. Each
case runs through the public decode call and is judged against the fp64
reference within the shipped tolerance.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from kernelverify_b200 import certificate as C  # noqa: E402
from oracle import cases, kv  # noqa: E402
from tests.kvq_cases import judge_gqa, judge_per_sequence, pack, run_decode  # noqa: E402

POLICY = ("gate fixed-case sweep: the reference's gate shapes at this head_dim "
          "(seed t + bits) + a grouped-query per-sequence case and a T > 1024 case")
SEEDS = ("gate: np.random.default_rng(t + bits) per shape in make_case(), q and new_k at "
         "peak 0.6; extensions: np.random.default_rng(9000 + bits) (grouped, per-sequence) "
         "and make_case(seed=7000 + bits) (long T)")


def _kernel_for(bits, dh, r, t_stride) -> str:
    """The kernel the library plans for an fp16 case of this shape (see
    kvq_plan_kernel): the register-fragment tensor-core kernels at head_dim
    128, at most 8 query heads per cache head and 8-row-aligned geometry."""
    tc = dh == 128 and r <= 8 and t_stride % 8 == 0
    if not tc:
        return "CUDA-core"
    return ("tensor-core (mma.sync, register fragments)" if bits == 4 else
            "tensor-core (mma.sync, byte codes)")


def _evidence(label, verdict, out, kernel) -> C.CaseEvidence:
    return C.CaseEvidence(label=label, passed=bool(verdict.ok), err=float(verdict.err),
                          tol=float(verdict.tol),
                          output_sha256=hashlib.sha256(np.ascontiguousarray(out).tobytes()).hexdigest(),
                          kernel=kernel, ref_max=float(verdict.ref_max))


def protocol_cases(bits: int, dh: int):
    """The protocol's cases in order: (label, kind, (q, k_cache, v_cache,
    new_k, new_v), kernel); kind "shared" is one cache for the batch (judged
    as one case), "per-sequence" one cache per sequence (judged per
    sequence). Host-only: seeded numpy inputs."""
    for (b, h, t, d) in cases.VERIFY_SHAPES:
        if d != dh:
            continue
        yield (f"gate B={b} H={h} T={t} DH={d} {bits}-bit", "shared",
               cases.make_case(b, h, t, d, seed=t + bits), _kernel_for(bits, d, 1, t))
    # grouped queries, per-sequence caches
    rng = np.random.default_rng(9000 + bits)
    b, h, hkv, t = 2, 32, 8, 1024
    q = rng.standard_normal((b, h, dh)).astype(np.float16)
    kc = rng.standard_normal((b, hkv, t, dh)).astype(np.float16)
    vc = rng.standard_normal((b, hkv, t, dh)).astype(np.float16)
    nk = rng.standard_normal((b, hkv, dh)).astype(np.float16)
    nv = rng.standard_normal((b, hkv, dh)).astype(np.float16)
    yield (f"grouped B=2 H=32 HKV=8 T=1024 DH={dh} {bits}-bit per-sequence", "per-sequence",
           (q, kc, vc, nk, nv), _kernel_for(bits, dh, 4, t))
    # past the reference's capacity
    yield (f"long B=1 H=4 T=5000 DH={dh} {bits}-bit", "shared",
           cases.make_case(1, 4, 5000, dh, seed=7000 + bits), _kernel_for(bits, dh, 1, 5000))


def run_protocol(bits: int, dh: int) -> list:
    evidence = []
    for label, kind, (q, kc, vc, nk, nv), kernel in protocol_cases(bits, dh):
        out = run_decode(q, kc, vc, nk, nv, bits)
        if kind == "shared":
            v = judge_gqa(q, kc, vc, nk, nv, bits, out)
        else:
            verdicts = judge_per_sequence(q, kc, vc, nk, nv, bits, out)
            worst = max(verdicts, key=lambda x: x.err / x.tol)
            v = type(worst)(all(x.ok for x in verdicts), worst.err, worst.tol, worst.ref_max)
        evidence.append(_evidence(label, v, out, kernel))
    return evidence


def certify(bits: int, dh: int) -> C.Certificate:
    import torch
    commit = os.environ.get("KVQ_HARNESS_COMMIT") or subprocess.run(
        ["git", "-C", str(ROOT), "rev-parse", "--short", "HEAD"],
        capture_output=True, text=True).stdout.strip() or "unknown"
    ev = run_protocol(bits, dh)
    n_gate = sum(1 for s in cases.VERIFY_SHAPES if s[3] == dh)
    return C.Certificate(
        bits=bits, head_dim=dh, dtype="float16", policy=POLICY, seed_protocol=SEEDS,
        cases=ev, clauses=C.contract_clauses("contract"), precision="contract",
        translation_unit=C.translation_unit_sha256(), library=C.library_sha256(),
        flags=C.build_flags(), chip=torch.cuda.get_device_name(0), toolchain=C.toolchain(),
        harness_commit=commit, budget=n_gate + 2,
        domain={"BITS": bits, "DH": dh, "dtype": "float16 q / scales / out",
                "T": "any: T is split into chunks merged by log-sum-exp; no capacity bound",
                "batch": "any B >= 1; per-sequence caches and ragged lengths accepted",
                "gqa": "any ratio of query to cache heads dividing n_heads",
                "cache_semantics": "MLX-affine artefacts (canonical quantizer, group "
                                   "64 here), the step's own new_k/new_v at full precision"})


def emit(out_dir: Path, bits_list, dh_list) -> list:
    out_dir.mkdir(parents=True, exist_ok=True)
    written, refused = [], []
    for bits in bits_list:
        for dh in dh_list:
            cert = certify(bits, dh)
            problems = C.audit(cert)
            if problems:
                refused.append((cert.kernel_name, problems))
                continue
            (out_dir / f"{cert.kernel_name}.certificate.json").write_text(cert.dumps())
            (out_dir / f"{cert.kernel_name}.md").write_text(C.render_markdown(cert))
            written.append(cert)
    lines = ["# Certificates", "",
             "One per kv_attn_decode specialization (fp16), emitted by `tests/certify.py` on the "
             "chip named in each file.", "",
             "| kernel | cases | worst err/tol | kernels serving it |", "|---|---|---|---|"]
    for cert in written:
        worst = max(c.margin for c in cert.cases)
        kernels = ", ".join(sorted({c.kernel for c in cert.cases}))
        lines.append(f"| `{cert.kernel_name}` | {cert.cases_passed}/{cert.cases_run} | "
                     f"{worst:.3f} | {kernels} |")
    for name, problems in refused:
        lines.append(f"| `{name}` | refused: {'; '.join(problems)} | | |")
    (out_dir / "MANIFEST.md").write_text("\n".join(lines) + "\n")
    return written, refused


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--out", default=str(ROOT / "certificates"))
    ap.add_argument("--bits", type=int, nargs="*", default=[2, 3, 4, 6, 8])
    ap.add_argument("--dh", type=int, nargs="*", default=[64, 128])
    args = ap.parse_args(argv)
    written, refused = emit(Path(args.out), args.bits, args.dh)
    for cert in written:
        print(f"certified {cert.kernel_name}: {cert.cases_passed}/{cert.cases_run}")
    for name, problems in refused:
        print(f"refused {name}: {problems}")
    return 0 if not refused else 1


if __name__ == "__main__":
    sys.exit(main())
