"""Max-abs and max-rel error versus the fp64 reference for every certified
case, from the committed certificates -- TEST INFRASTRUCTURE (it reads the
oracle). No GPU needed.

The certificates record each case's max-abs error and tolerance as measured
on the chip. The protocol's inputs are seeded and the fp64 reference is
deterministic, so where a certificate predates the recorded magnitude, max|ref|
is recomputed here and max-rel = err / max|ref|; for a per-sequence case the
judged sequence is the one whose tolerance equals the recorded one.

    python tests/parity_table.py [--certs certificates] [--out certificates/PARITY.md]
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from oracle import kv  # noqa: E402
from tests.certify import protocol_cases  # noqa: E402


def reference_magnitude(kind: str, arrays, bits: int, tol: float) -> tuple[float, str]:
    """(max|ref| of the judged case, how it was found). "recomputed" also
    means the recomputed tolerance equals the recorded one bit for bit."""
    q, kc, vc, nk, nv = arrays
    if kind == "shared":
        ref, t = kv.reference_and_tolerance(kv.gqa_tiled_inputs(q, kc, vc, nk, nv, bits),
                                            "float16")
        how = "recomputed" if t == tol else "recomputed (tolerance differs)"
        return float(np.max(np.abs(ref))), how
    mags = []
    for b in range(q.shape[0]):
        x = kv.gqa_tiled_inputs(q[b:b + 1], kc[b], vc[b], nk[b:b + 1], nv[b:b + 1], bits)
        ref, t = kv.reference_and_tolerance(x, "float16")
        mag = float(np.max(np.abs(ref)))
        if t == tol:
            return mag, f"recomputed (sequence {b})"
        mags.append(mag)
    return min(mags), "bound (smallest sequence magnitude)"


def rows(cert_dir: Path, pattern: str = "*.certificate.json") -> list:
    out = []
    for path in sorted(cert_dir.glob(pattern)):
        doc = json.loads(path.read_text())
        bits, dh = doc["validity"]["domain"]["BITS"], doc["validity"]["domain"]["DH"]
        protocol = {label: (kind, arrays) for label, kind, arrays, _ in protocol_cases(bits, dh)}
        for c in doc["advisory"]["cases"]:
            if "ref_max_abs" in c:
                mag, how = c["ref_max_abs"], "recorded"
            else:
                kind, arrays = protocol[c["label"]]
                mag, how = reference_magnitude(kind, arrays, bits, c["tol"])
            out.append({"kernel": doc["kernel"], "case": c["label"], "served_by": c["kernel"],
                        "err": c["err"], "rel": c["err"] / mag if mag > 0 else 0.0,
                        "tol": c["tol"], "tol_rel": c["tol"] / mag if mag > 0 else 0.0,
                        "ref_max": mag, "how": how, "passed": c["passed"]})
    return out


def render(table: list, chip: str) -> str:
    lines = ["# Parity of the certified cases: max-abs and max-rel error versus fp64", "",
             f"fp16 outputs on {chip}, from the committed certificates "
             "(`python tests/parity_table.py`). max-rel = max-abs / max|ref|; the tolerance "
             "is the reference's own (max(4 eps(fp16) max|ref|, 4 x the worst fp32 member)), "
             "shown also relative to max|ref|.", "",
             "| certificate | case | kernel | max-abs | max-rel | tolerance | tolerance rel | "
             "err / tol | max\\|ref\\| |",
             "|---|---|---|---|---|---|---|---|---|"]
    for r in table:
        lines.append(f"| `{r['kernel']}` | {r['case']} | {r['served_by']} | {r['err']:.3e} | "
                     f"{r['rel']:.3e} | {r['tol']:.3e} | {r['tol_rel']:.3e} | "
                     f"{r['err'] / r['tol']:.3f} | {r['ref_max']:.4g} |")
    worst_rel = max(r["rel"] for r in table)
    worst_margin = max(r["err"] / r["tol"] for r in table)
    lines += ["", f"Largest max-rel error: {worst_rel:.3e} (fp16's unit roundoff is 4.88e-4); "
              f"largest err / tol: {worst_margin:.3f}; every case passed: "
              f"{all(r['passed'] for r in table)}."]
    off = [r for r in table if "differs" in r["how"]]
    if off:
        lines.append(f"{len(off)} rows: the recomputed tolerance differs from the recorded one.")
    bounds = [r for r in table if r["how"].startswith("bound")]
    if bounds:
        lines.append(f"{len(bounds)} per-sequence rows use the smallest sequence magnitude (an "
                     "upper bound on max-rel): the recorded tolerance matched no sequence.")
    return "\n".join(lines) + "\n"


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--certs", default=str(ROOT / "certificates"))
    ap.add_argument("--out", default=str(ROOT / "certificates" / "PARITY.md"))
    args = ap.parse_args(argv)
    cert_dir = Path(args.certs)
    table = rows(cert_dir)
    chip = {json.loads(p.read_text())["validity"]["binding_on"]["chip_generation"]
            for p in cert_dir.glob("*.certificate.json")}
    Path(args.out).write_text(render(table, ", ".join(sorted(chip))))
    print(f"wrote {args.out}: {len(table)} cases")
    return 0


if __name__ == "__main__":
    sys.exit(main())
