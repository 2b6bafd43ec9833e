"""Certificates for the CUDA specializations of kv_attn_decode.

The B200 form of the reference's certificate (kernelverify/report/
certificate.py:129-253, bench/emit_pack_certificates.py:239-338): one JSON
document per specialization (bits x head_dim x dtype) saying WHAT was verified
(byte-bound: hashes of the CUDA translation units, build flags and target
architecture, and of the built library), HOW (protocol-bound: the fixed-case
sweep, its seeds, the tolerance model), which contract clauses hold and how
each is established, where the verdict binds (chip, toolchain, domain), and,
as advisory evidence only, the per-case error margins.

This module is the data model, the audit (complaints a reviewer would make,
refusing any certificate that reads stronger than its evidence) and the
markdown rendering; the cases are run and judged by the emitter, which lives
with the test infrastructure (tests/certify.py).
"""

from __future__ import annotations

import hashlib
import json
import platform
from dataclasses import asdict, dataclass, field
from pathlib import Path

SCHEMA_VERSION = 1
FAMILY = "kv_attn_decode"
NUMERIC = "numeric-battery"
STRUCTURAL = "source-attestation"

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"


def build_flags() -> list[str]:
    """The target architecture and the compile flags, without include paths
    (which name where the tree happens to sit, not what is built)."""
    from kernelverify_b200 import build
    flags, skip = [], False
    for a in list(build.ARCH) + list(build.NVCC_FLAGS):
        if skip:
            skip = False
            continue
        if a == "-I":
            skip = True
            continue
        if a.startswith("-I"):
            continue
        flags.append(a)
    return flags


def translation_unit_sha256() -> str:
    """sha256 over every CUDA source and header of the library (sorted by
    name, name and bytes each), the header of the C ABI, and the build flags
    and target architecture -- what the verified binary is built from."""
    h = hashlib.sha256()
    files = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) \
        + sorted(CSRC.glob("*.inc")) + [PACKAGE.parent / "include" / "kvq_b200.h"]
    for f in files:
        h.update(f.name.encode())
        h.update(f.read_bytes())
    h.update(" ".join(build_flags()).encode())
    return h.hexdigest()


def library_sha256() -> str:
    from kernelverify_b200 import _native
    return hashlib.sha256(_native.LIB_PATH.read_bytes()).hexdigest()


def nvcc_version() -> str:
    """The CUDA compiler's release line (the library's build toolchain)."""
    import subprocess
    from kernelverify_b200 import build
    try:
        out = subprocess.run([build.nvcc(), "--version"], capture_output=True, text=True,
                             timeout=30).stdout
        return next((l.strip() for l in out.splitlines() if "release" in l), "unknown")
    except Exception:
        return "unknown"


@dataclass
class ClauseAttestation:
    clause: str
    statement: str
    mechanism: str          # NUMERIC or STRUCTURAL
    evidence: str
    scope: str = ""

    def __post_init__(self):
        if self.mechanism not in (NUMERIC, STRUCTURAL):
            raise ValueError(f"clause {self.clause}: unknown mechanism {self.mechanism!r}")


@dataclass
class CaseEvidence:
    label: str
    passed: bool
    err: float
    tol: float
    output_sha256: str
    kernel: str             # which device kernel served the case
    ref_max: float = 0.0    # max|fp64 reference| of the judged case (0: not recorded)

    @property
    def margin(self) -> float:
        return self.err / self.tol if self.tol > 0 else float("inf")

    @property
    def max_rel(self) -> float | None:
        """max-abs error relative to max|ref|, when the magnitude was recorded."""
        return self.err / self.ref_max if self.ref_max > 0 else None


@dataclass
class Certificate:
    bits: int
    head_dim: int
    dtype: str
    policy: str
    seed_protocol: str
    cases: list = field(default_factory=list)           # CaseEvidence
    clauses: tuple = ()                                  # ClauseAttestation
    precision: str = "contract"                          # "contract" or "fast"
    translation_unit: str = ""
    library: str = ""
    flags: list = field(default_factory=list)
    chip: str = ""
    toolchain: dict = field(default_factory=dict)
    harness_commit: str = ""
    domain: dict = field(default_factory=dict)
    budget: int = 0

    @property
    def kernel_name(self) -> str:
        return f"{FAMILY}-BITS{self.bits}-DH{self.head_dim}-{self.dtype}"

    @property
    def cases_run(self) -> int:
        return len(self.cases)

    @property
    def cases_passed(self) -> int:
        return sum(1 for c in self.cases if c.passed)

    def to_json(self) -> dict:
        return {
            "schema_version": SCHEMA_VERSION,
            "kernel": self.kernel_name,
            "kernel_family": FAMILY,
            "byte_bound": {
                "_meaning": "these hashes identify WHAT was verified; they assert nothing about "
                            "output values",
                "translation_unit_sha256": self.translation_unit,
                "library_sha256": self.library,
                "build": self.flags,
                "precision": self.precision,
                "harness_commit": self.harness_commit,
                "contract_version": ("kv_attention contract (NATIVE_OPS['kv_attention']); K borrowed "
                                     "from quantized_matmul, uncalibrated over KV_MEMBERS"),
                "not_attested_by_these_hashes": [
                    "the caller's own copies or layout changes before the C entry",
                    "a library built from other sources or flags",
                ],
            },
            "protocol_bound": {
                "_assertion": "re-running the published protocol on a machine matching the recorded "
                              "chip and toolchain reproduces these verdicts",
                "operator": "kv_attention",
                "policy": self.policy,
                "cases_run": self.cases_run,
                "cases_passed": self.cases_passed,
                "all_passed": self.cases_passed == self.cases_run,
                "seed_protocol": self.seed_protocol,
                "tolerance_model": {
                    "anchor": "NATIVE_OPS['kv_attention'] fp64 reference",
                    "floor": "operator ensemble floor (4 fp32 members)",
                    "K_quant": 4.0,
                    "form": "max(base_tol(dtype), K_QUANT * floor)",
                },
            },
            "attestation": {
                "_meaning": "not every clause is established the same way; a clause no test can "
                            "separate is attested from source",
                "clauses": [asdict(c) for c in self.clauses],
            },
            "validity": {
                "binding_on": {"chip_generation": self.chip, "toolchain": self.toolchain},
                "elsewhere": "advisory: another chip or toolchain may move numerics legitimately",
                "domain": self.domain,
            },
            "advisory": {
                "_meaning": "advisory, NOT reproducible: GPU outputs need not be bit-stable across "
                            "runs, so fingerprints and margins describe this run only",
                "cases": [{"label": c.label, "kernel": c.kernel, "output_sha256": c.output_sha256,
                           "err": c.err, "tol": c.tol, "margin_err_over_tol": round(c.margin, 6),
                           **({"ref_max_abs": c.ref_max, "max_rel_err": c.max_rel}
                              if c.max_rel is not None else {}),
                           "passed": c.passed} for c in self.cases],
            },
        }

    def dumps(self) -> str:
        return json.dumps(self.to_json(), indent=1, sort_keys=False) + "\n"


def audit(cert: Certificate) -> list[str]:
    """Complaints a reviewer would make; empty means the certificate is honest.
    Deliberately picky: the failure it guards against is a certificate that
    reads stronger than the verification behind it."""
    problems: list[str] = []
    if cert.cases_run == 0:
        problems.append("no case was run")
    if cert.cases_passed != cert.cases_run:
        problems.append(f"{cert.cases_run - cert.cases_passed} of {cert.cases_run} cases failed; "
                        "a certificate is not issued for a kernel that did not pass")
    if cert.budget and cert.cases_run < cert.budget:
        problems.append(f"only {cert.cases_run} cases run against a stated budget of {cert.budget}")
    covered = {c.clause for c in cert.clauses}
    if "C1" not in covered:
        problems.append("C1 (working-precision floor) is unattested; its absence voids the "
                        "certificate")
    if cert.precision != "contract":
        problems.append(f"precision {cert.precision!r} carries the combine's weights below "
                        "binary32; C1 cannot hold for it")
    if not cert.translation_unit or not cert.library:
        problems.append("byte-bound hashes missing: the certificate would not say what it verified")
    if not cert.chip:
        problems.append("no chip recorded: the verdict would bind nowhere")
    return problems


def render_markdown(cert: Certificate) -> str:
    """A human-readable summary that leads with the limits, not the claim."""
    lines = [f"# Certificate: {cert.kernel_name}", "",
             f"Operator `kv_attention`, verified at {cert.cases_passed}/{cert.cases_run} cases "
             f"under the `{cert.policy}` policy.", "",
             "## What this asserts", "",
             "Re-running the published protocol on a matching machine reproduces these verdicts.",
             "", "## What this does not assert", "",
             "That output values are identical across runs or machines.", "",
             "## Contract clauses and how each was established", "",
             "| Clause | Requirement | Established by | Evidence |", "|---|---|---|---|"]
    for c in cert.clauses:
        how = "battery measurement" if c.mechanism == NUMERIC else "reading the kernel source"
        scope = f" ({c.scope})" if c.scope else ""
        lines.append(f"| {c.clause} | {c.statement} | {how}{scope} | {c.evidence} |")
    lines += ["", "## Validity", "",
              f"Binding on {cert.chip} with the recorded toolchain "
              f"({', '.join(f'{k} {v}' for k, v in sorted(cert.toolchain.items()))}); "
              "advisory elsewhere.", ""]
    problems = audit(cert)
    if problems:
        lines += ["## Audit complaints", ""] + [f"- {p}" for p in problems] + [""]
    return "\n".join(lines).rstrip() + "\n"


def contract_clauses(precision: str = "contract") -> tuple:
    """The clause set this library can attest, from its kernels' source."""
    clauses = []
    if precision == "contract":
        clauses.append(ClauseAttestation(
            "C1", "every intermediate at binary32 or wider", STRUCTURAL,
            "every accumulator is fp32; score products are fp16 x fp16 (exact in fp32); the "
            "tensor-core combine carries p * v_scale as three bf16 parts, 2^-23 relative, "
            "against exact codes; the CUDA-core kernel computes in fp32 throughout",
            scope="all kernels"))
    clauses += [
        ClauseAttestation(
            "C4", "exponential sums shifted by their own maximum", STRUCTURAL,
            "exponents are taken against a running reference point that moves whenever a score "
            "exceeds it by 2^8 (lazy rescaling), so every weight before normalisation is at most "
            "2^8 -- the shift of the clause, up to that bounded factor; the final merge shifts by "
            "the exact maximum"),
        ClauseAttestation(
            "C5", "the specified formula, not a defensible relative", NUMERIC,
            "judged against the operator's fp64 reference within the shipped tolerance on every "
            "case of the protocol (and on the 400-case battery in the test suite)"),
    ]
    return tuple(clauses)


def toolchain() -> dict:
    """Versions the verdict binds on (queried, not assumed)."""
    import numpy
    import torch
    tc = {"python": platform.python_version(), "numpy": numpy.__version__,
          "torch": torch.__version__, "torch_cuda": str(torch.version.cuda),
          "nvcc": nvcc_version()}
    try:
        import subprocess
        drv = subprocess.run(["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader"],
                             capture_output=True, text=True, timeout=20).stdout.strip().splitlines()
        if drv:
            tc["driver"] = drv[0]
    except Exception:
        pass
    return tc
