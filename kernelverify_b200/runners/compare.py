"""Interleaved A/B timing of two kernels in two live workers, with a canary.

The CUDA counterpart of the reference's comparison (kernelverify/runners/
compare.py:190-249): which of two working kernels is faster, under the same
discipline --

* each spec stays compiled in a worker of its own for the whole comparison
  (the worker's `--stream` mode), and every round times the reference arm and
  then the candidate on the same case, back to back;
* `spec_a` is the reference arm and the canary: a round in which its own
  repeats spread wider than `spread_limit` (worst over best, 1.5 by default)
  is rejected -- the device moved under it -- and a comparison with any
  rejected round is not `ok`;
* speedups are reference best over candidate best (interference only ever
  slows a kernel down), the median over the accepted rounds, with every
  round kept in the report;
* an arm that hangs, dies or fails a case aborts the comparison with the
  arm's status in `failure`: a kernel that did not finish has no timing.

Each arm is a `CompiledSession` (runners/cuda.py): a worker in its own
process group, as the batch runner's are, so a hung arm is killed with
everything it started.
"""

from __future__ import annotations

import contextlib
import statistics
from dataclasses import dataclass, field

from kernelverify_b200.runners.cuda import CompiledSession, CudaRunner, SessionError
from kernelverify_b200.runners.spec import KernelSpec, RunCase, SpecError

DEFAULT_SPREAD_LIMIT = 1.5
DEFAULT_ROUNDS = 5


@dataclass
class RoundSample:
    """One round of one case: the reference arm, then the candidate."""

    round_index: int
    ref_best: float
    cand_best: float
    ref_spread: float
    cand_spread: float
    accepted: bool

    @property
    def speedup(self) -> float:
        """Reference time over candidate time (above 1: the candidate is faster)."""
        return self.ref_best / self.cand_best if self.cand_best > 0 else float("nan")


@dataclass
class CaseComparison:
    label: str
    samples: list = field(default_factory=list)

    @property
    def accepted(self) -> list:
        return [s for s in self.samples if s.accepted]

    @property
    def rejected(self) -> int:
        return len(self.samples) - len(self.accepted)

    @property
    def speedup(self) -> float:
        """Median speedup of the accepted rounds (NaN when none stood)."""
        kept = self.accepted
        return statistics.median(s.speedup for s in kept) if kept else float("nan")


@dataclass
class CompareReport:
    cases: list = field(default_factory=list)
    spread_limit: float = DEFAULT_SPREAD_LIMIT
    failure: str = ""

    @property
    def rejected_rounds(self) -> int:
        return sum(c.rejected for c in self.cases)

    @property
    def ok(self) -> bool:
        """Every round of every case stood and no arm failed; a gate exits
        non-zero on anything else."""
        return not self.failure and bool(self.cases) and self.rejected_rounds == 0

    def summary(self) -> str:
        if self.failure:
            return f"comparison failed: {self.failure}"
        lines = []
        for c in self.cases:
            head = (f"speedup {c.speedup:6.3f}x" if c.accepted else "no accepted rounds")
            tail = f", {c.rejected} round(s) rejected" if c.rejected else ""
            lines.append(f"  [{c.label}] {head} over {len(c.accepted)} round(s){tail}")
        if self.rejected_rounds:
            lines.append(f"  REJECTED: the reference arm spread past {self.spread_limit}x in "
                         f"{self.rejected_rounds} round(s); rerun on a quiet device")
        return "\n".join(lines)


def _round(arms, case: RunCase, line: str, round_index: int, spread_limit: float) -> RoundSample:
    """One round of one case: the reference arm, then the candidate, back to
    back on the same wire line; the round stands if the reference arm's own
    repeats stayed within `spread_limit` of each other."""
    ref, cand = (arm.time(case, line).timing for arm in arms)
    return RoundSample(round_index=round_index, ref_best=ref.gpu_best, cand_best=cand.gpu_best,
                       ref_spread=ref.gpu_spread, cand_spread=cand.gpu_spread,
                       accepted=ref.gpu_spread <= spread_limit)


def compare(spec_a: KernelSpec, spec_b: KernelSpec, cases, *, rounds: int = DEFAULT_ROUNDS,
            warmup: int = 1, repeats: int = 3, spread_limit: float = DEFAULT_SPREAD_LIMIT,
            runner: CudaRunner | None = None) -> CompareReport:
    """Interleaved A/B over `cases`, `spec_a` the reference arm and canary.

    The report's `ok` is False -- and a gate built on it must fail -- when an
    arm failed or any round's reference spread passed `spread_limit`; the
    surviving rounds' ratios are still reported, labelled."""
    runner = runner or CudaRunner()
    cases = list(cases)
    report = CompareReport(spread_limit=spread_limit)
    bad = next(((name, c, err) for spec, name in ((spec_a, "A"), (spec_b, "B")) for c in cases
                for err in [_mismatch(c, spec)] if err), None)
    if bad is not None:
        name, c, err = bad
        report.failure = f"arm {name}, case {c.label!r}: {err}"
        return report
    lines = [CompiledSession.encode(i, c) for i, c in enumerate(cases)]
    table = [CaseComparison(label=c.label or f"case {i}") for i, c in enumerate(cases)]
    try:
        with contextlib.ExitStack() as held:
            arms = [held.enter_context(CompiledSession(runner, spec, warmup=warmup, repeats=repeats,
                                                       name=name))
                    for spec, name in ((spec_a, "A (reference)"), (spec_b, "B (candidate)"))]
            for r in range(rounds):
                for row, case, line in zip(table, cases, lines):
                    row.samples.append(_round(arms, case, line, r, spread_limit))
        report.cases = table
    except SessionError as error:
        report.failure = str(error)
    except OSError as error:
        report.failure = f"a worker would not start: {error}"
    return report


def _mismatch(case: RunCase, spec: KernelSpec) -> str:
    """Why `case` cannot run on `spec` ('' when it can)."""
    try:
        case.validate_against(spec)
    except SpecError as error:
        return str(error)
    return ""
