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

Each worker runs in its own process group, as the batch runner's do, so a
hung arm is killed with everything it started.
"""

from __future__ import annotations

import json
import statistics
from dataclasses import dataclass, field

from kernelverify_b200.runners.cuda import CudaRunner, _drain, _EventStream, _tail
from kernelverify_b200.runners.result import RunResult
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


class ComparisonAborted(RuntimeError):
    """An arm could not finish its half of the comparison."""


class _LiveArm:
    """A stream-mode worker holding one compiled spec across the rounds."""

    def __init__(self, runner: CudaRunner, spec: KernelSpec, name: str, warmup: int,
                 repeats: int):
        self.name, self.runner = name, runner
        self.proc = runner._spawn(["--stream"])
        self.stderr: list = []
        self.drain = _drain(self.proc.stderr, self.stderr)
        self.events = _EventStream(self.proc.stdout)
        try:
            self._send({"spec": spec.to_json(), "warmup": warmup, "repeats": repeats,
                        "math_mode": runner.math_mode})
            self._await_compiled()
        except BaseException:
            runner._terminate(self.proc)
            raise

    def _send(self, payload: dict) -> None:
        try:
            self.proc.stdin.write(json.dumps(payload) + "\n")
            self.proc.stdin.flush()
        except (BrokenPipeError, ValueError, OSError) as error:
            raise ComparisonAborted(self._died(f"while being sent work ({error})")) from None

    def _next(self, budget: float, what: str) -> dict:
        try:
            event = self.events.next_event(budget)
        except TimeoutError:
            raise ComparisonAborted(f"arm {self.name}: timed out {what}") from None
        if event is None:
            raise ComparisonAborted(self._died(what))
        if event.get("event") == "fatal":
            r = RunResult.from_json(event["result"])
            raise ComparisonAborted(f"arm {self.name}: {r.status.value}: {r.detail}")
        return event

    def _await_compiled(self) -> None:
        while self._next(self.runner.startup_timeout, "before compiling").get("event") != "compiled":
            pass

    def time_case(self, case: RunCase, line: str) -> RunResult:
        """Dispatch one case (its wire line is encoded once, outside the
        rounds, so encoding never widens the gap between the two arms)."""
        try:
            self.proc.stdin.write(line)
            self.proc.stdin.flush()
        except (BrokenPipeError, ValueError, OSError):
            raise ComparisonAborted(self._died(f"on case {case.label!r}")) from None
        while True:
            event = self._next(self.runner.case_timeout, f"on case {case.label!r}")
            if event.get("event") != "case":
                continue
            result = RunResult.from_json(event["result"])
            if not result.ok or result.timing is None:
                raise ComparisonAborted(f"arm {self.name} failed case {case.label!r}: "
                                        f"{result.status.value}: {result.detail}")
            return result

    def _died(self, when: str) -> str:
        self.drain.join(timeout=0.5)
        return f"arm {self.name}: the worker died {when}" + _tail("".join(self.stderr))

    def close(self) -> None:
        try:
            self.proc.stdin.write(json.dumps({"end": True}) + "\n")
            self.proc.stdin.flush()
        except (BrokenPipeError, ValueError, OSError):
            pass
        self.runner._terminate(self.proc)
        self.drain.join(timeout=1.0)


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
    for spec, name in ((spec_a, "A"), (spec_b, "B")):
        for c in cases:
            try:
                c.validate_against(spec)
            except SpecError as error:
                report.failure = f"arm {name}, case {c.label!r}: {error}"
                return report
    wire = [json.dumps({"index": i, "case": c.to_json()}) + "\n" for i, c in enumerate(cases)]
    arms: list = []
    try:
        ref = _LiveArm(runner, spec_a, "A (reference)", warmup, repeats)
        arms.append(ref)
        cand = _LiveArm(runner, spec_b, "B (candidate)", warmup, repeats)
        arms.append(cand)
        out = [CaseComparison(label=c.label or f"case {i}") for i, c in enumerate(cases)]
        for r in range(rounds):
            for i, c in enumerate(cases):
                a = ref.time_case(c, wire[i]).timing
                b = cand.time_case(c, wire[i]).timing
                out[i].samples.append(RoundSample(
                    round_index=r, ref_best=a.gpu_best, cand_best=b.gpu_best,
                    ref_spread=a.gpu_spread, cand_spread=b.gpu_spread,
                    accepted=a.gpu_spread <= spread_limit))
        report.cases = out
    except ComparisonAborted as error:
        report.failure = str(error)
    except OSError as error:
        report.failure = f"a worker would not start: {error}"
    finally:
        for arm in arms:
            arm.close()
    return report
