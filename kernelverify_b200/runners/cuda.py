"""Run candidate CUDA kernels from a process the candidate cannot break.

`CudaRunner` is the parent half, the drop-in for the reference's
`MetalRunner` (kernelverify/runners/metal.py:105-251): same fields, same
`probe` / `run` / `run_one` / `run_candidate` signatures, same results. It
never touches CUDA itself. Each call spawns `kernelverify_b200.runners.worker`
in its own session (process group), hands it one candidate's specs and cases
as JSON, and reads events back one line at a time:

* a hang costs one case: the parent keeps a rolling deadline (the start-up
  budget while the worker starts and compiles, the per-case budget while it
  runs cases); when it expires the process group is killed, the case in
  flight is recorded as TIMEOUT and a fresh worker resumes after it;
* a death mid-batch is the case in flight's CRASH, and the rest still run; a
  death while compiling fails that spec's remaining cases and its sibling
  specs still run;
* a worker that reports its CUDA context lost after a case (the `restart`
  event) is replaced without blaming the next case;
* nothing raises about the candidate: every failure is a RunStatus. Only a
  worker that never opens a device stops the loop, because then the
  environment, not the candidate, is broken.

A fresh process per candidate is deliberate: reusing a worker across
candidates would let one candidate's damage reach the next one's verdict.
"""

from __future__ import annotations

import json
import os
import signal
import subprocess
import sys
import threading
import time
from dataclasses import dataclass, field
from pathlib import Path
from queue import Empty, Queue

from kernelverify_b200.runners.result import DeviceInfo, RunResult, RunStatus
from kernelverify_b200.runners.spec import KernelSpec, RunCase, SpecError

REPO_ROOT = Path(__file__).resolve().parents[2]
WORKER_MODULE = "kernelverify_b200.runners.worker"

DEFAULT_CASE_TIMEOUT = 10.0
DEFAULT_STARTUP_TIMEOUT = 180.0   # a fresh box's first `import torch` can take a minute
DEFAULT_WARMUP = 1
DEFAULT_REPEATS = 5
STDERR_LINES = 200


@dataclass
class BatchResult:
    """One result per case, in case order, plus what the worker reported."""

    results: list = field(default_factory=list)
    device: DeviceInfo | None = None
    stderr: str = ""
    compile_options: dict = field(default_factory=dict)

    def __iter__(self):
        return iter(self.results)

    def __len__(self) -> int:
        return len(self.results)

    def __getitem__(self, index):
        return self.results[index]

    @property
    def all_ok(self) -> bool:
        return all(r.ok for r in self.results)


@dataclass
class _Outcome:
    """What one worker session produced before it finished, died or hung."""

    device: DeviceInfo | None = None
    fatal: RunResult | None = None
    done: bool = False
    timed_out: bool = False
    spawn_error: str = ""
    compiled: set = field(default_factory=set)     # runnable positions built here
    restart_after: tuple | None = None             # (runnable pos, case index)
    compile_options: dict = field(default_factory=dict)
    stderr: str = ""


@dataclass
class CudaRunner:
    """Runs candidate kernels on a CUDA GPU through an isolated worker."""

    case_timeout: float = DEFAULT_CASE_TIMEOUT
    startup_timeout: float = DEFAULT_STARTUP_TIMEOUT
    warmup: int = DEFAULT_WARMUP
    repeats: int = DEFAULT_REPEATS
    python: str = sys.executable
    #: "safe" (IEEE division/sqrt, no flush-to-zero), "relaxed" or "fast"
    math_mode: str = "safe"
    worker_module: str = WORKER_MODULE
    worker_env: dict = field(default_factory=dict)

    # -- device ------------------------------------------------------------
    def probe(self) -> DeviceInfo | None:
        """The GPU a worker sees, or None when there is none."""
        try:
            proc = self._spawn(["--probe"])
        except OSError:
            return None
        try:
            proc.stdin.close()
            events = _EventStream(proc.stdout)
            while True:
                event = events.next_event(self.startup_timeout)
                if event is None:
                    return None
                kind = event.get("event")
                if kind == "device":
                    return DeviceInfo.from_json(event["device"])
                if kind in ("fatal", "done"):
                    return None
        except TimeoutError:
            return None
        finally:
            self._terminate(proc)

    # -- running -------------------------------------------------------------
    def run_one(self, spec: KernelSpec, case: RunCase, **kwargs) -> RunResult:
        return self.run(spec, [case], **kwargs).results[0]

    def run(self, spec: KernelSpec, cases, *, warmup: int | None = None,
            repeats: int | None = None) -> BatchResult:
        return self.run_candidate([(spec, cases)], warmup=warmup, repeats=repeats)[0]

    def run_candidate(self, spec_batches, *, warmup: int | None = None,
                      repeats: int | None = None) -> list:
        """One candidate's (spec, cases) pairs through one worker session
        (more only when a hang or crash forces a resume)."""
        batches = [(spec, list(cases)) for spec, cases in spec_batches]
        slots = [[None] * len(cases) for _, cases in batches]
        runnable = []
        for pos, (spec, cases) in enumerate(batches):
            problem = _validate(spec, cases)
            if problem is not None:
                slots[pos] = [RunResult(status=RunStatus.INVALID_SPEC, detail=problem,
                                        label=c.label) for c in cases]
            elif cases:
                runnable.append(pos)

        device, options, errs = None, {}, []
        cursor = (0, 0)  # (index into runnable, case offset)
        while cursor[0] < len(runnable):
            out = self._session(batches, runnable, cursor, slots, warmup, repeats)
            device = device or out.device
            options = options or out.compile_options
            if out.stderr:
                errs.append(out.stderr)
            if out.done:
                break
            if out.spawn_error:
                _fill(batches, runnable, cursor, slots, RunStatus.CRASH,
                      f"the worker would not start: {out.spawn_error}")
                break
            if out.fatal is not None:
                _fill(batches, runnable, cursor, slots, out.fatal.status, out.fatal.detail)
                break
            if out.device is None:
                status = RunStatus.TIMEOUT if out.timed_out else RunStatus.CRASH
                detail = ("the worker produced nothing before its start-up budget expired"
                          if out.timed_out else
                          "the worker exited before opening the CUDA device" + _tail(out.stderr))
                _fill(batches, runnable, cursor, slots, status, detail)
                break
            hole = _first_hole(batches, runnable, cursor, slots)
            if hole is None:
                break
            rpos, ci = hole
            cases = batches[runnable[rpos]][1]
            if out.restart_after is not None and _next_of(batches, runnable, out.restart_after) == hole:
                cursor = hole                      # clean replacement, nobody blamed
            elif rpos in out.compiled:
                status, detail = _blame(out, "the worker exited before reporting this case")
                slots[runnable[rpos]][ci] = RunResult(status=status, detail=detail,
                                                      label=cases[ci].label)
                cursor = (rpos, ci + 1)
            else:
                status, detail = _blame(out, "the worker died while compiling this kernel",
                                        "the worker was killed while compiling this kernel")
                for i in range(ci, len(cases)):
                    if slots[runnable[rpos]][i] is None:
                        slots[runnable[rpos]][i] = RunResult(status=status, detail=detail,
                                                             label=cases[i].label)
                cursor = (rpos + 1, 0)
            if cursor[0] < len(runnable) and cursor[1] >= len(batches[runnable[cursor[0]]][1]):
                cursor = (cursor[0] + 1, 0)

        stderr = "\n".join(e for e in errs if e).strip()
        results = []
        for pos, (spec, cases) in enumerate(batches):
            row = slots[pos]
            for i, r in enumerate(row):
                if r is None:
                    row[i] = RunResult(status=RunStatus.CRASH,
                                       detail="the worker never reported this case",
                                       label=cases[i].label)
            results.append(BatchResult(results=row, device=device, stderr=stderr,
                                       compile_options=dict(options)))
        return results

    # -- one worker session --------------------------------------------------
    def _session(self, batches, runnable, cursor, slots, warmup, repeats) -> _Outcome:
        out = _Outcome()
        mapping = []         # request spec index -> (runnable pos, case offset)
        specs = []
        for rpos in range(cursor[0], len(runnable)):
            spec, cases = batches[runnable[rpos]]
            offset = cursor[1] if rpos == cursor[0] else 0
            specs.append({"spec": spec.to_json(), "cases": [c.to_json() for c in cases[offset:]]})
            mapping.append((rpos, offset))
        request = {"specs": specs,
                   "warmup": self.warmup if warmup is None else warmup,
                   "repeats": self.repeats if repeats is None else repeats,
                   "math_mode": self.math_mode}
        try:
            proc = self._spawn([])
        except OSError as error:
            out.spawn_error = str(error)
            return out
        tail: list = []
        drain = _drain(proc.stderr, tail)
        threading.Thread(target=_write_request, args=(proc, request), daemon=True).start()
        events = _EventStream(proc.stdout)
        budget = self.startup_timeout
        try:
            while True:
                event = events.next_event(budget)
                if event is None:
                    break
                kind = event.get("event")
                entry = _mapped(event, mapping)
                if kind == "device":
                    out.device = DeviceInfo.from_json(event["device"])
                elif kind == "compiled" and entry is not None:
                    req, (rpos, offset) = entry
                    out.compiled.add(rpos)
                    if isinstance(event.get("compile_options"), dict):
                        out.compile_options = event["compile_options"]
                    left = len(batches[runnable[rpos]][1]) - offset
                    budget = self.case_timeout if left else self.startup_timeout
                elif kind == "spec_failed":
                    try:
                        result = RunResult.from_json(event["result"])
                    except (KeyError, TypeError, ValueError):
                        continue
                    if entry is not None:
                        req, (rpos, offset) = entry
                        out.compiled.discard(rpos)
                        cases = batches[runnable[rpos]][1]
                        for i in range(offset, len(cases)):
                            slots[runnable[rpos]][i] = RunResult(
                                status=result.status, detail=result.detail, label=cases[i].label)
                    budget = self.startup_timeout
                elif kind == "case":
                    try:
                        index = int(event["index"])
                        result = RunResult.from_json(event["result"])
                    except (KeyError, TypeError, ValueError):
                        continue
                    budget = self.case_timeout
                    if entry is not None:
                        req, (rpos, offset) = entry
                        cases = batches[runnable[rpos]][1]
                        absolute = offset + index
                        if 0 <= absolute < len(cases):
                            result.label = result.label or cases[absolute].label
                            slots[runnable[rpos]][absolute] = result
                        if absolute == len(cases) - 1 and req < len(mapping) - 1:
                            budget = self.startup_timeout
                elif kind == "restart" and entry is not None:
                    req, (rpos, offset) = entry
                    try:
                        out.restart_after = (rpos, offset + int(event["index"]))
                    except (KeyError, TypeError, ValueError):
                        pass
                elif kind == "fatal":
                    try:
                        out.fatal = RunResult.from_json(event["result"])
                    except (KeyError, TypeError, ValueError):
                        out.fatal = RunResult(status=RunStatus.CRASH, detail="malformed fatal event")
                    break
                elif kind == "done":
                    out.done = True
                    break
        except TimeoutError:
            out.timed_out = True
        finally:
            self._terminate(proc)
            drain.join(timeout=1.0)
        out.stderr = "".join(tail).strip()
        return out

    # -- process plumbing ----------------------------------------------------
    def _spawn(self, args) -> subprocess.Popen:
        return spawn_isolated(self.python, self.worker_module, args, env=self.worker_env,
                              bufsize=1)

    @staticmethod
    def _terminate(proc: subprocess.Popen) -> None:
        if proc.poll() is None:
            for sig in (signal.SIGTERM, signal.SIGKILL):
                try:
                    os.killpg(os.getpgid(proc.pid), sig)
                except (ProcessLookupError, PermissionError):
                    break
                try:
                    proc.wait(timeout=0.5)
                    break
                except subprocess.TimeoutExpired:
                    continue
        for pipe in (proc.stdin, proc.stdout, proc.stderr):
            try:
                if pipe is not None:
                    pipe.close()
            except OSError:
                pass


class SessionError(RuntimeError):
    """A compiled session could not serve a request: its worker went silent
    past its budget, exited, reported a fatal status, or failed the case."""


class CompiledSession:
    """One kernel held compiled by an isolated worker in `--stream` mode, for
    timing many cases against the same compiled code (an interleaved A/B
    keeps one session per arm open for all its rounds).

        with CompiledSession(runner, spec, warmup=1, repeats=3, name="A") as s:
            result = s.time(case)

    `time` returns the case's RunResult or raises SessionError; the worker's
    process group ends on close() or leaving the `with` block, whatever state
    it is in."""

    def __init__(self, runner: CudaRunner, spec: KernelSpec, *, warmup: int, repeats: int,
                 name: str = "session"):
        self.runner, self.name = runner, name
        self._stderr: list = []
        self._proc = runner._spawn(["--stream"])
        self._stderr_reader = _drain(self._proc.stderr, self._stderr)
        self._events = _EventStream(self._proc.stdout)
        try:
            self._write(json.dumps({"spec": spec.to_json(), "warmup": warmup, "repeats": repeats,
                                    "math_mode": runner.math_mode}) + "\n", "before compiling")
            self._expect("compiled", runner.startup_timeout, "before compiling")
        except BaseException:
            self.close()
            raise

    @staticmethod
    def encode(index: int, case: RunCase) -> str:
        """The wire line of a case request (encode once, send many times)."""
        return json.dumps({"index": index, "case": case.to_json()}) + "\n"

    def time(self, case: RunCase, line: str | None = None) -> RunResult:
        what = f"on case {case.label!r}"
        self._write(line if line is not None else self.encode(0, case), what)
        result = RunResult.from_json(self._expect("case", self.runner.case_timeout, what)["result"])
        if not result.ok or result.timing is None:
            raise SessionError(f"arm {self.name} failed case {case.label!r}: "
                               f"{result.status.value}: {result.detail}")
        return result

    def close(self) -> None:
        proc, self._proc = self._proc, None
        if proc is None:
            return
        try:
            proc.stdin.write(json.dumps({"end": True}) + "\n")
            proc.stdin.flush()
        except (BrokenPipeError, ValueError, OSError):
            pass
        self.runner._terminate(proc)
        self._stderr_reader.join(timeout=1.0)

    def __enter__(self) -> "CompiledSession":
        return self

    def __exit__(self, *exc) -> None:
        self.close()

    # -- the wire --------------------------------------------------------------
    def _write(self, text: str, what: str) -> None:
        try:
            self._proc.stdin.write(text)
            self._proc.stdin.flush()
        except (BrokenPipeError, ValueError, OSError, AttributeError):
            raise SessionError(self._exited(what)) from None

    def _expect(self, kind: str, budget: float, what: str) -> dict:
        """The next event of `kind`; every wait for an event is bounded by
        `budget` seconds."""
        while True:
            try:
                event = self._events.next_event(budget)
            except TimeoutError:
                raise SessionError(f"arm {self.name}: timed out {what}") from None
            if event is None:
                raise SessionError(self._exited(what))
            tag = event.get("event")
            if tag == "fatal":
                failed = RunResult.from_json(event["result"])
                raise SessionError(f"arm {self.name}: {failed.status.value}: {failed.detail}")
            if tag == kind:
                return event

    def _exited(self, what: str) -> str:
        self._stderr_reader.join(timeout=0.5)
        return f"arm {self.name}: the worker died {what}" + _tail("".join(self._stderr))


def spawn_isolated(python: str, module: str, args=(), env=None, **popen_kwargs) -> subprocess.Popen:
    """`python -m module *args` in its own session (so a hung kernel can be
    killed by process group), cwd and PYTHONPATH at the repo root, text pipes
    on all three streams (kernelverify/runners/metal.py:394-421)."""
    environment = dict(os.environ)
    environment.update(env or {})
    prior = environment.get("PYTHONPATH", "")
    environment["PYTHONPATH"] = f"{REPO_ROOT}{os.pathsep}{prior}" if prior else str(REPO_ROOT)
    return subprocess.Popen([python, "-m", module, *args], stdin=subprocess.PIPE,
                            stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                            cwd=str(REPO_ROOT), env=environment, start_new_session=True,
                            **popen_kwargs)


def _validate(spec: KernelSpec, cases) -> str | None:
    for case in cases:
        try:
            case.validate_against(spec)
        except SpecError as error:
            return str(error)
    return None


def _mapped(event: dict, mapping: list):
    try:
        req = int(event["spec"])
    except (KeyError, TypeError, ValueError):
        return None
    if not 0 <= req < len(mapping):
        return None
    return req, mapping[req]


def _holes(batches, runnable, cursor, slots):
    for rpos in range(cursor[0], len(runnable)):
        start = cursor[1] if rpos == cursor[0] else 0
        for i in range(start, len(batches[runnable[rpos]][1])):
            if slots[runnable[rpos]][i] is None:
                yield rpos, i


def _first_hole(batches, runnable, cursor, slots):
    return next(_holes(batches, runnable, cursor, slots), None)


def _next_of(batches, runnable, at):
    rpos, ci = at
    if ci + 1 < len(batches[runnable[rpos]][1]):
        return (rpos, ci + 1)
    return (rpos + 1, 0) if rpos + 1 < len(runnable) else None


def _fill(batches, runnable, cursor, slots, status, detail) -> None:
    for rpos, i in list(_holes(batches, runnable, cursor, slots)):
        slots[runnable[rpos]][i] = RunResult(status=status, detail=detail,
                                             label=batches[runnable[rpos]][1][i].label)


def _tail(stderr: str) -> str:
    lines = stderr.strip().splitlines()[-4:]
    return f": {' / '.join(lines)}" if lines else ""


def _blame(out: _Outcome, crashed: str, timed: str = "the worker was killed after exceeding its time budget"):
    if out.timed_out:
        return RunStatus.TIMEOUT, timed
    return RunStatus.CRASH, crashed + _tail(out.stderr)


def _write_request(proc: subprocess.Popen, request: dict) -> None:
    try:
        json.dump(request, proc.stdin)
        proc.stdin.close()
    except (BrokenPipeError, ValueError, OSError):
        pass


_EOF = object()


class _EventStream:
    """Worker stdout, one decoded event at a time, each wait bounded."""

    def __init__(self, pipe):
        self.queue: Queue = Queue()
        threading.Thread(target=self._pump, args=(pipe,), daemon=True).start()

    def _pump(self, pipe) -> None:
        try:
            for line in pipe:
                self.queue.put(line)
        except (ValueError, OSError):
            pass
        finally:
            self.queue.put(_EOF)

    def next_event(self, budget: float):
        deadline = time.monotonic() + budget
        while True:
            left = deadline - time.monotonic()
            if left <= 0:
                raise TimeoutError(f"the worker produced nothing for {budget:.1f}s")
            try:
                line = self.queue.get(timeout=left)
            except Empty:
                raise TimeoutError(f"the worker produced nothing for {budget:.1f}s") from None
            if line is _EOF:
                return None
            try:
                return json.loads(line)
            except json.JSONDecodeError:
                continue


def _drain(pipe, sink: list, keep: int = STDERR_LINES) -> threading.Thread:
    def run():
        try:
            for line in pipe:
                sink.append(line)
                if len(sink) > keep:
                    del sink[:-keep]
        except (ValueError, OSError):
            pass
    t = threading.Thread(target=run, daemon=True)
    t.start()
    return t
