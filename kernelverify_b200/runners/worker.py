"""The subprocess that touches the GPU: `python -m kernelverify_b200.runners.worker`.

Reads one JSON request on stdin, streams one JSON event per line on stdout,
in the reference's wire format (kernelverify/runners/worker.py:24-34):

    {"event": "device", "device": {...}}      first, when a device opened
    {"event": "compiled", "spec": s, ...}     spec s is built
    {"event": "spec_failed", "spec": s, "result": {...}}
    {"event": "case", "spec": s, "index": i, "result": {...}}
    {"event": "fatal", "result": {...}}       nothing can run here
    {"event": "done"}

plus one CUDA-specific event:

    {"event": "restart", "spec": s, "index": i}

sent after case i when its launch left the CUDA context unusable (a sticky
error: every later launch in this process would fail). The worker exits; the
parent resumes from case i+1 in a fresh process without blaming it.

`--probe` reports the device and stops; `--stream` serves one spec with cases
paced line by line by the parent (kernelverify/runners/worker.py:153-193).
`KVQ_FORCE_NO_GPU=1` makes the worker report UNSUPPORTED, as if no device
existed.
"""

from __future__ import annotations

import json
import os
import sys
import traceback

from kernelverify_b200.runners.result import RunResult, RunStatus
from kernelverify_b200.runners.spec import KernelSpec, RunCase, SpecError

# CUDA errors after which the context cannot launch again in this process.
_STICKY = ("illegal address", "illegal instruction", "misaligned address",
           "unspecified launch failure", "hardware stack error", "an illegal memory access",
           "CUDA_ERROR_ILLEGAL", "CUDA_ERROR_LAUNCH_FAILED", "cudaErrorIllegal",
           "cudaErrorLaunchFailure", "cudaErrorMisalignedAddress")


def emit(payload: dict) -> None:
    sys.stdout.write(json.dumps(payload) + "\n")
    sys.stdout.flush()


def fatal(status: RunStatus, detail: str) -> int:
    emit({"event": "fatal", "result": RunResult(status=status, detail=detail).to_json()})
    emit({"event": "done"})
    return 0


def compiled_event(spec_index: int, kernel) -> dict:
    return {"event": "compiled", "spec": spec_index,
            "max_threads_per_threadgroup": kernel.max_threads,
            "thread_execution_width": kernel.execution_width,
            "compile_options": {"math_mode": kernel.math_mode,
                                "nvrtc": list(getattr(kernel, "options", []) or []),
                                "library": getattr(kernel, "entry", "")}}


def spec_failed_event(spec_index: int, status: RunStatus, detail: str) -> dict:
    return {"event": "spec_failed", "spec": spec_index,
            "result": RunResult(status=status, detail=detail).to_json()}


def _sticky(detail: str) -> bool:
    return any(s.lower() in detail.lower() for s in _STICKY)


def _run_case(kernel, raw_case: dict, warmup: int, repeats: int) -> RunResult:
    try:
        case = RunCase.from_json(raw_case)
        return kernel.run(case, warmup=warmup, repeats=repeats)
    except SpecError as error:
        return RunResult(status=RunStatus.INVALID_SPEC, detail=str(error),
                         label=raw_case.get("label", ""))
    except Exception:  # a driver failure is the kernel's problem
        return RunResult(status=RunStatus.LAUNCH_ERROR,
                         detail=traceback.format_exc(limit=3).strip(),
                         label=raw_case.get("label", ""))


def _open_device():
    if os.environ.get("KVQ_FORCE_NO_GPU") == "1":
        raise RuntimeError("KVQ_FORCE_NO_GPU=1: behaving as if no CUDA device existed")
    from kernelverify_b200.runners.device import CudaDevice
    return CudaDevice(int(os.environ.get("KVQ_RUNNER_DEVICE", "0")))


def main(argv: list) -> int:
    try:
        from kernelverify_b200.runners.device import CompileError  # noqa: F401
    except ImportError as error:
        return fatal(RunStatus.UNSUPPORTED, f"the CUDA device layer is unavailable: {error}")
    try:
        device = _open_device()
    except Exception as error:  # no GPU, no driver, wrong arch
        return fatal(RunStatus.UNSUPPORTED, str(error))

    emit({"event": "device", "device": device.info().to_json()})
    if "--probe" in argv:
        emit({"event": "done"})
        return 0
    if "--stream" in argv:
        return stream(device)

    try:
        request = json.loads(sys.stdin.read())
    except ValueError as error:
        return fatal(RunStatus.INVALID_SPEC, f"the request was not valid JSON: {error}")
    warmup = int(request.get("warmup", 1))
    repeats = int(request.get("repeats", 5))
    math_mode = request.get("math_mode", "safe")

    from kernelverify_b200.runners.device import CompileError
    for spec_index, entry in enumerate(request.get("specs", [])):
        device.release_pool()
        try:
            spec = KernelSpec.from_json(entry["spec"])
        except (SpecError, KeyError, TypeError) as error:
            emit(spec_failed_event(spec_index, RunStatus.INVALID_SPEC, str(error)))
            continue
        try:
            kernel = device.compile(spec, math_mode=math_mode)
        except CompileError as error:
            emit(spec_failed_event(spec_index, RunStatus.COMPILE_ERROR, str(error)))
            continue
        emit(compiled_event(spec_index, kernel))
        for index, raw_case in enumerate(entry.get("cases", [])):
            result = _run_case(kernel, raw_case, warmup, repeats)
            emit({"event": "case", "spec": spec_index, "index": index,
                  "result": result.to_json()})
            if not result.ok and _sticky(result.detail):
                emit({"event": "restart", "spec": spec_index, "index": index})
                sys.stdout.flush()
                os._exit(0)
    emit({"event": "done"})
    return 0


def stream(device) -> int:
    """One spec; cases arrive one line at a time:
    first line {"spec", "warmup", "repeats", "math_mode"}, then
    {"index": i, "case": {...}} lines and {"end": true}."""
    from kernelverify_b200.runners.device import CompileError
    header = json.loads(sys.stdin.readline())
    warmup = int(header.get("warmup", 1))
    repeats = int(header.get("repeats", 5))
    try:
        spec = KernelSpec.from_json(header["spec"])
    except (SpecError, KeyError, TypeError) as error:
        return fatal(RunStatus.INVALID_SPEC, str(error))
    try:
        kernel = device.compile(spec, math_mode=header.get("math_mode", "safe"))
    except CompileError as error:
        return fatal(RunStatus.COMPILE_ERROR, str(error))
    emit(compiled_event(0, kernel))
    for line in sys.stdin:
        if not line.strip():
            continue
        message = json.loads(line)
        if message.get("end"):
            break
        index = int(message.get("index", 0))
        result = _run_case(kernel, message.get("case", {}), warmup, repeats)
        emit({"event": "case", "spec": 0, "index": index, "result": result.to_json()})
    emit({"event": "done"})
    return 0


if __name__ == "__main__":
    raise SystemExit(main(sys.argv[1:]))
