"""A scripted stand-in for kernelverify_b200.runners.worker, for testing the
runner's process logic on a machine without a GPU. Behaviour is chosen by
each case's label: "hang" sleeps past any budget, "crash" exits without
reporting, "sticky" reports a lost-context launch error and asks for a
restart; a spec named "die-compiling" exits before its compiled event.
FAKE_NO_DEVICE=1 reports UNSUPPORTED like a machine without a device."""

import json
import os
import sys
import time

import numpy as np

from kernelverify_b200.runners.result import RunResult, RunStatus, Timing
from kernelverify_b200.runners.spec import KernelSpec, RunCase


def emit(p):
    sys.stdout.write(json.dumps(p) + "\n")
    sys.stdout.flush()


def main():
    if os.environ.get("FAKE_NO_DEVICE") == "1":
        emit({"event": "fatal", "result": RunResult(status=RunStatus.UNSUPPORTED,
                                                    detail="no CUDA device").to_json()})
        emit({"event": "done"})
        return
    emit({"event": "device", "device": {"name": "fake", "max_threads_per_threadgroup": 1024}})
    if "--probe" in sys.argv:
        emit({"event": "done"})
        return
    if "--stream" in sys.argv:
        return stream()
    req = json.loads(sys.stdin.read())
    for s, entry in enumerate(req["specs"]):
        spec = KernelSpec.from_json(entry["spec"])
        if spec.name == "die-compiling":
            os._exit(5)
        emit({"event": "compiled", "spec": s, "compile_options": {"math_mode": req["math_mode"]}})
        for i, raw in enumerate(entry["cases"]):
            case = RunCase.from_json(raw)
            if case.label == "hang":
                time.sleep(60)
            if case.label == "crash":
                os._exit(7)
            if case.label == "sticky":
                emit({"event": "case", "spec": s, "index": i, "result": RunResult(
                    status=RunStatus.LAUNCH_ERROR, detail="an illegal memory access",
                    label=case.label).to_json()})
                emit({"event": "restart", "spec": s, "index": i})
                os._exit(0)
            outs = [np.full(shape, float(case.params.get("fill", 1)), dtype=dtype)
                    for shape, dtype in case.output_shapes]
            emit({"event": "case", "spec": s, "index": i, "result": RunResult(
                status=RunStatus.OK, outputs=outs, timing=Timing((1e-6,), (2e-6,), 1),
                label=case.label).to_json()})
    emit({"event": "done"})


# stream mode: the spec's name sets the timings -- "slow" twice "fast"'s, and
# "noisy" spreads 2x on every second dispatch; case labels "hang" and "crash"
# behave as in batch mode, "fail" reports a launch error
TIMES = {"fast": 1e-6, "slow": 2e-6, "noisy": 1e-6}


def stream():
    header = json.loads(sys.stdin.readline())
    spec = KernelSpec.from_json(header["spec"])
    if spec.name == "die-compiling":
        os._exit(5)
    emit({"event": "compiled", "spec": 0, "compile_options": {"math_mode": header["math_mode"]}})
    base = TIMES.get(spec.name, 1e-6)
    dispatches = 0
    for line in sys.stdin:
        msg = json.loads(line)
        if msg.get("end"):
            break
        case = RunCase.from_json(msg["case"])
        if case.label == "hang":
            time.sleep(60)
        if case.label == "crash":
            os._exit(7)
        dispatches += 1
        if case.label == "fail":
            result = RunResult(status=RunStatus.LAUNCH_ERROR, detail="launch failed",
                               label=case.label)
        else:
            spread = 2.0 if spec.name == "noisy" and dispatches % 2 == 0 else 1.05
            result = RunResult(status=RunStatus.OK, outputs=[],
                               timing=Timing((base, base * spread, base), (base,), 1),
                               label=case.label)
        emit({"event": "case", "spec": 0, "index": msg["index"], "result": result.to_json()})
    emit({"event": "done"})


if __name__ == "__main__":
    main()
