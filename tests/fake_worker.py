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


if __name__ == "__main__":
    main()
