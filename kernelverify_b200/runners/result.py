"""What a run returns: a status, the outputs, a timing sample.

Same statuses, types and wire form as the reference
(kernelverify/runners/result.py:67-173). Execution failures are statuses,
never exceptions: OK (judge the outputs), COMPILE_ERROR / LAUNCH_ERROR (the
candidate is rejected; `detail` says why), TIMEOUT (did not finish inside the
budget), CRASH (the worker died -- usually an out-of-bounds write),
INVALID_SPEC (the launch description is unusable; not a verdict on the
kernel), UNSUPPORTED (no usable device here; not a verdict either).

On CUDA, `gpu_seconds` come from CUDA events recorded on the launch stream
around each timed dispatch, `wall_seconds` from the host clock around launch
+ synchronize. Compare candidates on `gpu_best` and read `gpu_spread` before
believing a small difference.
"""

from __future__ import annotations

import statistics
from dataclasses import dataclass, field
from enum import Enum

from kernelverify_b200.runners.spec import array_from_json, array_to_json


class RunStatus(str, Enum):
    OK = "ok"
    COMPILE_ERROR = "compile_error"
    LAUNCH_ERROR = "launch_error"
    TIMEOUT = "timeout"
    CRASH = "crash"
    INVALID_SPEC = "invalid_spec"
    UNSUPPORTED = "unsupported"


@dataclass(frozen=True)
class Timing:
    """Per-repeat GPU and wall samples, warm-up excluded."""

    gpu_seconds: tuple = ()
    wall_seconds: tuple = ()
    warmup: int = 0

    @property
    def repeats(self) -> int:
        return len(self.gpu_seconds)

    @property
    def gpu_best(self) -> float:
        return min(self.gpu_seconds) if self.gpu_seconds else float("nan")

    @property
    def gpu_median(self) -> float:
        return statistics.median(self.gpu_seconds) if self.gpu_seconds else float("nan")

    @property
    def wall_median(self) -> float:
        return statistics.median(self.wall_seconds) if self.wall_seconds else float("nan")

    @property
    def gpu_spread(self) -> float:
        """Worst over best; a wide spread means the candidate was not measured."""
        if not self.gpu_seconds or self.gpu_best <= 0.0:
            return float("nan")
        return max(self.gpu_seconds) / self.gpu_best

    def to_json(self) -> dict:
        return {"gpu_seconds": list(self.gpu_seconds), "wall_seconds": list(self.wall_seconds),
                "warmup": self.warmup}

    @staticmethod
    def from_json(raw: dict) -> "Timing":
        return Timing(gpu_seconds=tuple(raw.get("gpu_seconds", ())),
                      wall_seconds=tuple(raw.get("wall_seconds", ())),
                      warmup=int(raw.get("warmup", 0)))


@dataclass
class RunResult:
    status: RunStatus = RunStatus.OK
    outputs: list = field(default_factory=list)
    timing: Timing | None = None
    detail: str = ""
    label: str = ""

    @property
    def ok(self) -> bool:
        return self.status is RunStatus.OK

    def to_json(self) -> dict:
        return {"status": self.status.value, "outputs": [array_to_json(o) for o in self.outputs],
                "timing": self.timing.to_json() if self.timing is not None else None,
                "detail": self.detail, "label": self.label}

    @staticmethod
    def from_json(raw: dict) -> "RunResult":
        return RunResult(status=RunStatus(raw["status"]),
                         outputs=[array_from_json(o) for o in raw.get("outputs", ())],
                         timing=Timing.from_json(raw["timing"]) if raw.get("timing") else None,
                         detail=raw.get("detail", ""), label=raw.get("label", ""))


@dataclass(frozen=True)
class DeviceInfo:
    """The device the worker opened, for the record. On CUDA
    `max_threads_per_threadgroup` is max threads per block,
    `max_threadgroup_memory` the opt-in shared memory per block, and
    `registry_id` the PCI bus id packed into an int."""

    name: str = ""
    max_threads_per_threadgroup: int = 0
    max_threadgroup_memory: int = 0
    has_unified_memory: bool = True
    registry_id: int = 0

    def to_json(self) -> dict:
        return {"name": self.name, "max_threads_per_threadgroup": self.max_threads_per_threadgroup,
                "max_threadgroup_memory": self.max_threadgroup_memory,
                "has_unified_memory": self.has_unified_memory, "registry_id": self.registry_id}

    @staticmethod
    def from_json(raw: dict) -> "DeviceInfo":
        return DeviceInfo(**{k: raw[k] for k in raw if k in DeviceInfo.__annotations__})
