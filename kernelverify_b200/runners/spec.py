"""The contract a candidate kernel arrives in, and its JSON wire form.

Same types, fields, validation rules and wire form as the reference's runner
contract (kernelverify/runners/spec.py:47-414), so cases built for the Metal
runner run unchanged on the CUDA runner:

* `Binding(kind, name, dtype, index)` -- one kernel argument: an input tensor
  by name, an output, or a scalar run parameter by name (:134-168);
* `LaunchSpec(grid, threadgroup, mode, threadgroup_memory)` -- sizes as
  extents: an int, a run-parameter name, or a list multiplied out (:174-260);
* `KernelSpec(source, entry_point, bindings, launch, name)` (:266-320);
* `RunCase(inputs, params, output_shapes, label)` with `validate_against`
  (:326-397);
* arrays travel as {"shape", "dtype", "data": base64} (:403-414).

On the CUDA backend `source` is either CUDA C++ compiled at run time (NVRTC),
with `entry_point` the `extern "C" __global__` name and the binding order the
parameter order, or a kvq library translation unit naming a precompiled
C-ABI entry and the instantiation it selects (see runners/device.py). A
"threadgroup" is a CUDA thread block; `LaunchMode.THREADS` launches
ceil(grid / block) blocks and the kernel must bound-check its own tail,
because CUDA, unlike Metal's dispatchThreads, runs whole blocks.
"""

from __future__ import annotations

import base64
from dataclasses import dataclass, field
from enum import Enum
from typing import Any

import numpy as np

# Element types a tensor binding may carry; uint32 holds packed code words.
TENSOR_DTYPES = {
    "float32": np.float32,
    "float16": np.float16,
    "int32": np.int32,
    "int64": np.int64,
    "uint32": np.uint32,
}

# Scalar arguments, passed by value.
SCALAR_DTYPES = {
    "uint32": np.uint32,
    "int32": np.int32,
    "float32": np.float32,
    "float16": np.float16,
}

MAX_DIMENSIONS = 3


class SpecError(ValueError):
    """The spec or case is unrunnable as written (bad binding, name, extent)."""


class BindingKind(str, Enum):
    INPUT = "input"
    OUTPUT = "output"
    SCALAR = "scalar"


@dataclass(frozen=True)
class Binding:
    """One kernel argument. `index` is its argument slot; by default its
    position in the binding list."""

    kind: BindingKind
    name: str = ""
    dtype: str = ""
    index: int | None = None

    def __post_init__(self):
        object.__setattr__(self, "kind", BindingKind(self.kind))
        if self.kind is BindingKind.SCALAR:
            if not self.name:
                raise SpecError("a scalar binding needs the name of a run parameter")
            if self.dtype not in SCALAR_DTYPES:
                raise SpecError(f"scalar {self.name!r} has dtype {self.dtype!r}; "
                                f"expected one of {sorted(SCALAR_DTYPES)}")
        elif self.kind is BindingKind.INPUT and not self.name:
            raise SpecError("an input binding needs the name of an input tensor")

    def to_json(self) -> dict:
        return {"kind": self.kind.value, "name": self.name, "dtype": self.dtype,
                "index": self.index}

    @staticmethod
    def from_json(raw: dict) -> "Binding":
        return Binding(kind=BindingKind(raw["kind"]), name=raw.get("name", ""),
                       dtype=raw.get("dtype", ""), index=raw.get("index"))


def resolve_extent(extent: Any, params: dict, where: str) -> int:
    """An extent is an int, a run-parameter name, or a list of extents whose
    product is the size. Booleans, empty lists and non-positive results are
    errors."""
    if isinstance(extent, bool):
        raise SpecError(f"{where}: {extent!r} is not a valid extent")
    if isinstance(extent, int):
        size = extent
    elif isinstance(extent, str):
        if extent not in params:
            raise SpecError(f"{where}: no run parameter named {extent!r}")
        size = params[extent]
        if isinstance(size, bool) or not isinstance(size, int):
            raise SpecError(f"{where}: parameter {extent!r} is {size!r}, not an integer")
    elif isinstance(extent, (list, tuple)):
        if len(extent) == 0:
            raise SpecError(f"{where}: an empty product is not a size")
        size = 1
        for part in extent:
            size *= resolve_extent(part, params, where)
    else:
        raise SpecError(f"{where}: {extent!r} is not a valid extent")
    if size < 1:
        raise SpecError(f"{where}: resolved to {size}, which is not a positive size")
    return size


def _extent_json(extent: Any) -> Any:
    return list(extent) if isinstance(extent, tuple) else extent


class LaunchMode(str, Enum):
    #: the grid counts threads (blocks = ceil(grid / block); the kernel guards its tail)
    THREADS = "threads"
    #: the grid counts whole blocks
    THREADGROUPS = "threadgroups"


@dataclass(frozen=True)
class LaunchSpec:
    """Grid and block in extents; `threadgroup_memory` is dynamic shared
    memory in bytes (summed into one dynamic allocation on CUDA)."""

    grid: tuple = (1, 1, 1)
    threadgroup: tuple = (1, 1, 1)
    mode: LaunchMode = LaunchMode.THREADS
    threadgroup_memory: tuple = ()

    def __post_init__(self):
        object.__setattr__(self, "mode", LaunchMode(self.mode))
        for name in ("grid", "threadgroup"):
            value = tuple(getattr(self, name))
            if len(value) != MAX_DIMENSIONS:
                raise SpecError(f"{name} must have {MAX_DIMENSIONS} components, got {value!r}")
            object.__setattr__(self, name, value)
        object.__setattr__(self, "threadgroup_memory", tuple(self.threadgroup_memory))

    def resolve(self, params: dict):
        grid = tuple(resolve_extent(e, params, f"grid[{i}]") for i, e in enumerate(self.grid))
        block = tuple(resolve_extent(e, params, f"threadgroup[{i}]")
                      for i, e in enumerate(self.threadgroup))
        memory = tuple(resolve_extent(e, params, f"threadgroup_memory[{i}]")
                       for i, e in enumerate(self.threadgroup_memory))
        return grid, block, memory

    def to_json(self) -> dict:
        return {"grid": [_extent_json(e) for e in self.grid],
                "threadgroup": [_extent_json(e) for e in self.threadgroup],
                "mode": self.mode.value,
                "threadgroup_memory": [_extent_json(e) for e in self.threadgroup_memory]}

    @staticmethod
    def from_json(raw: dict) -> "LaunchSpec":
        return LaunchSpec(grid=tuple(raw["grid"]), threadgroup=tuple(raw["threadgroup"]),
                          mode=LaunchMode(raw.get("mode", LaunchMode.THREADS.value)),
                          threadgroup_memory=tuple(raw.get("threadgroup_memory", ())))


@dataclass(frozen=True)
class KernelSpec:
    """Source plus everything needed to launch it."""

    source: str
    entry_point: str
    bindings: tuple = ()
    launch: LaunchSpec = field(default_factory=LaunchSpec)
    name: str = ""

    def __post_init__(self):
        object.__setattr__(self, "bindings", tuple(self.bindings))
        if not self.source.strip():
            raise SpecError("kernel source is empty")
        if not self.entry_point:
            raise SpecError("kernel needs an entry point name")
        if not any(b.kind is BindingKind.OUTPUT for b in self.bindings):
            raise SpecError("a kernel with no output binding has nothing to verify")
        taken: set = set()
        for position, binding in enumerate(self.bindings):
            slot = position if binding.index is None else binding.index
            if slot < 0:
                raise SpecError(f"buffer index {slot} is negative")
            if slot in taken:
                raise SpecError(f"buffer index {slot} bound twice")
            taken.add(slot)

    def buffer_index(self, position: int) -> int:
        b = self.bindings[position]
        return position if b.index is None else b.index

    def input_names(self) -> tuple:
        return tuple(b.name for b in self.bindings if b.kind is BindingKind.INPUT)

    def output_count(self) -> int:
        return sum(1 for b in self.bindings if b.kind is BindingKind.OUTPUT)

    def to_json(self) -> dict:
        return {"source": self.source, "entry_point": self.entry_point,
                "bindings": [b.to_json() for b in self.bindings],
                "launch": self.launch.to_json(), "name": self.name}

    @staticmethod
    def from_json(raw: dict) -> "KernelSpec":
        return KernelSpec(source=raw["source"], entry_point=raw["entry_point"],
                          bindings=tuple(Binding.from_json(b) for b in raw.get("bindings", ())),
                          launch=LaunchSpec.from_json(raw["launch"]), name=raw.get("name", ""))


@dataclass(eq=False)
class RunCase:
    """Input tensors, run parameters (scalars and extents) and one
    (shape, dtype) per output binding, in binding order."""

    inputs: dict
    params: dict = field(default_factory=dict)
    output_shapes: tuple = ()
    label: str = ""

    def __post_init__(self):
        shapes = []
        for shape, dtype in self.output_shapes:
            shape = tuple(int(d) for d in shape)
            if dtype not in TENSOR_DTYPES:
                raise SpecError(f"output dtype {dtype!r} is not one of {sorted(TENSOR_DTYPES)}")
            if any(d < 1 for d in shape):
                raise SpecError(f"output shape {shape} has a non-positive dimension")
            shapes.append((shape, dtype))
        self.output_shapes = tuple(shapes)
        if not self.output_shapes:
            raise SpecError("a case needs at least one output shape")

    def validate_against(self, spec: KernelSpec) -> None:
        """Every name the spec binds must be here, before any process starts."""
        if spec.output_count() != len(self.output_shapes):
            raise SpecError(f"kernel binds {spec.output_count()} outputs, "
                            f"the case describes {len(self.output_shapes)}")
        for name in spec.input_names():
            if name not in self.inputs:
                raise SpecError(f"kernel binds input {name!r}, which the case does not supply")
            if str(self.inputs[name].dtype) not in TENSOR_DTYPES:
                raise SpecError(f"input {name!r} has dtype {self.inputs[name].dtype}, "
                                f"expected one of {sorted(TENSOR_DTYPES)}")
        for b in spec.bindings:
            if b.kind is BindingKind.SCALAR and b.name not in self.params:
                raise SpecError(f"kernel binds scalar {b.name!r}, which the case does not supply")
        spec.launch.resolve(self.params)

    def to_json(self) -> dict:
        return {"inputs": {n: array_to_json(a) for n, a in self.inputs.items()},
                "params": self.params,
                "output_shapes": [{"shape": list(s), "dtype": d} for s, d in self.output_shapes],
                "label": self.label}

    @staticmethod
    def from_json(raw: dict) -> "RunCase":
        return RunCase(inputs={n: array_from_json(a) for n, a in raw["inputs"].items()},
                       params=raw.get("params", {}),
                       output_shapes=tuple((tuple(o["shape"]), o["dtype"])
                                           for o in raw.get("output_shapes", ())),
                       label=raw.get("label", ""))


def array_to_json(array: np.ndarray) -> dict:
    a = np.ascontiguousarray(array)
    return {"shape": list(a.shape), "dtype": str(a.dtype),
            "data": base64.b64encode(a.tobytes()).decode()}


def array_from_json(raw: dict) -> np.ndarray:
    flat = np.frombuffer(base64.b64decode(raw["data"]), dtype=np.dtype(raw["dtype"]))
    return flat.reshape(raw["shape"]).copy()
