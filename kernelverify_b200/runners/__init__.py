"""Backends that execute a candidate kernel and hand its output to the oracle.

The CUDA counterpart of kernelverify's runner package
(kernelverify/runners/__init__.py): the backend-neutral contract (`spec`,
`result`, `specialize`) plus `CudaRunner`, which compiles each candidate once
per spec and dispatches it over a batch of cases inside a worker process the
candidate cannot take down with it. Importing this package touches no GPU;
ask `CudaRunner().probe()` whether a device is present.
"""

from kernelverify_b200.runners.cuda import BatchResult, CompiledSession, CudaRunner, SessionError
from kernelverify_b200.runners.result import DeviceInfo, RunResult, RunStatus, Timing
from kernelverify_b200.runners.spec import (
    Binding,
    BindingKind,
    KernelSpec,
    LaunchMode,
    LaunchSpec,
    RunCase,
    SpecError,
)
from kernelverify_b200.runners.specialize import specialize

__all__ = ["BatchResult", "Binding", "BindingKind", "CompiledSession", "CudaRunner", "DeviceInfo",
           "KernelSpec", "LaunchMode", "LaunchSpec", "RunCase", "RunResult", "RunStatus",
           "SessionError", "SpecError", "Timing", "specialize"]
