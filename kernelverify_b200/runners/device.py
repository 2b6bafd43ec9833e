"""Compile and dispatch a candidate kernel on the CUDA device (worker side).

The CUDA counterpart of the reference's Metal device layer
(kernelverify/runners/device.py:123-341), with its load-bearing behaviours:

* every failure is a status: a compile error, an unknown entry point, a block
  larger than the function allows or a shared-memory request above the device
  limit come back as COMPILE_ERROR / LAUNCH_ERROR before anything launches;
* correctness and timing are separate dispatches: outputs are zeroed, one
  clean dispatch produces the tensors the oracle sees, then warm-up and
  timed repeats follow (:309-341);
* buffers are pooled per binding index, grown to the largest extent ever
  bound there, and the slack beyond the current case's extent is zeroed
  whenever a case is smaller than the buffer it gets, so a kernel reading
  past its declared extent reads zeros, never a previous case's bytes
  (:22-55,134-166); `release_pool` frees them between specs.

Two kinds of spec compile here:

* CUDA C++ source (no kvq pragma): compiled by NVRTC for sm_100a, loaded with
  the driver API and launched on torch's current stream; argument i is
  binding i (sorted by `index`): tensors as device pointers, scalars by value.
  `math_mode` "safe" compiles with IEEE division and square root and no
  flush-to-zero (the CUDA reading of the reference's default), "relaxed"
  adds FMA contraction explicitly, "fast" is --use_fast_math.
* a kvq library translation unit (`#pragma kvq library <entry>` and
  `#pragma kvq instantiate T=.. BITS=.. DH=.. [GROUP=..]`): the precompiled
  sm_100a kernels of libkvq_b200.so behind the C ABI, called with the
  reference's raw-door bindings (q, k_wq, ..., out, n_heads, t_cached,
  n_kv_heads, t_stride; b_rows from the case's params).
"""

from __future__ import annotations

import ctypes
import re
import time

import numpy as np

from kernelverify_b200.runners.result import DeviceInfo, RunResult, RunStatus, Timing
from kernelverify_b200.runners.spec import (
    SCALAR_DTYPES,
    TENSOR_DTYPES,
    BindingKind,
    KernelSpec,
    LaunchMode,
    RunCase,
    SpecError,
)

MATH_MODES = {
    "safe": ["--prec-div=true", "--prec-sqrt=true", "--ftz=false"],
    "relaxed": ["--prec-div=true", "--prec-sqrt=true", "--ftz=false", "--fmad=true"],
    "fast": ["--use_fast_math"],
}
DEFAULT_MATH_MODE = "safe"
ARCH = "sm_100a"

_LIB_RE = re.compile(r"^\s*#pragma\s+kvq\s+library\s+(\w+)", re.M)
_INST_RE = re.compile(r"^\s*#pragma\s+kvq\s+instantiate\s+(.*)$", re.M)
_T_NAMES = {"half": "float16", "float16": "float16", "float": "float32", "float32": "float32"}


class CompileError(RuntimeError):
    """The source did not become a launchable kernel."""


class LaunchError(RuntimeError):
    """The kernel exists but this dispatch cannot be made or did not finish."""


def _torch():
    import torch
    return torch


class CudaDevice:
    """cuda:<index> and torch's stream on it."""

    def __init__(self, index: int = 0):
        torch = _torch()
        if not torch.cuda.is_available():
            raise RuntimeError("no CUDA device on this machine")
        torch.cuda.set_device(index)
        torch.cuda.init()
        self.index = index
        self.device = torch.device("cuda", index)
        self.props = torch.cuda.get_device_properties(index)
        if self.props.major != 10:
            raise RuntimeError(f"{self.props.name} is sm_{self.props.major}{self.props.minor}; "
                               "this runner targets sm_100a (B200)")
        torch.zeros(1, device=self.device)  # make the primary context current
        self._pool: dict = {}
        self._driver = None

    @property
    def driver(self):
        if self._driver is None:
            from kernelverify_b200.runners._cuda import Driver
            self._driver = Driver()
        return self._driver

    def info(self) -> DeviceInfo:
        p = self.props
        bus = getattr(p, "pci_bus_id", 0) or 0
        return DeviceInfo(name=str(p.name), max_threads_per_threadgroup=1024,
                          max_threadgroup_memory=int(getattr(p, "shared_memory_per_block_optin",
                                                             232448)),
                          has_unified_memory=False,
                          registry_id=int(bus) * 256 + int(getattr(p, "pci_device_id", 0) or 0))

    # -- pooled buffers ---------------------------------------------------
    def pooled_buffer(self, index, nbytes: int):
        """(uint8 tensor, bytes held) for binding `index`; the region past
        `nbytes` is zeroed before it changes hands."""
        torch = _torch()
        if nbytes <= 0:
            raise LaunchError(f"buffer index {index} asks for {nbytes} bytes")
        held = self._pool.get(index)
        if held is not None and held.numel() >= nbytes:
            if held.numel() > nbytes:
                held[nbytes:].zero_()
            return held, held.numel()
        try:
            buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        except RuntimeError as error:
            raise LaunchError(f"the device would not allocate {nbytes} bytes for buffer "
                              f"index {index}: {error}") from error
        self._pool[index] = buf
        return buf, nbytes

    def release_pool(self) -> None:
        self._pool.clear()
        _torch().cuda.empty_cache()

    # -- compile ------------------------------------------------------------
    def compile(self, spec: KernelSpec, math_mode: str = DEFAULT_MATH_MODE):
        if math_mode not in MATH_MODES:
            raise CompileError(f"math mode {math_mode!r} is not one of {sorted(MATH_MODES)}")
        lib_entry = _LIB_RE.search(spec.source)
        if lib_entry:
            return LibraryKernel(self, spec, lib_entry.group(1), math_mode)
        from kernelverify_b200.runners._cuda import CudaApiError
        import os
        opts = [f"--gpu-architecture={ARCH}", "-std=c++17", "-default-device",
                *MATH_MODES[math_mode]]
        inc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "include")
        if os.path.isdir(inc):
            opts.append(f"--include-path={inc}")
        try:
            cubin, _log = self.driver.compile(spec.source, (spec.name or spec.entry_point) + ".cu",
                                              opts)
            module, fn = self.driver.load(cubin, spec.entry_point)
        except CudaApiError as error:
            raise CompileError(str(error)) from error
        return NvrtcKernel(self, spec, module, fn, math_mode, opts)


class _Kernel:
    """Shared case flow: validate, buffers, zeroed outputs, one clean
    dispatch, read back, then warm-up + timed repeats."""

    max_threads = 1024
    execution_width = 32

    def __init__(self, device: CudaDevice, spec: KernelSpec, math_mode: str):
        self.device = device
        self.spec = spec
        self.math_mode = math_mode

    def _buffers(self, case: RunCase):
        torch = _torch()
        tensors, outputs = {}, []
        for pos, b in enumerate(self.spec.bindings):
            idx = self.spec.buffer_index(pos)
            if b.kind is BindingKind.SCALAR:
                continue
            if b.kind is BindingKind.INPUT:
                arr = np.ascontiguousarray(case.inputs[b.name])
                buf, _ = self.device.pooled_buffer(idx, arr.nbytes)
                src = torch.from_numpy(arr.view(np.uint8).reshape(-1))
                buf[:arr.nbytes].copy_(src)
                tensors[idx] = (buf, arr.dtype, arr.shape)
            else:
                shape, dtype = case.output_shapes[len(outputs)]
                nb = int(np.prod(shape)) * np.dtype(TENSOR_DTYPES[dtype]).itemsize
                buf, _ = self.device.pooled_buffer(idx, nb)
                buf[:nb].zero_()
                tensors[idx] = (buf, np.dtype(TENSOR_DTYPES[dtype]), shape)
                outputs.append(idx)
        return tensors, outputs

    def run(self, case: RunCase, warmup: int = 1, repeats: int = 5) -> RunResult:
        torch = _torch()
        try:
            case.validate_against(self.spec)
            launch = self.spec.launch.resolve(case.params)
        except SpecError as error:
            return RunResult(status=RunStatus.INVALID_SPEC, detail=str(error), label=case.label)
        try:
            tensors, outputs = self._buffers(case)
            dispatch = self._prepare(case, tensors, launch)
            stream = torch.cuda.current_stream(self.device.device)
            dispatch(stream)
            stream.synchronize()
            result = []
            for slot, idx in enumerate(outputs):
                buf, dt, shape = tensors[idx]
                nb = int(np.prod(shape)) * dt.itemsize
                result.append(buf[:nb].cpu().numpy().view(dt).reshape(shape).copy())
            gpu, wall = [], []
            for rep in range(warmup + repeats):
                e0 = torch.cuda.Event(enable_timing=True)
                e1 = torch.cuda.Event(enable_timing=True)
                t0 = time.perf_counter()
                e0.record(stream)
                dispatch(stream)
                e1.record(stream)
                e1.synchronize()
                t1 = time.perf_counter()
                if rep >= warmup:
                    gpu.append(e0.elapsed_time(e1) * 1e-3)
                    wall.append(t1 - t0)
        except LaunchError as error:
            return RunResult(status=RunStatus.LAUNCH_ERROR, detail=str(error), label=case.label)
        return RunResult(status=RunStatus.OK, outputs=result,
                         timing=Timing(tuple(gpu), tuple(wall), warmup), label=case.label)


class NvrtcKernel(_Kernel):
    def __init__(self, device, spec, module, fn, math_mode, options):
        super().__init__(device, spec, math_mode)
        self.module, self.fn, self.options = module, fn, options
        self.max_threads = device.driver.func_attr(fn, 0)

    def _prepare(self, case, tensors, launch):
        grid, block, memory = launch
        threads = block[0] * block[1] * block[2]
        if threads > self.max_threads:
            raise LaunchError(f"threadgroup {block} is {threads} threads, above the "
                              f"{self.max_threads} this kernel allows")
        smem = int(sum(memory))
        limit = self.device.info().max_threadgroup_memory
        if smem > limit:
            raise LaunchError(f"threadgroup memory {smem} bytes is above the device limit of {limit}")
        if smem > 48 * 1024:
            self.device.driver.set_dynamic_smem(self.fn, smem)
        if self.spec.launch.mode is LaunchMode.THREADS:
            blocks = tuple(-(-g // b) for g, b in zip(grid, block))
        else:
            blocks = grid
        order = sorted(range(len(self.spec.bindings)), key=self.spec.buffer_index)
        args = []
        for pos in order:
            b = self.spec.bindings[pos]
            idx = self.spec.buffer_index(pos)
            if b.kind is BindingKind.SCALAR:
                value = np.asarray(case.params[b.name], dtype=SCALAR_DTYPES[b.dtype])
                ctype = {"uint32": ctypes.c_uint32, "int32": ctypes.c_int32,
                         "float32": ctypes.c_float, "float16": ctypes.c_uint16}[b.dtype]
                raw = value.view(np.uint16) if b.dtype == "float16" else value
                args.append(ctype(raw.item()))
            else:
                args.append(ctypes.c_uint64(tensors[idx][0].data_ptr()))
        driver = self.device.driver

        def dispatch(stream):
            from kernelverify_b200.runners._cuda import CudaApiError
            try:
                driver.launch(self.fn, blocks, block, smem, stream.cuda_stream, args)
            except CudaApiError as error:
                raise LaunchError(str(error)) from error

        return dispatch


class LibraryKernel(_Kernel):
    """A kvq library instantiation, called through the C ABI."""

    REQUIRED = ("q", "k_wq", "k_scales", "k_biases", "v_wq", "v_scales", "v_biases",
                "new_k", "new_v")

    def __init__(self, device, spec, entry, math_mode):
        super().__init__(device, spec, math_mode)
        from kernelverify_b200 import _native
        if entry != "kvq_decode":
            raise CompileError(f"the kvq library has no decode entry {entry!r}")
        m = _INST_RE.search(spec.source)
        if not m:
            raise CompileError("a kvq library unit needs '#pragma kvq instantiate T=.. BITS=.. DH=..'")
        inst = dict(kv.split("=", 1) for kv in m.group(1).split())
        try:
            self.dtype = _T_NAMES[inst["T"]]
            self.bits = int(inst["BITS"])
            self.head_dim = int(inst["DH"])
            self.group = int(inst.get("GROUP", 64))
        except (KeyError, ValueError) as error:
            raise CompileError(f"bad instantiation {m.group(1)!r}: {error}") from error
        try:
            self.lib = _native.lib()
        except _native.NativeUnavailable as error:
            raise CompileError(str(error)) from error
        dt = 0 if self.dtype == "float16" else 1
        if not self.lib.kvq_supports(self.head_dim, self.bits, self.group, dt):
            raise CompileError(f"libkvq_b200 carries no kernel for T={inst['T']} BITS={self.bits} "
                               f"DH={self.head_dim} GROUP={self.group}")
        names = {b.name for b in spec.bindings if b.kind is BindingKind.INPUT}
        missing = [n for n in self.REQUIRED if n not in names]
        if missing or spec.output_count() != 1:
            raise CompileError(f"the kvq_decode entry needs inputs {self.REQUIRED} and one output; "
                               f"missing {missing}")
        self.entry = entry

    def _prepare(self, case, tensors, launch):
        from kernelverify_b200 import _native
        by_name = {}
        out_idx = None
        for pos, b in enumerate(self.spec.bindings):
            idx = self.spec.buffer_index(pos)
            if b.kind is BindingKind.INPUT:
                by_name[b.name] = tensors[idx]
            elif b.kind is BindingKind.OUTPUT:
                out_idx = idx
        p = case.params
        try:
            b_rows = int(p["b_rows"])
            n_heads, n_kv = int(p["n_heads"]), int(p["n_kv_heads"])
            t_cached, t_stride = int(p["t_cached"]), int(p["t_stride"])
        except (KeyError, ValueError) as error:
            raise LaunchError(f"kvq_decode needs params b_rows, n_heads, n_kv_heads, t_cached, "
                              f"t_stride: {error}") from error
        dh, bits, group = self.head_dim, self.bits, self.group
        esz = 2 if self.dtype == "float16" else 4
        batch_stride = int(p.get("cache_batch_stride", 0))
        cache_rows = n_kv * t_stride + (b_rows - 1) * batch_stride
        need = {"q": b_rows * n_heads * dh * esz,
                "k_wq": cache_rows * dh * bits // 32 * 4, "v_wq": cache_rows * dh * bits // 32 * 4,
                "k_scales": cache_rows * (dh // group) * esz,
                "k_biases": cache_rows * (dh // group) * esz,
                "v_scales": cache_rows * (dh // group) * esz,
                "v_biases": cache_rows * (dh // group) * esz,
                "new_k": b_rows * n_kv * dh * esz, "new_v": b_rows * n_kv * dh * esz}
        for name, nbytes in need.items():
            buf, dt, shape = by_name[name]
            have = int(np.prod(shape)) * dt.itemsize
            if have < nbytes:
                raise LaunchError(f"input {name!r} holds {have} bytes; the case's geometry reads "
                                  f"{nbytes}")
        seq_lens = None
        if "seq_lens" in by_name:
            buf, dt, shape = by_name["seq_lens"]
            if dt != np.dtype(np.int32) or int(np.prod(shape)) < b_rows:
                raise LaunchError(f"input 'seq_lens' must be int32 with at least b_rows={b_rows} "
                                  f"entries")
            seq_lens = buf
        obuf, odt, oshape = tensors[out_idx]
        if int(np.prod(oshape)) * odt.itemsize < b_rows * n_heads * dh * esz:
            raise LaunchError("the output is smaller than b_rows x n_heads x DH")
        a = _native.KvqArgs()
        for name in self.REQUIRED:
            setattr(a, name, by_name[name][0].data_ptr())
        a.seq_lens = seq_lens.data_ptr() if seq_lens is not None else None
        a.b_rows, a.n_heads, a.n_kv_heads = b_rows, n_heads, n_kv
        a.t_cached, a.t_stride, a.head_dim = t_cached, t_stride, dh
        a.bits, a.group_size = bits, group
        a.dtype = 0 if self.dtype == "float16" else 1
        a.has_new_entry = int(p.get("has_new_entry", 1))
        a.cache_batch_stride = batch_stride
        a.t_begin = int(p.get("t_begin", 0))
        a.t_end = int(p.get("t_end", _native.KVQ_T_END_ALL))
        ws_need = self.lib.kvq_workspace_bytes(a)
        ws = None
        if ws_need:
            ws, _ = self.device.pooled_buffer("workspace", ws_need + 256)
        lib = self.lib

        def dispatch(stream):
            base = ws.data_ptr() if ws is not None else 0
            aligned = (base + 255) // 256 * 256 if base else None
            status = lib.kvq_decode(a, obuf.data_ptr(), aligned, ws_need if ws is not None else 0,
                                    stream.cuda_stream)
            if status != 0:
                raise LaunchError(lib.kvq_last_error().decode(errors="replace"))

        return dispatch
