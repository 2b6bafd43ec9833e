"""Minimal ctypes binding of NVRTC and the CUDA driver's module/launch API,
enough for the runner to compile a candidate's CUDA C++ at run time and
launch it on torch's current stream (the primary context torch made
current). Used only inside the worker process."""

from __future__ import annotations

import ctypes
import glob
import os

CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK = 0
CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES = 8


class CudaApiError(RuntimeError):
    pass


def _load(names):
    errors = []
    for name in names:
        try:
            return ctypes.CDLL(name)
        except OSError as error:
            errors.append(f"{name}: {error}")
    raise CudaApiError("; ".join(errors))


def _nvrtc_candidates():
    out = ["libnvrtc.so.12"]
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    out += sorted(glob.glob(os.path.join(home, "lib64", "libnvrtc.so.12*")))
    try:
        import nvidia.cuda_nvrtc  # torch's wheel dependency
        base = os.path.dirname(nvidia.cuda_nvrtc.__file__)
        out += sorted(glob.glob(os.path.join(base, "lib", "libnvrtc.so*")))
    except Exception:
        pass
    return out


class Driver:
    def __init__(self):
        self.cu = _load(["libcuda.so.1", "libcuda.so"])
        self.nvrtc = _load(_nvrtc_candidates())
        cu, nv = self.cu, self.nvrtc
        P, I, U = ctypes.c_void_p, ctypes.c_int, ctypes.c_uint
        cu.cuModuleLoadData.argtypes = [ctypes.POINTER(P), P]
        cu.cuModuleGetFunction.argtypes = [ctypes.POINTER(P), P, ctypes.c_char_p]
        cu.cuModuleUnload.argtypes = [P]
        cu.cuLaunchKernel.argtypes = [P, U, U, U, U, U, U, U, P, ctypes.POINTER(P), P]
        cu.cuFuncGetAttribute.argtypes = [ctypes.POINTER(I), I, P]
        cu.cuFuncSetAttribute.argtypes = [P, I, I]
        cu.cuGetErrorString.argtypes = [I, ctypes.POINTER(ctypes.c_char_p)]
        nv.nvrtcCreateProgram.argtypes = [ctypes.POINTER(P), ctypes.c_char_p, ctypes.c_char_p, I,
                                          P, P]
        nv.nvrtcCompileProgram.argtypes = [P, I, ctypes.POINTER(ctypes.c_char_p)]
        nv.nvrtcGetProgramLogSize.argtypes = [P, ctypes.POINTER(ctypes.c_size_t)]
        nv.nvrtcGetProgramLog.argtypes = [P, ctypes.c_char_p]
        nv.nvrtcGetCUBINSize.argtypes = [P, ctypes.POINTER(ctypes.c_size_t)]
        nv.nvrtcGetCUBIN.argtypes = [P, ctypes.c_char_p]
        nv.nvrtcDestroyProgram.argtypes = [ctypes.POINTER(P)]

    def _check(self, rc, what):
        if rc != 0:
            msg = ctypes.c_char_p()
            self.cu.cuGetErrorString(rc, ctypes.byref(msg))
            text = msg.value.decode() if msg.value else f"error {rc}"
            raise CudaApiError(f"{what}: {text}")

    def compile(self, source: str, name: str, options: list[str]) -> tuple[bytes, str]:
        """(cubin, log) or raises CudaApiError with the compiler log."""
        prog = ctypes.c_void_p()
        rc = self.nvrtc.nvrtcCreateProgram(ctypes.byref(prog), source.encode(), name.encode(), 0,
                                           None, None)
        if rc != 0:
            raise CudaApiError(f"nvrtcCreateProgram failed ({rc})")
        try:
            opts = (ctypes.c_char_p * len(options))(*[o.encode() for o in options])
            rc = self.nvrtc.nvrtcCompileProgram(prog, len(options), opts)
            size = ctypes.c_size_t()
            self.nvrtc.nvrtcGetProgramLogSize(prog, ctypes.byref(size))
            buf = ctypes.create_string_buffer(size.value)
            self.nvrtc.nvrtcGetProgramLog(prog, buf)
            log = buf.value.decode(errors="replace").strip()
            if rc != 0:
                raise CudaApiError(log or f"nvrtc compile failed ({rc})")
            self.nvrtc.nvrtcGetCUBINSize(prog, ctypes.byref(size))
            cubin = ctypes.create_string_buffer(size.value)
            self.nvrtc.nvrtcGetCUBIN(prog, cubin)
            return cubin.raw, log
        finally:
            self.nvrtc.nvrtcDestroyProgram(ctypes.byref(prog))

    def load(self, cubin: bytes, entry: str):
        mod = ctypes.c_void_p()
        self._check(self.cu.cuModuleLoadData(ctypes.byref(mod), cubin), "cuModuleLoadData")
        fn = ctypes.c_void_p()
        rc = self.cu.cuModuleGetFunction(ctypes.byref(fn), mod, entry.encode())
        if rc != 0:
            self.cu.cuModuleUnload(mod)
            raise CudaApiError(f"no kernel function named {entry!r} (declare it extern \"C\")")
        return mod, fn

    def func_attr(self, fn, attr: int) -> int:
        v = ctypes.c_int()
        self._check(self.cu.cuFuncGetAttribute(ctypes.byref(v), attr, fn), "cuFuncGetAttribute")
        return v.value

    def set_dynamic_smem(self, fn, nbytes: int) -> None:
        self._check(self.cu.cuFuncSetAttribute(fn, CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES,
                                               nbytes), "cuFuncSetAttribute")

    def launch(self, fn, grid, block, smem: int, stream: int, args: list) -> None:
        """args: ctypes scalars (pointers as c_uint64)."""
        arr = (ctypes.c_void_p * max(1, len(args)))()
        for i, a in enumerate(args):
            arr[i] = ctypes.cast(ctypes.pointer(a), ctypes.c_void_p)
        self._check(self.cu.cuLaunchKernel(fn, grid[0], grid[1], grid[2], block[0], block[1],
                                           block[2], smem, ctypes.c_void_p(stream), arr, None),
                    "cuLaunchKernel")
