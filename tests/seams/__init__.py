"""The CUDA mutation battery's seam kernel -- TEST INFRASTRUCTURE ONLY.

`kvq_seams.cu` is the reference's fp32 kv_attention port with its seven
fault seams (kernelverify/reference/native_kernels.py:168-221) written as one
CUDA source, each fault its own compile-time instantiation. This module
builds it (nvcc, sm_100a, into tests/seams/_build/) and runs it on the host
build of the same functions or on the device, over the battery's inputs
(oracle.battery.case_inputs) quantized by the oracle's canonical quantizer.
"""

from __future__ import annotations

import ctypes
import hashlib
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
SRC = HERE / "kvq_seams.cu"
LIB = HERE / "_build" / "libkvq_seams.so"
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-fmad=false",
         "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC", "-Xcompiler", "-ffp-contract=off",
         "-shared"]

# fault bit of each catalogue entry (kernelverify/mutation/catalogue.py:153-166)
FAULT_BITS = {
    (): 0,
    (("scores_dtype", "float16"),): 1,
    (("accum_dtype", "float16"),): 2,
    (("accum_dtype", "float16-seq"),): 4,
    (("k_scales_rotated", True),): 8,
    (("v_bias_dropped", True),): 16,
    (("new_entry_skipped", True),): 32,
    (("dhead_scale_dropped", True),): 64,
}


def fault_bit(params: dict) -> int:
    return FAULT_BITS[tuple(sorted(params.items()))]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stamp() -> str:
    return hashlib.sha256(SRC.read_bytes() + " ".join(FLAGS).encode()).hexdigest()


def build(force: bool = False) -> Path:
    """Compile the seam source (host and sm_100a device code) unless the
    built library already matches the source and flags."""
    stamp = LIB.with_suffix(".stamp")
    want = _stamp()
    if not force and LIB.exists() and stamp.exists() and stamp.read_text() == want:
        return LIB
    LIB.parent.mkdir(exist_ok=True)
    tmp = LIB.with_suffix(".tmp.so")
    res = subprocess.run([_nvcc(), *FLAGS, "-o", str(tmp), str(SRC)], capture_output=True,
                         text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {SRC.name}:\n{res.stderr[-4000:]}")
    os.replace(tmp, LIB)
    stamp.write_text(want)
    return LIB


_lib = None


def lib():
    global _lib
    if _lib is None:
        handle = ctypes.CDLL(str(build()))
        fn = handle.kvq_seams_decode
        fn.restype = ctypes.c_int
        fn.argtypes = [ctypes.c_int] * 3 + [ctypes.c_void_p] * 10 + [ctypes.c_int] * 7 + \
            [ctypes.c_void_p]
        _lib = handle
    return _lib


def artefacts(inputs: dict):
    """(q, k words, k scales, k biases, v words, v scales, v biases, new_k,
    new_v) of a battery case: the caches through the canonical quantizer."""
    from oracle import kv, quant
    bits, group = int(inputs["bits"][0]), kv.group_of(inputs)
    kw, ks, kb = quant.quantize_cache(inputs["k_cache"], bits, group)
    vw, vs, vb = quant.quantize_cache(inputs["v_cache"], bits, group)
    return [np.ascontiguousarray(a) for a in
            (inputs["q"], kw, ks, kb, vw, vs, vb, inputs["new_k"], inputs["new_v"])]


def _geometry(inputs: dict):
    from oracle import kv
    b, h, dh = inputs["q"].shape
    hkv, t, _ = inputs["k_cache"].shape
    return b, h, hkv, t, dh, int(inputs["bits"][0]), kv.group_of(inputs)


def _call(on_device: int, fault: int, dtype_code: int, ptrs, out_ptr, geom, stream) -> None:
    b, h, hkv, t, dh, bits, group = geom
    rc = lib().kvq_seams_decode(on_device, fault, dtype_code, *ptrs, out_ptr, b, h, hkv, t, dh,
                                bits, group, stream)
    if rc != 0:
        raise RuntimeError(f"kvq_seams_decode returned {rc}")


def run_host(inputs: dict, params: dict) -> np.ndarray:
    """The seam source's host build on one battery case: out [B, H, DH]."""
    arrays = artefacts(inputs)
    q = arrays[0]
    out = np.empty_like(q)
    _call(0, fault_bit(params), 0 if q.dtype == np.float16 else 1,
          [a.ctypes.data for a in arrays], out.ctypes.data, _geometry(inputs), None)
    return out


def run_device(inputs: dict, params: dict) -> np.ndarray:
    """The seam source's sm_100a kernel on one battery case, on cuda:0."""
    import torch
    arrays = artefacts(inputs)
    dev = [torch.from_numpy(a.view(np.int32) if a.dtype == np.uint32 else a).cuda()
           for a in arrays]
    out = torch.empty_like(dev[0])
    stream = torch.cuda.current_stream()
    _call(1, fault_bit(params), 0 if arrays[0].dtype == np.float16 else 1,
          [t.data_ptr() for t in dev], out.data_ptr(), _geometry(inputs), stream.cuda_stream)
    stream.synchronize()
    return out.cpu().numpy()
