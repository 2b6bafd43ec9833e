"""B200 roofline: machine ceilings measured on the GPU at hand, beside the
spec figures -- the CUDA counterpart of the reference's bench/roofline.py
(`measure`, bench/roofline.py:95-138; spec table :54-62) and its Metal probe.

    python -m kernelverify_b200.roofline [--gib 2] [--out ceilings.json]

Measures HBM read-stream bandwidth (the ceiling a read-dominated decode step
sees), copy bandwidth (read + write bytes, the figure MEASURED_PEAKS.json's
`hbm_gbs` uses), the fp32 FMA rate, and a host triad on the CPU cores. Each
device figure is the best of `repeats` timed passes (CUDA events on the
launching stream) over a buffer larger than L2, after warm-up passes. The
probes live in their own library (kernelverify_b200/roofline/_lib), apart
from the decode library.
"""

from __future__ import annotations

import ctypes
import hashlib
import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "probe.cu"
LIB = HERE / "_lib" / "libkvq_probe.so"
FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a", "-O3", "-std=c++17", "-Xcompiler",
         "-fPIC", "-shared"]

# Spec ceilings of one B200 (HGX figures; DGX quotes 8 TB/s HBM). fp32 FMA:
# 148 SMs x 128 lanes x 2 flops at the 1965 MHz boost clock.
SPEC = {"hbm_gbs": 7700.0, "hbm_gbs_dgx": 8000.0, "fp32_tflops": 148 * 128 * 2 * 1.965e9 / 1e12,
        "l2_bytes": 126 * 2 ** 20, "sms": 148}


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def build(force: bool = False) -> Path:
    """Compile the probe library (sm_100a) unless it matches source and flags."""
    stamp = LIB.with_suffix(".stamp")
    want = hashlib.sha256(SRC.read_bytes() + " ".join(FLAGS).encode()).hexdigest()
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
        h = ctypes.CDLL(str(build()))
        h.kvq_probe_blocks.restype = ctypes.c_int
        h.kvq_probe_blocks.argtypes = [ctypes.c_int]
        h.kvq_probe_read.restype = ctypes.c_int
        h.kvq_probe_read.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p,
                                     ctypes.c_int, ctypes.c_void_p]
        h.kvq_probe_copy.restype = ctypes.c_int
        h.kvq_probe_copy.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t,
                                     ctypes.c_int, ctypes.c_void_p]
        h.kvq_probe_fma.restype = ctypes.c_int
        h.kvq_probe_fma.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
        h.kvq_probe_host_triad.restype = ctypes.c_int
        h.kvq_probe_host_triad.argtypes = [ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                                           ctypes.POINTER(ctypes.c_double)]
        _lib = h
    return _lib


def host_triad(n: int = 1 << 25, reps: int = 5, threads: int | None = None) -> dict:
    """The host cores' triad bandwidth (a[i] = b[i] + s c[i], doubles)."""
    threads = threads or os.cpu_count() or 1
    g = ctypes.c_double()
    if lib().kvq_probe_host_triad(n, reps, threads, ctypes.byref(g)) != 0:
        raise RuntimeError("host triad failed")
    return {"host_triad_gbs": round(g.value, 2), "host_threads": threads}


def _best_ms(torch, launch, warmup: int, repeats: int, stream) -> float:
    for _ in range(warmup):
        launch()
    best = float("inf")
    for _ in range(repeats):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        launch()
        e1.record(stream)
        e1.synchronize()
        best = min(best, e0.elapsed_time(e1))
    return best


def measure(gib: float = 2.0, repeats: int = 10, warmup: int = 3, fma_iters: int = 4096) -> dict:
    """Device ceilings on the current CUDA device (needs a GPU)."""
    import torch
    h = lib()
    nbytes = int(gib * 2 ** 30) // 16 * 16
    if nbytes <= 2 * SPEC["l2_bytes"]:
        raise ValueError("the probe buffer must be well above L2 (126 MB)")
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)
    src = torch.ones(nbytes, dtype=torch.uint8, device=dev)
    dst = torch.empty(nbytes, dtype=torch.uint8, device=dev)
    blocks = h.kvq_probe_blocks(4)
    sink = torch.zeros(blocks, dtype=torch.int32, device=dev)
    fout = torch.zeros(blocks * 512, dtype=torch.float32, device=dev)

    def check(rc):
        if rc != 0:
            raise RuntimeError(f"probe launch failed ({rc})")

    read_ms = _best_ms(torch, lambda: check(h.kvq_probe_read(src.data_ptr(), nbytes,
                                                             sink.data_ptr(), blocks,
                                                             stream.cuda_stream)),
                       warmup, repeats, stream)
    copy_ms = _best_ms(torch, lambda: check(h.kvq_probe_copy(src.data_ptr(), dst.data_ptr(),
                                                             nbytes, blocks, stream.cuda_stream)),
                       warmup, repeats, stream)
    fma_ms = _best_ms(torch, lambda: check(h.kvq_probe_fma(fout.data_ptr(), blocks, fma_iters,
                                                           stream.cuda_stream)),
                      warmup, repeats, stream)
    flops = 2.0 * 8 * fma_iters * blocks * 512
    props = torch.cuda.get_device_properties(dev)
    out = {"device": props.name, "bytes": nbytes, "blocks": blocks,
           "read_gbs": round(nbytes / (read_ms * 1e-3) / 1e9, 1),
           "copy_gbs": round(2 * nbytes / (copy_ms * 1e-3) / 1e9, 1),
           "fp32_tflops": round(flops / (fma_ms * 1e-3) / 1e12, 2),
           "spec": SPEC}
    out["read_frac_of_spec"] = round(out["read_gbs"] / SPEC["hbm_gbs"], 3)
    del src, dst
    return out


def main(argv=None) -> int:
    import argparse
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--gib", type=float, default=2.0)
    ap.add_argument("--repeats", type=int, default=10)
    ap.add_argument("--out", default=None)
    args = ap.parse_args(argv)
    res = measure(args.gib, args.repeats)
    res.update(host_triad())
    text = json.dumps(res, indent=1)
    if args.out:
        Path(args.out).write_text(text + "\n")
    print(text)
    return 0


if __name__ == "__main__":
    sys.exit(main())
