"""Build the in-tree C-ABI library kernelverify_b200/_lib/libkvq_b200.so.

    python -m kernelverify_b200.build [--force] [--ptxas-verbose]

nvcc compiles every csrc/*.cu for sm_100a only (the kernels use Blackwell
instructions), one process per translation unit in parallel, and links a
shared library with the CUDA runtime linked statically, so the library loads
beside torch's own runtime without version coupling. A stamp of the sources'
hash and the flags skips the build when nothing changed.
"""

from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIBDIR = PKG / "_lib"
BUILD = ROOT / "_build"
LIB_NAME = "libkvq_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", str(ROOT / "include"), "-I", str(CSRC)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def stamp(extra: list[str]) -> str:
    h = hashlib.sha256()
    for p in sorted(list(CSRC.glob("*")) + [ROOT / "include" / "kvq_b200.h"]):
        if p.is_file():
            h.update(p.name.encode())
            h.update(p.read_bytes())
    h.update(" ".join(ARCH + NVCC_FLAGS + extra).encode())
    return h.hexdigest()


def lib_path() -> Path:
    return LIBDIR / LIB_NAME


def build(force: bool = False, ptxas_verbose: bool = False, jobs: int | None = None) -> Path:
    extra = ["-Xptxas", "-v"] if ptxas_verbose else []
    want = stamp(extra)
    stamp_file = LIBDIR / (LIB_NAME + ".stamp")
    out = lib_path()
    if not force and out.exists() and stamp_file.exists() and stamp_file.read_text() == want:
        return out
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    cc = nvcc()
    srcs = sources()

    def compile_one(src: Path):
        obj = BUILD / (src.stem + ".o")
        cmd = [cc, *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        return src, obj, res

    with ThreadPoolExecutor(max_workers=jobs or min(len(srcs), os.cpu_count() or 4)) as pool:
        results = list(pool.map(compile_one, srcs))
    logs = []
    for src, obj, res in results:
        if res.stderr.strip():
            logs.append(f"== {src.name}\n{res.stderr}")
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stderr}")
    if logs:
        (BUILD / "nvcc.log").write_text("\n".join(logs))
    tmp = out.with_suffix(".so.tmp")
    link = [cc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp),
            *[str(o) for _, o, _ in results]]
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stderr}")
    os.replace(tmp, out)
    stamp_file.write_text(want)
    return out


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-verbose", action="store_true",
                    help="pass -Xptxas -v; the report lands in _build/nvcc.log")
    args = ap.parse_args(argv)
    path = build(force=args.force, ptxas_verbose=args.ptxas_verbose)
    print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
