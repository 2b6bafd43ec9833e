"""The tensor-core kernels' shared-memory layouts, read from the CUDA headers
themselves (a host program compiled with nvcc): every (group, code width)
ring plus scratch and barriers fits three CTAs on a B200 SM (228 KB, 1 KB
reserved per CTA), so no format silently drops to two CTAs per SM."""

from __future__ import annotations

import shutil
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
SM_SMEM = 228 * 1024
CTA_RESERVED = 1024

PROGRAM = r'''
#include <cstdio>
#include "kvq_mma.cuh"
using namespace kvq::mma4;
template <int GROUP, int BITS> void one() {
    std::printf("%d %d %d %d\n", GROUP, BITS, (int)Layout<GROUP, BITS>::NST,
                (int)smem_bytes<GROUP, BITS>());
}
int main() {
    one<32, 2>(); one<64, 2>(); one<128, 2>();
    one<32, 3>(); one<64, 3>(); one<128, 3>();
    one<32, 4>(); one<64, 4>(); one<128, 4>();
    one<32, 6>(); one<64, 6>(); one<128, 6>();
    one<32, 8>(); one<64, 8>(); one<128, 8>();
    return 0;
}
'''


def test_every_layout_fits_three_ctas(tmp_path):
    from kernelverify_b200 import build
    nvcc = build.nvcc()
    if not shutil.which(nvcc) and not Path(nvcc).exists():
        pytest.skip("nvcc is not available")
    src = tmp_path / "layout.cu"
    src.write_text(PROGRAM)
    exe = tmp_path / "layout"
    subprocess.run([nvcc, *build.ARCH, "-std=c++17", "--expt-relaxed-constexpr",
                    "-I", str(ROOT / "include"), "-I", str(build.CSRC), str(src), "-o", str(exe)],
                   check=True, capture_output=True, timeout=600)
    rows = [tuple(int(x) for x in line.split())
            for line in subprocess.run([str(exe)], capture_output=True, text=True,
                                       check=False).stdout.splitlines() if line.strip()]
    if not rows:
        pytest.skip("the layout program does not run on this host")
    assert len(rows) == 15
    for group, bits, nst, nbytes in rows:
        assert nst >= 3, (group, bits, nst)
        assert 3 * (nbytes + CTA_RESERVED) <= SM_SMEM, (group, bits, nst, nbytes)
