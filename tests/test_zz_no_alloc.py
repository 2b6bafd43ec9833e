"""kvq_decode_noalloc -- the decode step for callers that cannot allocate
device memory (a host binding the library through a plain C FFI with no CUDA
allocator of its own, or a serving process that reserves all device memory up
front and forbids allocation on its decode path). Its scratch is a buffer
built into the library, shared by every call on a device.

Checked here through the C ABI against kvq_decode with a caller-provided
workspace: two calls in a row (a larger step, then a smaller one, so stale
scratch from the first cannot pass for the second's), each equal to the
workspace entry's output and within the oracle's tolerance; and a step whose
scratch would exceed the built-in size is refused with a status. This file is
collected last so a run that stops at the first failure has run every other
test first.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import cases, kv
from tests.kvq_cases import pack, to_dev

pytestmark = pytest.mark.gpu


def _case(b, h, hkv, t, seed):
    q, kc, vc, nk, nv = cases.make_case(b, h, t, 128, seed=seed)
    kc, vc, nk, nv = kc[:hkv], vc[:hkv], nk[:, :hkv], nv[:, :hkv]
    return q, kc, vc, nk, nv


def _run_both(native, q, kc, vc, nk, nv, bits=4):
    import torch
    from kernelverify_b200 import _native
    from kernelverify_b200.pack import kv_attention as kva

    ins = [to_dev(x) for x in (q, *pack(kc, bits), *pack(vc, bits), nk, nv)]
    a = kva._args(*ins, bits=bits)
    stream = torch.cuda.current_stream().cuda_stream
    need = native.kvq_workspace_bytes(ctypes.byref(a))
    assert 0 < need <= _native.KVQ_NOALLOC_SCRATCH_BYTES
    ws = torch.empty(need + 256, dtype=torch.uint8, device="cuda")
    base = (ws.data_ptr() + 255) // 256 * 256
    ref_out = torch.empty_like(ins[0])
    _native.check(native.kvq_decode(ctypes.byref(a), ref_out.data_ptr(), base, need, stream))
    out = torch.full_like(ins[0], float("nan"))
    _native.check(native.kvq_decode_noalloc(ctypes.byref(a), out.data_ptr(), stream))
    torch.cuda.synchronize()
    return out.cpu().numpy(), ref_out.cpu().numpy()


def test_no_alloc_entry_matches_the_workspace_entry_on_two_calls(native):
    steps = [_case(4, 32, 8, 3000, seed=71), _case(1, 8, 2, 700, seed=72)]
    for q, kc, vc, nk, nv in steps:
        got, want = _run_both(native, q, kc, vc, nk, nv)
        ref, tol = kv.reference_and_tolerance(kv.gqa_tiled_inputs(q, kc, vc, nk, nv, 4))
        assert kv.max_abs_error(got, want) <= tol
        assert np.array_equal(got, want)
        assert kv.judge(got, ref, tol).ok


def test_no_alloc_entry_refuses_steps_beyond_its_scratch(native):
    from kernelverify_b200 import _native

    a = _native.KvqArgs()
    for name in ("q", "k_wq", "k_scales", "k_biases", "v_wq", "v_scales", "v_biases",
                 "new_k", "new_v"):
        setattr(a, name, 1 << 20)
    a.b_rows, a.n_heads, a.n_kv_heads = 512, 64, 8
    a.t_cached, a.t_stride, a.head_dim = 4096, 4096, 128
    a.bits, a.group_size, a.dtype, a.has_new_entry = 4, 64, 0, 1
    a.t_begin, a.t_end = 0, _native.KVQ_T_END_ALL
    assert native.kvq_workspace_bytes(ctypes.byref(a)) > _native.KVQ_NOALLOC_SCRATCH_BYTES
    status = native.kvq_decode_noalloc(ctypes.byref(a), 1 << 20, None)
    assert status == _native.KVQ_ERR_INVALID
    assert b"scratch" in native.kvq_last_error()
