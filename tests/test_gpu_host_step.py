"""kv_attention.HostStep on a B200: a decode step fed from pinned host
memory (one staging copy in, one copy out), eager and as a CUDA graph, equal
bit for bit to the device-resident call on the same inputs, over several
calls with changing inputs; and the same door over the one-kernel sequence
split (SequenceSplitDecoder.launch)."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import cases
from tests.kvq_cases import judge_gqa, pack, to_dev

pytestmark = pytest.mark.gpu


def _case(h, hkv, t, seed):
    q, kc, vc, nk, nv = cases.make_case(1, h, t, 128, seed=seed)
    return q, kc[:hkv], vc[:hkv], nk[:, :hkv], nv[:, :hkv]


@pytest.mark.parametrize("graph", [True, False])
def test_host_step_matches_the_device_call(native, graph):
    import torch
    from kernelverify_b200.pack import kv_attention as kva
    h, hkv, t = 32, 8, 3000
    q, kc, vc, nk, nv = _case(h, hkv, t, seed=61)
    kart = [to_dev(x) for x in pack(kc, 4)]
    vart = [to_dev(x) for x in pack(vc, 4)]

    def make(dq, dk, dv, dout):
        return kva.decode_launch(dq, *kart, *vart, dk, dv, bits=4, out=dout, t_cached=t)

    step = kva.HostStep(make, q.shape, nk.shape, torch.float16, "cuda", graph=graph)
    rng = np.random.default_rng(7)
    try:
        for _ in range(4):
            qn = rng.standard_normal(q.shape).astype(np.float16)
            nkn = rng.standard_normal(nk.shape).astype(np.float16)
            nvn = rng.standard_normal(nv.shape).astype(np.float16)
            got = step(torch.from_numpy(qn), torch.from_numpy(nkn), torch.from_numpy(nvn))
            assert got.device.type == "cpu" and got.is_pinned()
            ref = kva.decode(to_dev(qn), *kart, *vart, to_dev(nkn), to_dev(nvn), bits=4,
                             t_cached=t)
            torch.cuda.synchronize()
            assert torch.equal(got, ref.cpu())
        v = judge_gqa(qn, kc, vc, nkn, nvn, 4, got.numpy())
        assert v.ok, v
        # the staging views are the step's inputs: writing them directly works too
        step.q.copy_(torch.from_numpy(q))
        step.new_k.copy_(torch.from_numpy(nk))
        step.new_v.copy_(torch.from_numpy(nv))
        got = step().clone()
        assert judge_gqa(q, kc, vc, nk, nv, 4, got.numpy()).ok
        assert step.h2d_bytes >= (q.size + 2 * nk.size) * 2
        assert step.d2h_bytes == q.size * 2
    finally:
        step.close()


def test_host_step_over_the_fused_sequence_split(native):
    import torch
    from kernelverify_b200.pack import kv_attention as kva
    from kernelverify_b200.pack.tsplit import SequenceSplitDecoder
    h, hkv, t = 64, 8, 8192
    q, kc, vc, nk, nv = _case(h, hkv, t, seed=62)
    kart = [to_dev(x) for x in pack(kc, 4)]
    vart = [to_dev(x) for x in pack(vc, 4)]
    dec = SequenceSplitDecoder(1, h, 128, torch.device("cuda"), transport="fused")

    def make(dq, dk, dv, dout):
        return dec.launch(dq, *kart, *vart, dk, dv, bits=4, t_local=t, out=dout)

    step = kva.HostStep(make, q.shape, nk.shape, torch.float16, "cuda", graph=True)
    try:
        for _ in range(3):
            got = step(torch.from_numpy(q), torch.from_numpy(nk), torch.from_numpy(nv))
            v = judge_gqa(q, kc, vc, nk, nv, 4, got.numpy())
            assert v.ok, v
        assert dec.exchange.status() == 0
    finally:
        step.close()
        dec.close()


def test_stage_copy_both_ways_and_pageable_memory_refused(native):
    """kvq_stage_copy: pinned -> device and device -> pinned, sizes with and
    without a tail under 16 bytes, bit for bit; pageable host memory is
    refused with a status before anything runs."""
    import torch
    from kernelverify_b200 import _native
    lib = _native.lib()
    s = torch.cuda.current_stream().cuda_stream
    for nbytes in (16, 4096 + 6, 20480, 70000 * 16 + 2):
        src = torch.randint(0, 256, (nbytes,), dtype=torch.uint8).pin_memory()
        dev = torch.zeros(nbytes, dtype=torch.uint8, device="cuda")
        back = torch.zeros(nbytes, dtype=torch.uint8).pin_memory()
        _native.check(lib.kvq_stage_copy(dev.data_ptr(), src.data_ptr(), nbytes, s))
        _native.check(lib.kvq_stage_copy(back.data_ptr(), dev.data_ptr(), nbytes, s))
        torch.cuda.synchronize()
        assert torch.equal(dev.cpu(), src) and torch.equal(back, src)
    pageable = torch.zeros(4096, dtype=torch.uint8)
    dev = torch.zeros(4096, dtype=torch.uint8, device="cuda")
    st = lib.kvq_stage_copy(dev.data_ptr(), pageable.data_ptr(), 4096, s)
    assert st == _native.KVQ_ERR_INVALID and b"pageable" in lib.kvq_last_error()
