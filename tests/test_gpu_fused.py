"""The one-kernel sequence split (kvq_tsplit_decode) on one B200: one rank
holds the whole sequence, so the step is the split stage, the merge of each
cache head's splits by its last CTAs and the output, all in one launch --
against the oracle, against the two-launch kvq_decode on the same inputs,
across split counts (1 to the planner's full wave), head tiles of 4 and 8,
partial head tiles, batches with ragged lengths, repeated steps (the step
count in the region advances, the record parity alternates) and a CUDA graph
replayed over many steps. Two ranks on one GPU (both regions local) show the
bounded wait for a peer whose record never arrives: the status word, NaN
rows, a usable context. Formats the one-kernel form does not serve are
refused."""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

from oracle import cases
from tests.kvq_cases import judge_gqa, judge_per_sequence, pack, to_dev

pytestmark = pytest.mark.gpu


class _Region:
    """A zeroed region for kvq_tsplit_decode, sized for `world` ranks."""

    def __init__(self, rows, dh=128, world=1):
        from kernelverify_b200 import _native
        self.lib = _native.lib()
        self.nbytes = self.lib.kvq_tsplit_region_bytes(rows, dh, world)
        assert self.nbytes > 0
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_char * _native.KVQ_PEER_HANDLE_BYTES)()
        _native.check_peer(self.lib.kvq_peer_alloc(self.nbytes, ctypes.byref(ptr), handle))
        self.ptr = ptr.value

    def status(self):
        import torch
        from kernelverify_b200 import _native
        st = ctypes.c_uint32()
        _native.check_peer(self.lib.kvq_peer_status(self.ptr, ctypes.byref(st),
                                                    torch.cuda.current_stream().cuda_stream))
        return st.value

    def free(self):
        import torch
        from kernelverify_b200 import _native
        torch.cuda.synchronize()
        _native.check_peer(self.lib.kvq_peer_free(self.ptr))


def _fused(dev, bits, t, region, *, seq_lens=None, regions=None, world=1, rank=0, timeout_us=0,
           out=None):
    """One kvq_tsplit_decode call; (out, split count, what must outlive it)."""
    import torch
    from kernelverify_b200 import _native
    from kernelverify_b200.pack import kv_attention as kva
    lib = _native.lib()
    q = dev[0]
    sl = None if seq_lens is None else torch.from_numpy(np.asarray(seq_lens, np.int32)).cuda()
    a = kva._args(*dev, bits=bits, t_cached=t, t_begin=0, t_end=t, has_new_entry=rank == world - 1,
                  seq_lens=sl)
    out = torch.empty_like(q) if out is None else out
    ptrs = regions if regions is not None else [region.ptr]
    arr = (ctypes.c_void_p * len(ptrs))(*ptrs)
    _native.check(lib.kvq_tsplit_decode(a, arr, region.nbytes, world, rank, out.data_ptr(),
                                        timeout_us, torch.cuda.current_stream().cuda_stream))
    return out, lib.kvq_split_count(a), sl


def _shared_case(h, hkv, t, seed):
    q, kc, vc, nk, nv = cases.make_case(1, h, t, 128, seed=seed)
    return q, kc[:hkv], vc[:hkv], nk[:, :hkv], nv[:, :hkv]


@pytest.mark.parametrize("h,hkv,t", [(8, 1, 64), (64, 8, 1000), (64, 8, 6000), (64, 8, 131072 // 8),
                                     (32, 8, 4096), (16, 4, 2048), (12, 2, 3000), (28, 4, 5000)])
def test_one_rank_against_the_oracle_and_the_two_launch_step(native, h, hkv, t):
    """r = 8 (head tile 8), r = 4 (tile 4), r = 6 and 7 (one partial tile):
    the fused step's verdict, and its output against kvq_decode's."""
    import torch
    from tests.test_gpu_paths import close
    from kernelverify_b200.pack import kv_attention as kva
    q, kc, vc, nk, nv = _shared_case(h, hkv, t, seed=h + hkv + t)
    dev = [to_dev(x) for x in (q, *pack(kc, 4), *pack(vc, 4), nk, nv)]
    region = _Region(h)
    try:
        out, splits, keep = _fused(dev, 4, t, region)
        torch.cuda.synchronize()
        assert region.status() == 0
        got = out.cpu().numpy()
        v = judge_gqa(q, kc, vc, nk, nv, 4, got)
        assert v.ok, (splits, v)
        ref = kva.decode(*dev, bits=4, t_cached=t).cpu().numpy()
        assert close(got, ref), splits
        print(f"h={h} hkv={hkv} t={t}: {splits} splits, err/tol {v.err / v.tol:.3f}")
    finally:
        region.free()


def test_batch_ragged_lengths(native):
    """Per-sequence caches with ragged lengths, 0 included (out = new_v)."""
    import torch
    rng = np.random.default_rng(9)
    b, h, hkv, t_pad = 5, 32, 8, 3072
    lens = np.array([0, 1, 3072, 777, 2049], dtype=np.int32)
    q = rng.standard_normal((b, h, 128)).astype(np.float16)
    kc = rng.standard_normal((b, hkv, t_pad, 128)).astype(np.float16)
    vc = rng.standard_normal((b, hkv, t_pad, 128)).astype(np.float16)
    nk = rng.standard_normal((b, hkv, 128)).astype(np.float16)
    nv = rng.standard_normal((b, hkv, 128)).astype(np.float16)
    dev = [to_dev(x) for x in (q, *pack(kc, 4), *pack(vc, 4), nk, nv)]
    region = _Region(b * h)
    try:
        out, _, keep = _fused(dev, 4, t_pad, region, seq_lens=lens)
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.array_equal(got[0], np.repeat(nv[0], h // hkv, axis=0))
        for v in judge_per_sequence(q, kc, vc, nk, nv, 4, got, lens, rows=range(1, b)):
            assert v.ok, v
    finally:
        region.free()


def test_repeated_steps_and_graph_replay(native):
    """Eight eager steps on changing q (the step count and the record parity
    advance), then one CUDA graph replayed over ten more: every step equal to
    a fresh eager step on its inputs, bit for bit, and the oracle's verdict on
    the last one."""
    import torch
    from kernelverify_b200.pack.tsplit import SequenceSplitDecoder
    h, hkv, t = 64, 8, 6000
    q, kc, vc, nk, nv = _shared_case(h, hkv, t, seed=41)
    dev = [to_dev(x) for x in (q, *pack(kc, 4), *pack(vc, 4), nk, nv)]
    dec = SequenceSplitDecoder(1, h, 128, torch.device("cuda"), transport="fused")
    ref_dec = SequenceSplitDecoder(1, h, 128, torch.device("cuda"), transport="fused")
    rng = np.random.default_rng(3)
    try:
        out = torch.empty_like(dev[0])
        for _ in range(8):
            dev[0].copy_(to_dev(rng.standard_normal(q.shape).astype(np.float16)))
            dec.step(*dev, bits=4, t_local=t, out=out)
            ref = ref_dec.step(*dev, bits=4, t_local=t)
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
        graph = dec.capture(*dev, bits=4, t_local=t, out=out)
        for _ in range(10):
            qn = rng.standard_normal(q.shape).astype(np.float16)
            dev[0].copy_(to_dev(qn))
            graph.replay(out=out)
            ref = ref_dec.step(*dev, bits=4, t_local=t)
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
        v = judge_gqa(qn, kc, vc, nk, nv, 4, out.cpu().numpy())
        assert v.ok, v
        assert dec.exchange.status() == 0 and ref_dec.exchange.status() == 0
        del graph
    finally:
        dec.close()
        ref_dec.close()


def test_wait_for_a_silent_peer_runs_out_and_reports(native):
    """world 2 with both regions on this GPU and one launch (rank 0): rank 1
    never stores its records, so every merging CTA's wait for words tagged
    with this step expires (bounded, 20 ms): status 1, NaN rows, and the
    context still runs kernels. Nothing waits on another kernel."""
    import torch
    h, hkv, t = 64, 8, 2000
    q, kc, vc, nk, nv = _shared_case(h, hkv, t, seed=5)
    dev = [to_dev(x) for x in (q, *pack(kc, 4), *pack(vc, 4), nk, nv)]
    r0, r1 = _Region(h, world=2), _Region(h, world=2)
    try:
        out, _, keep = _fused(dev, 4, t, r0, regions=[r0.ptr, r1.ptr], world=2, rank=0,
                              timeout_us=20_000)
        torch.cuda.synchronize()
        assert r0.status() == 1
        assert torch.isnan(out.float()).all()
        assert float((torch.ones(1000, device="cuda") * 2).sum()) == 2000.0
    finally:
        r0.free()
        r1.free()


def test_formats_it_does_not_serve_are_refused(native):
    import torch
    from kernelverify_b200 import _native
    from kernelverify_b200.pack import kv_attention as kva
    h, hkv, t = 16, 2, 512
    q, kc, vc, nk, nv = _shared_case(h, hkv, t, seed=8)
    dev = [to_dev(x) for x in (q, *pack(kc, 8), *pack(vc, 8), nk, nv)]
    a = kva._args(*dev, bits=8, t_cached=t, t_begin=0, t_end=t, has_new_entry=True)
    lib = _native.lib()
    assert lib.kvq_tsplit_supported(a) == 0
    region = _Region(h)
    try:
        with pytest.raises(_native.KvqError) as err:
            _fused(dev, 8, t, region)
        assert err.value.status == _native.KVQ_ERR_UNSUPPORTED
        torch.cuda.synchronize()
    finally:
        region.free()
