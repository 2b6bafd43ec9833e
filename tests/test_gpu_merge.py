"""The log-sum-exp merges on a B200: stacked partials and partial records give
the same bits, the merge against an fp64 restatement of its formula, empty
(m = -inf) and poisoned (NaN) parts, the part-count bound, and the
sequence-split decoder on one rank -- eager, and replayed from a CUDA graph."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import cases, kv

pytestmark = pytest.mark.gpu


def _partials(n_parts, rows, dh, seed, empty=()):
    rng = np.random.default_rng(seed)
    o = rng.standard_normal((n_parts, rows, dh)).astype(np.float32)
    m = (rng.standard_normal((n_parts, rows)) * 4).astype(np.float32)
    l = rng.uniform(0.5, 40.0, (n_parts, rows)).astype(np.float32)
    for p in empty:
        o[p] = 0.0
        m[p] = -np.inf
        l[p] = 0.0
    return o, m, l


def _merge64(o, m, l):
    mm = m.max(axis=0)
    w = np.where(np.isneginf(m), 0.0, np.exp(m.astype(np.float64) - mm))
    return (o * w[..., None]).sum(axis=0) / (l * w).sum(axis=0)[..., None]


def _records(torch, o, m, l):
    n, rows, dh = o.shape
    rec = np.concatenate([o.reshape(n, -1), m, l], axis=1)
    assert rec.shape[1] == rows * (dh + 2)
    return torch.from_numpy(np.ascontiguousarray(rec)).cuda()


@pytest.mark.parametrize("n_parts,rows,dh", [(1, 3, 64), (2, 64, 128), (8, 64, 128),
                                             (54, 64, 128), (129, 17, 128), (4096, 2, 64)])
def test_records_and_stacked_merge_agree_bitwise(native, n_parts, rows, dh):
    import torch
    from kernelverify_b200.pack import kv_attention as kva
    o, m, l = _partials(n_parts, rows, dh, seed=n_parts + rows)
    stacked = kva.lse_merge(torch.from_numpy(o).cuda().view(n_parts, 1, rows, dh),
                            torch.from_numpy(m).cuda().view(n_parts, 1, rows),
                            torch.from_numpy(l).cuda().view(n_parts, 1, rows), torch.float32)
    recs = kva.lse_merge_records(_records(torch, o, m, l), 1, rows, dh, torch.float32)
    assert torch.equal(stacked, recs)
    ref = _merge64(o, m, l)
    got = recs.cpu().numpy().reshape(rows, dh)
    assert np.max(np.abs(got - ref)) <= 1e-4 * max(1.0, np.max(np.abs(ref)))


def test_empty_parts_add_nothing_and_nan_parts_poison(native):
    import torch
    from kernelverify_b200.pack import kv_attention as kva
    o, m, l = _partials(6, 4, 128, seed=3, empty=(0, 4))
    got = kva.lse_merge_records(_records(torch, o, m, l), 1, 4, 128, torch.float32).cpu().numpy()
    keep = [1, 2, 3, 5]
    ref = _merge64(o[keep], m[keep], l[keep])
    assert np.max(np.abs(got.reshape(4, 128) - ref)) <= 1e-5 * max(1.0, np.max(np.abs(ref)))
    m[2, 1] = np.nan
    bad = kva.lse_merge_records(_records(torch, o, m, l), 1, 4, 128, torch.float32).cpu().numpy()
    bad = bad.reshape(4, 128)
    assert np.isnan(bad[1]).all()
    assert np.isfinite(bad[[0, 2, 3]]).all()


def test_merge_rejects_more_parts_than_it_holds(native):
    import torch
    from kernelverify_b200._native import KvqError
    from kernelverify_b200.pack import kv_attention as kva
    recs = torch.zeros((4097, 2 * 66), dtype=torch.float32, device="cuda")
    with pytest.raises(KvqError, match="parts"):
        kva.lse_merge_records(recs, 1, 2, 64, torch.float32)
    with pytest.raises(ValueError):
        kva.lse_merge_records(recs[:, :-1].contiguous(), 1, 2, 64, torch.float32)


def test_single_rank_sequence_split_eager_and_graph(native):
    """group=None: the decoder's step equals the fp64 oracle's verdict; its
    captured graph, replayed after new inputs are copied into the captured
    tensors, gives exactly what an eager step gives on those inputs."""
    import torch
    from kernelverify_b200.pack import kv_attention as kva
    from kernelverify_b200.pack.tsplit import SequenceSplitDecoder
    from tests.kvq_cases import pack, to_dev
    t = 9000
    q, kc, vc, nk, nv = cases.make_case(1, 64, t, 128, seed=21)
    kc, vc, nk, nv = kc[:8], vc[:8], nk[:, :8], nv[:, :8]
    dev = [to_dev(x) for x in (q, *pack(kc, 4), *pack(vc, 4), nk, nv)]
    dec = SequenceSplitDecoder(1, 64, 128, torch.device("cuda"))
    out = torch.empty_like(dev[0])
    dec.step(*dev, bits=4, t_local=t, out=out)
    torch.cuda.synchronize()
    v = kv.verify_output(kv.gqa_tiled_inputs(q, kc, vc, nk, nv, 4), out.cpu().numpy())
    assert v.ok, v
    graph = dec.capture(*dev, bits=4, t_local=t, out=out)
    q2 = np.random.default_rng(5).standard_normal(q.shape).astype(np.float16)
    dev[0].copy_(to_dev(q2))
    graph.replay()
    torch.cuda.synchronize()
    replayed = out.clone()
    eager = dec.step(*dev, bits=4, t_local=t, out=torch.empty_like(out))
    torch.cuda.synchronize()
    assert torch.equal(replayed, eager)
    v2 = kv.verify_output(kv.gqa_tiled_inputs(q2, kc, vc, nk, nv, 4), replayed.cpu().numpy())
    assert v2.ok, v2
    del graph


def test_single_rank_peer_transport_eager_and_graph(native):
    """The peer transport on one rank: its record and kvq_peer_merge give the
    oracle's verdict, and the graphs (one per record parity) replay it."""
    import torch
    from kernelverify_b200.pack.tsplit import SequenceSplitDecoder
    from tests.kvq_cases import pack, to_dev
    t = 5000
    q, kc, vc, nk, nv = cases.make_case(1, 64, t, 128, seed=23)
    kc, vc, nk, nv = kc[:8], vc[:8], nk[:, :8], nv[:, :8]
    dev = [to_dev(x) for x in (q, *pack(kc, 4), *pack(vc, 4), nk, nv)]
    dec = SequenceSplitDecoder(1, 64, 128, torch.device("cuda"), transport="peer")
    try:
        out = torch.empty_like(dev[0])
        for _ in range(3):   # both record parities, eagerly
            dec.step(*dev, bits=4, t_local=t, out=out)
            torch.cuda.synchronize()
            v = kv.verify_output(kv.gqa_tiled_inputs(q, kc, vc, nk, nv, 4), out.cpu().numpy())
            assert v.ok, v
        step = dec.capture(*dev, bits=4, t_local=t, out=out)
        for _ in range(3):
            out.zero_()
            step.replay(out=out)
            torch.cuda.synchronize()
            v = kv.verify_output(kv.gqa_tiled_inputs(q, kc, vc, nk, nv, 4), out.cpu().numpy())
            assert v.ok, v
        assert dec.exchange.status() == 0
        del step
    finally:
        dec.close()


def test_peer_merge_wait_runs_out_and_reports(native):
    """A rank whose peer never publishes: the merge's wait on a flag that
    nothing sets expires (bounded), the region's status says so, the rows are
    NaN, and the device stays usable. Both regions are on this GPU and only
    one merge kernel runs, so nothing waits on another kernel."""
    import ctypes
    import torch
    from kernelverify_b200 import _native
    lib = _native.lib()
    rows, dh = 4, 128
    nbytes = lib.kvq_peer_region_bytes(rows, dh)
    regions = []
    for _ in range(2):
        ptr = ctypes.c_void_p()
        handle = (ctypes.c_char * _native.KVQ_PEER_HANDLE_BYTES)()
        _native.check_peer(lib.kvq_peer_alloc(nbytes, ctypes.byref(ptr), handle))
        regions.append(ptr.value)
    try:
        arr = (ctypes.c_void_p * 2)(*regions)
        out = torch.zeros((rows, dh), dtype=torch.float32, device="cuda")
        _native.check_peer(lib.kvq_peer_merge(arr, 2, 0, 1, rows, dh, _native.KVQ_F32, out.data_ptr(),
                                              200_000, torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        st = ctypes.c_uint32()
        _native.check_peer(lib.kvq_peer_status(regions[0], ctypes.byref(st),
                                               torch.cuda.current_stream().cuda_stream))
        assert st.value == 1
        assert torch.isnan(out).all()
        # the context is intact: an ordinary kernel still runs
        assert float((torch.ones(1000, device="cuda") * 2).sum()) == 2000.0
    finally:
        torch.cuda.synchronize()
        for r in regions:
            _native.check_peer(lib.kvq_peer_free(r))


def test_peer_merge_with_the_wrong_parity_publishes_nothing(native):
    """A merge told the parity its step does not have (a fresh region is at
    step 1, parity 1; the call says 0): nothing is published, the status word
    is 2, the rows are NaN, and the step counter still advances, so the next
    call at the right parity (step 2, parity 0) merges normally."""
    import ctypes
    import torch
    from kernelverify_b200 import _native
    lib = _native.lib()
    rows, dh = 4, 128
    nbytes = lib.kvq_peer_region_bytes(rows, dh)
    ptr = ctypes.c_void_p()
    handle = (ctypes.c_char * _native.KVQ_PEER_HANDLE_BYTES)()
    _native.check_peer(lib.kvq_peer_alloc(nbytes, ctypes.byref(ptr), handle))
    region = ptr.value
    s = torch.cuda.current_stream().cuda_stream
    try:
        arr = (ctypes.c_void_p * 1)(region)
        out = torch.zeros((rows, dh), dtype=torch.float32, device="cuda")
        _native.check_peer(lib.kvq_peer_merge(arr, 1, 0, 0, rows, dh, _native.KVQ_F32, out.data_ptr(),
                                              200_000, s))
        torch.cuda.synchronize()
        st = ctypes.c_uint32()
        _native.check_peer(lib.kvq_peer_status(region, ctypes.byref(st), s))
        assert st.value == 2
        assert torch.isnan(out).all()
        # step 2 has parity 0: its record (O = 1, m = 0, l = 2 in every row)
        # merges to 0.5 everywhere
        base = region + lib.kvq_peer_record_offset(rows, dh, 0)

        class _Rec:    # the record's device memory as a torch view
            __cuda_array_interface__ = {"shape": (rows * (dh + 2),), "typestr": "<f4",
                                        "data": (base, False), "version": 3, "strides": None}

        rec = torch.as_tensor(_Rec(), device="cuda")
        rec[: rows * dh] = 1.0
        rec[rows * dh: rows * dh + rows] = 0.0
        rec[rows * dh + rows:] = 2.0
        torch.cuda.synchronize()
        _native.check_peer(lib.kvq_peer_merge(arr, 1, 0, 0, rows, dh, _native.KVQ_F32, out.data_ptr(),
                                              200_000, s))
        torch.cuda.synchronize()
        assert torch.equal(out, torch.full_like(out, 0.5))
    finally:
        torch.cuda.synchronize()
        _native.check_peer(lib.kvq_peer_free(region))
