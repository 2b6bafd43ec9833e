"""The sequence split on CPU ranks (gloo): shard bounds, the partial /
all-gather / log-sum-exp decomposition against the single-pass fp64 oracle,
and a rank that leaves before the collective (the survivor's collective fails
within its short timeout instead of hanging)."""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from kernelverify_b200.pack.tsplit import owns_new_entry, shard_bounds


@pytest.mark.parametrize("t", [1, 7, 8, 100, 131072, 131071])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_cover_the_sequence_once(t, world):
    bounds = [shard_bounds(t, world, r) for r in range(world)]
    assert bounds[0][0] == 0 and bounds[-1][1] == t
    for (a0, a1), (b0, b1) in zip(bounds, bounds[1:]):
        assert a1 == b0
    for r, (a, b) in enumerate(bounds):
        assert a <= b
        assert a % 8 == 0 or a == t
    assert [owns_new_entry(world, r) for r in range(world)].count(True) == 1


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _partial64(q, kd, vd, lo, hi, nk, nv, with_new):
    """fp64 partial (O unnormalised, m, l) over positions [lo, hi) (+ new entry)."""
    scale = 1.0 / np.sqrt(q.shape[-1])
    s = np.einsum("bhd,htd->bht", q, kd[:, lo:hi]) * scale
    v = np.broadcast_to(vd[None, :, lo:hi], (q.shape[0],) + vd[:, lo:hi].shape)
    if with_new:
        s = np.concatenate([s, (np.sum(q * nk, axis=-1) * scale)[..., None]], axis=-1)
        v = np.concatenate([v, nv[:, :, None, :]], axis=2)
    if s.shape[-1] == 0:
        return np.zeros(q.shape), np.full(q.shape[:2], -np.inf), np.zeros(q.shape[:2])
    m = s.max(axis=-1)
    p = np.exp(s - m[..., None])
    return np.einsum("bht,bhtd->bhd", p, v), m, p.sum(axis=-1)


def _rank_main(rank, world, port, path, leave_early):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    from oracle import cases, kv
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    t = 3001
    q, kc, vc, nk, nv = cases.make_case(2, 4, t, 64, seed=5)
    inputs = kv.kv_inputs(q, kc, vc, nk, nv, 4)
    kd = kv.dequant64(kc, 4)
    vd = kv.dequant64(vc, 4)
    lo, hi = shard_bounds(t, world, rank)
    o, m, l = _partial64(q.astype(np.float64), kd, vd, lo, hi, nk.astype(np.float64),
                         nv.astype(np.float64), owns_new_entry(world, rank))
    if leave_early and rank == 1:
        os._exit(0)   # leaves between steps: nothing of its is in flight
    status = "ok"
    try:
        packed = torch.from_numpy(np.concatenate([o.ravel(), m.ravel(), l.ravel()]))
        gathered = [torch.empty_like(packed) for _ in range(world)]
        dist.all_gather(gathered, packed)
        n_o, n_m = o.size, m.size
        parts = [g.numpy() for g in gathered]
        O = np.stack([p[:n_o].reshape(o.shape) for p in parts])
        M = np.stack([p[n_o:n_o + n_m].reshape(m.shape) for p in parts])
        L = np.stack([p[n_o + n_m:].reshape(l.shape) for p in parts])
        mm = M.max(axis=0)
        w = np.exp(M - mm)
        out = (O * w[..., None]).sum(axis=0) / (L * w).sum(axis=0)[..., None]
        ref = kv.kv_reference(inputs)
        err = float(np.max(np.abs(out - ref)))
        status = f"ok {err:.3e}" if err < 1e-12 * max(1.0, float(np.max(np.abs(ref)))) else f"bad {err}"
    except Exception as error:  # the collective failed
        status = f"error {type(error).__name__}"
    with open(f"{path}.{rank}", "w") as fh:
        fh.write(status)
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def _spawn(world, tmp_path, leave_early=False):
    import torch.multiprocessing as mp
    port = _free_port()
    path = str(tmp_path / "status")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, path, leave_early))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    return [open(f"{path}.{r}").read() if os.path.exists(f"{path}.{r}") else "missing"
            for r in range(world)]


@pytest.mark.parametrize("world", [2, 3])
def test_partials_gathered_and_merged_equal_the_single_pass(tmp_path, world):
    status = _spawn(world, tmp_path)
    assert all(s.startswith("ok") for s in status), status


def test_a_rank_that_leaves_makes_the_collective_fail_not_hang(tmp_path):
    status = _spawn(2, tmp_path, leave_early=True)
    assert status[1] == "missing"
    assert status[0].startswith("error"), status


def test_decoder_rejects_unknown_transports_and_unserved_geometry():
    """Host checks of the sequence-split decoder, before any device work: an
    unknown transport, and a fused region for a head_dim the one-kernel step
    does not serve (kvq_tsplit_region_bytes is 0 there)."""
    import pytest
    from kernelverify_b200.pack.tsplit import SequenceSplitDecoder
    with pytest.raises(ValueError, match="transport"):
        SequenceSplitDecoder(1, 8, 128, "cpu", transport="bogus")
    with pytest.raises(ValueError, match="no fused region"):
        SequenceSplitDecoder(1, 8, 64, "cpu", transport="fused")
