"""The sequence split on two GPUs, one process per GPU (skipped with fewer):
all three transports -- NCCL all-gather of the partial records, the peer
merge over CUDA-IPC-mapped exchange regions, and the one-kernel step that
stores each head row's record into every rank's region -- give the
single-GPU oracle's verdict, eagerly and replayed from CUDA graphs."""

from __future__ import annotations

import os
import socket

import pytest

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, path):
    import datetime

    import torch
    import torch.distributed as dist

    from kernelverify_b200.pack.tsplit import SequenceSplitDecoder, shard_bounds
    from oracle import cases, kv
    from tests.kvq_cases import pack, to_dev

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    status = []
    try:
        t = 6000
        q, kc, vc, nk, nv = cases.make_case(1, 64, t, 128, seed=31)
        kc, vc, nk, nv = kc[:8], vc[:8], nk[:, :8], nv[:, :8]
        inputs = kv.gqa_tiled_inputs(q, kc, vc, nk, nv, 4)
        lo, hi = shard_bounds(t, world, rank)
        dev = [to_dev(x, f"cuda:{rank}") for x in
               (q, *pack(kc[:, lo:hi], 4), *pack(vc[:, lo:hi], 4), nk, nv)]
        for transport in ("nccl", "peer", "fused"):
            dec = SequenceSplitDecoder(1, 64, 128, torch.device("cuda", rank),
                                       group=dist.group.WORLD, transport=transport)
            out = torch.empty_like(dev[0])
            for _ in range(2):
                dec.step(*dev, bits=4, t_local=hi - lo, out=out)
                torch.cuda.synchronize()
                v = kv.verify_output(inputs, out.cpu().numpy())
                status.append(f"{transport}-eager {'ok' if v.ok else v}")
            step = dec.capture(*dev, bits=4, t_local=hi - lo, out=out)
            for _ in range(3):
                out.zero_()
                step.replay(out=out)
                torch.cuda.synchronize()
                v = kv.verify_output(inputs, out.cpu().numpy())
                status.append(f"{transport}-graph {'ok' if v.ok else v}")
            if transport in ("peer", "fused"):
                status.append(f"{transport}-status {dec.exchange.status()}")
            del step
            dec.close()
            dist.barrier()
    except Exception as error:   # reported through the status file
        status.append(f"error {type(error).__name__}: {error}")
    with open(f"{path}.{rank}", "w") as fh:
        fh.write("\n".join(status))
    dist.destroy_process_group()


def test_two_gpu_sequence_split_both_transports(tmp_path):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    world, port, path = 2, _free_port(), str(tmp_path / "status")
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, path)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        if p.is_alive():
            p.kill()
    for r in range(world):
        lines = open(f"{path}.{r}").read().splitlines() if os.path.exists(f"{path}.{r}") else ["missing"]
        assert lines and all(x.endswith(" ok") or x in ("peer-status 0", "fused-status 0")
                             for x in lines), (r, lines)
