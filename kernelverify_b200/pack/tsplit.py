"""Sequence-split decode: one long sequence's cached positions sharded by
T range across the ranks of a process group, merged by log-sum-exp.

The reference has no multi-GPU path (its kernel holds T <= 1024 in one
threadgroup, kernelverify/pack/kv_attention.py:53-65); this is the
long-context extension. Each rank holds the cache rows of its own range, runs
`kvq_decode_partial` over them (the step's own new entry enters on the last
rank only), the per-rank partials (O unnormalised, m, l) are all-gathered,
and every rank merges them with `kvq_lse_merge`:

    m = max_r m_r,  l = sum_r l_r e^(m_r - m),  out = sum_r O_r e^(m_r - m) / l.

Batch x KV-head work is never split across ranks; only T is.
"""

from __future__ import annotations

from dataclasses import dataclass

# Shard starts are multiples of this many positions, so every rank's rows
# stay on the tensor-core kernel's 8-row TMA alignment.
SHARD_ALIGN = 8


def shard_bounds(t_total: int, world: int, rank: int, align: int = SHARD_ALIGN) -> tuple[int, int]:
    """[begin, end) of `rank`'s contiguous share of t_total positions: equal
    shares rounded to `align`, the last rank taking the remainder."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    share = -(-t_total // world)
    share = -(-share // align) * align
    begin = min(rank * share, t_total)
    end = t_total if rank == world - 1 else min(begin + share, t_total)
    return begin, end


def owns_new_entry(world: int, rank: int) -> bool:
    """The step's own K/V enter exactly once: on the last rank."""
    return rank == world - 1


@dataclass
class SequenceSplitDecoder:
    """One decode step over a T-sharded cache, reusing its buffers.

    `group` is a torch.distributed process group (None: a single rank). The
    local cache tensors hold only this rank's rows ([HKV, T_local, ...] or
    [B, HKV, T_local, ...]); positions are local to them. Each rank's partial
    lands in one fp32 record (O, then m, then l), so a step makes one
    all-gather; `capture` records a whole step as a CUDA graph.
    """

    b_rows: int
    n_heads: int
    head_dim: int
    device: object
    group: object = None

    def __post_init__(self):
        import torch
        from kernelverify_b200.pack.kv_attention import Workspace, record_floats, record_views
        self.world = 1 if self.group is None else torch.distributed.get_world_size(self.group)
        self.rank = 0 if self.group is None else torch.distributed.get_rank(self.group)
        n = record_floats(self.b_rows * self.n_heads, self.head_dim)
        self.records = torch.empty((self.world, n), dtype=torch.float32, device=self.device)
        self.record = torch.empty((n,), dtype=torch.float32, device=self.device)
        self.part_o, self.part_m, self.part_l = record_views(self.record, self.b_rows,
                                                             self.n_heads, self.head_dim)
        self.workspace = Workspace()

    def partial(self, q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *,
                bits: int, t_local: int):
        """This rank's partial into its record (the local step alone)."""
        from kernelverify_b200.pack import kv_attention as kva
        kva.decode_partial(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v,
                           bits=bits, t_begin=0, t_end=t_local, t_cached=t_local,
                           has_new_entry=owns_new_entry(self.world, self.rank),
                           part_o=self.part_o, part_m=self.part_m, part_l=self.part_l,
                           workspace=self.workspace)

    def finish(self, out_dtype, out=None):
        """Gather every rank's record and merge them: out [B, H, DH]."""
        import torch
        from kernelverify_b200.pack import kv_attention as kva
        if self.group is None:
            self.records[0].copy_(self.record)
        else:
            torch.distributed.all_gather_into_tensor(self.records, self.record, group=self.group)
        return kva.lse_merge_records(self.records, self.b_rows, self.n_heads, self.head_dim,
                                     out_dtype, out=out)

    def step(self, q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *,
             bits: int, t_local: int, out=None):
        """out [B, H, DH] in q's dtype, identical on every rank."""
        self.partial(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v,
                     bits=bits, t_local=t_local)
        return self.finish(q.dtype, out=out)

    def capture(self, q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *,
                bits: int, t_local: int, out=None, pool=None):
        """A CUDA graph of this rank's local work on these tensors; replay it
        and then call `finish` for the step. With one rank (group None) the
        graph holds the whole step, writing `out`. With more, it holds the
        partial only: the all-gather stays an eager NCCL call, watched by the
        process group's timeout (a collective inside a graph is not). Run one
        eager `step` first (it sets the kernels' attributes and sizes the
        workspace)."""
        import torch
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, pool=pool):
            if self.group is None:
                self.step(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v,
                          bits=bits, t_local=t_local, out=out)
            else:
                self.partial(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k,
                             new_v, bits=bits, t_local=t_local)
        return graph
