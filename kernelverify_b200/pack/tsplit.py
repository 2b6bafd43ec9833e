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
    [B, HKV, T_local, ...]); positions are local to them.
    """

    b_rows: int
    n_heads: int
    head_dim: int
    device: object
    group: object = None

    def __post_init__(self):
        import torch
        self.world = 1 if self.group is None else torch.distributed.get_world_size(self.group)
        self.rank = 0 if self.group is None else torch.distributed.get_rank(self.group)
        rows = self.b_rows * self.n_heads
        f32 = dict(dtype=torch.float32, device=self.device)
        self.part_o = torch.empty((rows, self.head_dim), **f32)
        self.part_m = torch.empty((rows,), **f32)
        self.part_l = torch.empty((rows,), **f32)
        self.all_o = torch.empty((self.world, rows, self.head_dim), **f32)
        self.all_m = torch.empty((self.world, rows), **f32)
        self.all_l = torch.empty((self.world, rows), **f32)
        from kernelverify_b200.pack.kv_attention import Workspace
        self.workspace = Workspace()

    def step(self, q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *,
             bits: int, t_local: int, out=None, partial_events=None):
        """out [B, H, DH] in q's dtype, identical on every rank.
        `partial_events`, a (start, stop) pair of CUDA events, brackets the
        local partial on the current stream (for timing it alone)."""
        import torch
        from kernelverify_b200.pack import kv_attention as kva

        if partial_events is not None:
            partial_events[0].record()
        kva.decode_partial(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v,
                           bits=bits, t_begin=0, t_end=t_local, t_cached=t_local,
                           has_new_entry=owns_new_entry(self.world, self.rank),
                           part_o=self.part_o.view(self.b_rows, self.n_heads, self.head_dim),
                           part_m=self.part_m.view(self.b_rows, self.n_heads),
                           part_l=self.part_l.view(self.b_rows, self.n_heads),
                           workspace=self.workspace)
        if partial_events is not None:
            partial_events[1].record()
        if self.group is None:
            self.all_o[0].copy_(self.part_o)
            self.all_m[0].copy_(self.part_m)
            self.all_l[0].copy_(self.part_l)
        else:
            dist = torch.distributed
            dist.all_gather_into_tensor(self.all_o, self.part_o, group=self.group)
            dist.all_gather_into_tensor(self.all_m, self.part_m, group=self.group)
            dist.all_gather_into_tensor(self.all_l, self.part_l, group=self.group)
        return kva.lse_merge(self.all_o.view(self.world, self.b_rows, self.n_heads, self.head_dim),
                             self.all_m.view(self.world, self.b_rows, self.n_heads),
                             self.all_l.view(self.world, self.b_rows, self.n_heads),
                             q.dtype, out=out)
