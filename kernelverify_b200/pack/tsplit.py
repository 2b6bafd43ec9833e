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

Three transports move the partials. "nccl": one all_gather_into_tensor of
the ranks' fp32 records (O, m, l) and kvq_lse_merge_records. "peer": every
rank's record stays in an exchange region in its own GPU memory, mapped into
the peers over CUDA IPC, and kvq_peer_merge publishes, waits (bounded) and
merges in one kernel reading the peers' records over NVLink -- no collective,
so a whole step can be captured in a CUDA graph. "fused": the whole step is
ONE kernel per rank (kvq_tsplit_decode): the split stage's last CTAs of each
cache head merge its splits, store each head row's record into every rank's
region, and once every rank's record of the row is there (each word carries
the step number; the wait is bounded) merge the records into the output --
for the tensor-core kernel's 4-bit group-64 format.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass, field

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


class PeerExchange:
    """The ranks' exchange regions: this rank's own (allocated, zeroed) and
    every peer's, mapped over CUDA IPC. Create it on every rank of `group`
    together; close() it on every rank together."""

    def __init__(self, rows: int, head_dim: int, device, group=None, timeout_us: int = 2_000_000,
                 layout: str = "peer"):
        import torch
        from kernelverify_b200 import _native
        lib = _native.lib()
        self.rows, self.head_dim, self.timeout_us = rows, head_dim, timeout_us
        self.group = group
        self.world = 1 if group is None else torch.distributed.get_world_size(group)
        self.rank = 0 if group is None else torch.distributed.get_rank(group)
        if self.world > _native.KVQ_PEER_MAX_RANKS:
            raise ValueError(f"the peer transport serves at most {_native.KVQ_PEER_MAX_RANKS} ranks")
        self.device = torch.device(device)
        # "peer": kvq_peer_merge's layout; "fused": kvq_tsplit_decode's
        self.layout = layout
        self.nbytes = (lib.kvq_peer_region_bytes(rows, head_dim) if layout == "peer"
                       else lib.kvq_tsplit_region_bytes(rows, head_dim, self.world))
        if not self.nbytes:
            raise ValueError(f"no {layout} region for {rows} rows of head_dim {head_dim}")
        handle = (ctypes.c_char * _native.KVQ_PEER_HANDLE_BYTES)()
        own = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _native.check_peer(lib.kvq_peer_alloc(self.nbytes, ctypes.byref(own), handle))
        self.own = own.value
        handles = [bytes(handle)]
        if self.world > 1:
            handles = [None] * self.world
            torch.distributed.all_gather_object(handles, bytes(handle), group=group)
        self.regions = []
        with torch.cuda.device(self.device):
            for p, h in enumerate(handles):
                if p == self.rank:
                    self.regions.append(self.own)
                    continue
                ptr = ctypes.c_void_p()
                buf = (ctypes.c_char * _native.KVQ_PEER_HANDLE_BYTES).from_buffer_copy(h)
                _native.check_peer(lib.kvq_peer_open(buf, ctypes.byref(ptr)))
                self.regions.append(ptr.value)
        self._array = (ctypes.c_void_p * self.world)(*self.regions)
        if self.world > 1:
            torch.distributed.barrier(group=group)   # every mapping exists before first use

    def record(self, parity: int) -> tuple[int, int, int]:
        """Device addresses (O, m, l) of this rank's record of `parity`."""
        from kernelverify_b200 import _native
        base = self.own + _native.lib().kvq_peer_record_offset(self.rows, self.head_dim, parity)
        o_bytes = self.rows * self.head_dim * 4
        return base, base + o_bytes, base + o_bytes + self.rows * 4

    def merge(self, parity: int, out, stream=None) -> None:
        """All ranks' records of `parity` merged into out [rows, head_dim]."""
        import torch
        from kernelverify_b200 import _native
        from kernelverify_b200.pack.kv_attention import _check_buffers, _dtype_code
        _dtype_code(out.dtype)
        _check_buffers(self.device, ("out", out, (self.rows, self.head_dim), out.dtype))
        s = stream if stream is not None else torch.cuda.current_stream(out.device)
        _native.check_peer(_native.lib().kvq_peer_merge(
            self._array, self.world, self.rank, parity, self.rows, self.head_dim,
            _dtype_code(out.dtype), out.data_ptr(), self.timeout_us, s.cuda_stream))

    def status(self) -> int:
        """0; 1 when a peer's flag (or record) did not arrive in time; 2
        (peer layout) a merge named the wrong parity; 3 (fused layout) a
        unit's partials did not all arrive in time."""
        import torch
        from kernelverify_b200 import _native
        v = ctypes.c_uint32()
        with torch.cuda.device(self.device):
            _native.check_peer(_native.lib().kvq_peer_status(
                self.own, ctypes.byref(v), torch.cuda.current_stream(self.device).cuda_stream))
        return v.value

    def close(self) -> None:
        import torch
        from kernelverify_b200 import _native
        if not self.regions:
            return
        lib = _native.lib()
        torch.cuda.synchronize(self.device)
        with torch.cuda.device(self.device):
            for p, ptr in enumerate(self.regions):
                if p != self.rank:
                    _native.check_peer(lib.kvq_peer_close(ptr))
            if self.world > 1:
                torch.distributed.barrier(group=self.group)   # no peer maps us any more
            _native.check_peer(lib.kvq_peer_free(self.own))
        self.regions = []


@dataclass
class CapturedStep:
    """A step captured as CUDA graphs; replay() runs the next one."""

    decoder: "SequenceSplitDecoder"
    graphs: tuple
    finish: bool = False        # the all-gather and merge follow the replay eagerly

    def replay(self, out=None):
        dec = self.decoder
        g = self.graphs[dec._parity()] if len(self.graphs) == 2 else self.graphs[0]
        g.replay()
        if self.finish:
            dec.finish(dec._dtype, out=out)
        dec.steps += 1


@dataclass
class SequenceSplitDecoder:
    """One decode step over a T-sharded cache, reusing its buffers.

    `group` is a torch.distributed process group (None: a single rank). The
    local cache tensors hold only this rank's rows ([HKV, T_local, ...] or
    [B, HKV, T_local, ...]); positions are local to them. `transport` is
    "nccl" (one all-gather of fp32 records, then kvq_lse_merge_records),
    "peer" (kvq_peer_merge over the ranks' exchange regions) or "fused" (the
    whole step as one kvq_tsplit_decode launch per rank, one rank included).
    """

    b_rows: int
    n_heads: int
    head_dim: int
    device: object
    group: object = None
    transport: str = "nccl"
    steps: int = field(default=0, init=False)

    def __post_init__(self):
        import torch
        from kernelverify_b200.pack.kv_attention import Workspace, record_floats, record_views
        if self.transport not in ("nccl", "peer", "fused"):
            raise ValueError(f"transport {self.transport!r} is not 'nccl', 'peer' or 'fused'")
        self.world = 1 if self.group is None else torch.distributed.get_world_size(self.group)
        self.rank = 0 if self.group is None else torch.distributed.get_rank(self.group)
        rows = self.b_rows * self.n_heads
        self.workspace = Workspace()
        self._dtype = None
        if self.transport in ("peer", "fused"):
            self.exchange = PeerExchange(rows, self.head_dim, self.device, self.group,
                                         layout=self.transport)
            return
        n = record_floats(rows, self.head_dim)
        self.records = torch.empty((self.world, n), dtype=torch.float32, device=self.device)
        self.record = torch.empty((n,), dtype=torch.float32, device=self.device)
        self.part_o, self.part_m, self.part_l = record_views(self.record, self.b_rows,
                                                             self.n_heads, self.head_dim)

    def _parity(self) -> int:
        return (self.steps + 1) & 1

    def partial(self, q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *,
                bits: int, t_local: int, parity: int | None = None):
        """This rank's partial into its record (the local step alone)."""
        import torch
        from kernelverify_b200 import _native
        from kernelverify_b200.pack import kv_attention as kva
        has_new = owns_new_entry(self.world, self.rank)
        if self.transport == "nccl":
            kva.decode_partial(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v,
                               bits=bits, t_begin=0, t_end=t_local, t_cached=t_local,
                               has_new_entry=has_new, part_o=self.part_o, part_m=self.part_m,
                               part_l=self.part_l, workspace=self.workspace)
            return
        a = kva._args(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v,
                      bits=bits, t_cached=t_local, t_begin=0, t_end=t_local, has_new_entry=has_new)
        lib = _native.lib()
        o, m, l = self.exchange.record(self._parity() if parity is None else parity)
        need = lib.kvq_workspace_bytes(a)
        buf, have = self.workspace.get(need, q.device)
        _native.check(lib.kvq_decode_partial(a, o, m, l, buf.data_ptr() if buf is not None else None,
                                             have, torch.cuda.current_stream(q.device).cuda_stream))

    def finish(self, out_dtype, out=None, parity: int | None = None):
        """Gather every rank's record and merge them: out [B, H, DH]."""
        import torch
        from kernelverify_b200.pack import kv_attention as kva
        if out is None:
            out = torch.empty((self.b_rows, self.n_heads, self.head_dim), dtype=out_dtype,
                              device=self.device)
        if self.transport == "peer":
            self.exchange.merge(self._parity() if parity is None else parity,
                                out.view(self.b_rows * self.n_heads, self.head_dim))
            return out
        if self.group is None:
            self.records[0].copy_(self.record)
        else:
            torch.distributed.all_gather_into_tensor(self.records, self.record, group=self.group)
        return kva.lse_merge_records(self.records, self.b_rows, self.n_heads, self.head_dim,
                                     out_dtype, out=out)

    def fused(self, q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *,
              bits: int, t_local: int, out=None):
        """The step as one kvq_tsplit_decode launch on this rank."""
        import torch
        from kernelverify_b200 import _native
        from kernelverify_b200.pack import kv_attention as kva
        if out is None:
            out = torch.empty((self.b_rows, self.n_heads, self.head_dim), dtype=q.dtype,
                              device=self.device)
        kva._check_buffers(self.device, ("out", out, (self.b_rows, self.n_heads, self.head_dim),
                                         q.dtype))
        a = kva._args(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v,
                      bits=bits, t_cached=t_local, t_begin=0, t_end=t_local,
                      has_new_entry=owns_new_entry(self.world, self.rank))
        ex = self.exchange
        _native.check(_native.lib().kvq_tsplit_decode(
            a, ex._array, ex.nbytes, self.world, self.rank, out.data_ptr(), ex.timeout_us,
            torch.cuda.current_stream(q.device).cuda_stream))
        return out

    def launch(self, q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *,
               bits: int, t_local: int, out):
        """The step on these exact tensors as launch(stream) (for `HostStep`):
        with the fused transport the argument block is built once and each
        call is one kvq_tsplit_decode; otherwise each call is `step`. Every
        rank must call it every step."""
        import torch
        from kernelverify_b200 import _native
        from kernelverify_b200.pack import kv_attention as kva
        args = (q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v)
        if self.transport != "fused":
            def eager(stream=None):
                with torch.cuda.stream(stream if stream is not None
                                       else torch.cuda.current_stream(self.device)):
                    return self.step(*args, bits=bits, t_local=t_local, out=out)
            return eager
        kva._check_buffers(self.device, ("out", out, (self.b_rows, self.n_heads, self.head_dim),
                                         q.dtype))
        a = kva._args(*args, bits=bits, t_cached=t_local, t_begin=0, t_end=t_local,
                      has_new_entry=owns_new_entry(self.world, self.rank))
        lib, ex, out_ptr = _native.lib(), self.exchange, out.data_ptr()

        def fused(stream=None):
            s = stream if stream is not None else torch.cuda.current_stream(self.device)
            _native.check(lib.kvq_tsplit_decode(a, ex._array, ex.nbytes, self.world, self.rank,
                                                out_ptr, ex.timeout_us, s.cuda_stream))
            self.steps += 1
            return out
        fused.keep = args
        return fused

    def step(self, q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *,
             bits: int, t_local: int, out=None):
        """out [B, H, DH] in q's dtype, identical on every rank. On a single
        rank the split is the whole sequence: one kvq_decode (or, with the
        fused transport, one kvq_tsplit_decode)."""
        if self.transport == "fused":
            res = self.fused(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v,
                             bits=bits, t_local=t_local, out=out)
            self.steps += 1
            return res
        if self.world == 1:
            from kernelverify_b200.pack import kv_attention as kva
            res = kva.decode(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v,
                             bits=bits, t_cached=t_local, out=out, workspace=self.workspace)
            self.steps += 1
            return res
        self.partial(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v,
                     bits=bits, t_local=t_local)
        res = self.finish(q.dtype, out=out)
        self.steps += 1
        return res

    def capture(self, q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *,
                bits: int, t_local: int, out, pool=None) -> CapturedStep:
        """This step on these tensors as CUDA graphs; `.replay()` reruns it on
        whatever they then hold. With the fused transport one graph holds the
        whole step (its step count lives in the exchange regions). With the
        peer transport, or with one rank, the graphs hold the whole step (one
        graph per record parity for the peer transport). With NCCL on more ranks they hold the partial only and
        the all-gather and merge run eagerly after each replay: a collective
        inside a graph is outside the process group's timeout. Run one eager
        `step` first (it sets the kernels' attributes and sizes the workspace)."""
        import torch
        self._dtype = q.dtype
        args = (q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v)
        if self.world == 1 or self.transport == "fused":
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, pool=pool):
                self.step(*args, bits=bits, t_local=t_local, out=out)
            self.steps -= 1          # capture does not count as a step
            return CapturedStep(self, (g,))
        if self.transport == "peer":
            graphs = []
            for parity in (0, 1):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, pool=pool):
                    self.partial(*args, bits=bits, t_local=t_local, parity=parity)
                    self.finish(q.dtype, out=out, parity=parity)
                graphs.append(g)
            return CapturedStep(self, tuple(graphs))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, pool=pool):
            if self.group is None:
                self.partial(*args, bits=bits, t_local=t_local)
                self.finish(q.dtype, out=out)
            else:
                self.partial(*args, bits=bits, t_local=t_local)
        return CapturedStep(self, (g,), finish=self.group is not None)

    def close(self) -> None:
        """Release the peer or fused transport's regions (on every rank together)."""
        if self.transport in ("peer", "fused"):
            self.exchange.close()
