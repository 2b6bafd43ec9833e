"""The serving caller: a decode loop's attention calls routed to the fused
quantized-KV kernel.

B200 form of the reference's mlx-lm runtime patch (bench/spike_mlx_e2e.py:
103-229). Two seams, as there:

* the cache's update step stashes the step's own post-rope full-precision
  K/V before the entry is quantized into the cache
  (`QuantizedKVCache.update_and_fetch`, the reference's `_stashing_update`,
  spike_mlx_e2e.py:116-119): the kernel's contract takes the new entry at full
  precision;
* the attention call becomes a router below the cache update
  (`DecodeRouter.__call__`, the reference's `_router`, spike_mlx_e2e.py:
  201-229). An eligible call (one query position, a quantized cache with a
  stashed entry, supported bits / group / head_dim, no mask arithmetic, no
  sinks, the standard 1/sqrt(DH) scale) launches the fused step on the PADDED
  cache buffers with the logical length as a scalar -- never slicing, which
  would charge the stock path's contiguity copies to the fused arm (the
  convention of tests/test_pack_kv_attention.py:143-173). Everything else
  falls through to the stock composition and is counted by reason
  (`_ineligible`, spike_mlx_e2e.py:126-152): an arm that silently stopped
  being the arm is the first thing to catch.

Differences from the reference's spike, all widenings the CUDA kernel serves:
any batch size (one cache per sequence), any logical length (no T <= 1024
capacity), bits 6 and groups 32/128, and a cache the library quantizes on the
device (`kvq_cache_append`) rather than a framework's own quantizer.

`stock_attention` is the incumbent the fused arm is measured against: the
packed cache dequantized (positions [0, offset), the step's own entry read
back quantized, as the framework's stock path does) and torch's
scaled-dot-product attention over it. `FullPrecisionKVCache` is the third
arm: an fp16 cache and the same torch attention.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

from kernelverify_b200.pack import kv_attention as kva


ROW_ALIGN = 64


def _torch():
    import torch
    return torch


class QuantizedKVCache:
    """One layer's packed K/V cache for a batch of sequences.

    keys / values: (words int32 [B, HKV, t_stride, DH*bits/32], scales
    [B, HKV, t_stride, DH/group], biases) -- the padded buffers the fused
    kernel reads whole; t_stride is `capacity` rounded up to 64 rows. `offset` is the logical length (positions written),
    uniform over the batch; `positions` is its device copy (int32 [B]) for a
    captured step. `new_keys` / `new_values` hold the last update's
    full-precision entry ([B, HKV, L, DH])."""

    def __init__(self, batch: int, n_kv_heads: int, head_dim: int, capacity: int, bits: int,
                 group_size: int = 64, dtype=None, device="cuda"):
        torch = _torch()
        dtype = torch.float16 if dtype is None else dtype
        if bits not in kva.SUPPORTED_BITS:
            raise ValueError(f"bits {bits} not in {kva.SUPPORTED_BITS}")
        if head_dim not in kva.SUPPORTED_DH:
            raise ValueError(f"head_dim {head_dim} not in {kva.SUPPORTED_DH}")
        if group_size not in kva.SUPPORTED_GROUPS or head_dim % group_size:
            raise ValueError(f"group_size {group_size} not in {kva.SUPPORTED_GROUPS}")
        if capacity < 1:
            raise ValueError("capacity must be >= 1")
        self.bits, self.group_size, self.dtype = bits, group_size, dtype
        self.batch, self.n_kv_heads, self.head_dim, self.capacity = (batch, n_kv_heads, head_dim,
                                                                      capacity)
        words = head_dim * bits // 32
        groups = head_dim // group_size
        # physical rows per head: a multiple of 64, so the tensor-core kernels
        # (8-row-aligned geometry) serve every length up to `capacity`
        self.t_stride = -(-capacity // ROW_ALIGN) * ROW_ALIGN
        lead = (batch, n_kv_heads, self.t_stride)

        def triplet():
            return (torch.zeros(lead + (words,), dtype=torch.int32, device=device),
                    torch.zeros(lead + (groups,), dtype=dtype, device=device),
                    torch.zeros(lead + (groups,), dtype=dtype, device=device))

        self.keys, self.values = triplet(), triplet()
        self.offset = 0
        self.positions = torch.zeros(batch, dtype=torch.int32, device=device)
        self.new_keys = self.new_values = None

    @property
    def device(self):
        return self.keys[0].device

    def nbytes(self) -> int:
        return sum(t.numel() * t.element_size() for t in self.keys + self.values)

    def update_and_fetch(self, keys, values):
        """Quantize keys / values [B, HKV, L, DH] into positions
        [offset, offset + L), stash them at full precision, advance `offset`;
        returns the padded (keys, values) triplets."""
        b, hkv, n, dh = keys.shape
        if (b, hkv, dh) != (self.batch, self.n_kv_heads, self.head_dim):
            raise ValueError(f"update of shape {tuple(keys.shape)} for a cache of "
                             f"[{self.batch}, {self.n_kv_heads}, *, {self.head_dim}]")
        if tuple(values.shape) != tuple(keys.shape):
            raise ValueError("keys and values differ in shape")
        if self.offset + n > self.capacity:
            raise ValueError(f"cache full: {self.offset} + {n} positions > capacity "
                             f"{self.capacity}")
        keys = keys.to(self.dtype).contiguous()
        values = values.to(self.dtype).contiguous()
        kva.cache_append(keys, *self.keys, self.bits, position=self.offset)
        kva.cache_append(values, *self.values, self.bits, position=self.offset)
        self.new_keys, self.new_values = keys, values
        self.offset += n
        self.positions.fill_(self.offset)
        return self.keys, self.values

    def append_at(self, keys, values, positions):
        """Quantize keys / values [B, HKV, 1, DH] into each sequence's row
        positions[b] (an int32 [B] device tensor) and stash them; the host
        `offset` is left alone (a captured step advances `positions` on the
        device)."""
        keys = keys.to(self.dtype).contiguous()
        values = values.to(self.dtype).contiguous()
        kva.cache_append(keys, *self.keys, self.bits, positions=positions)
        kva.cache_append(values, *self.values, self.bits, positions=positions)
        self.new_keys, self.new_values = keys, values

    def dequantized(self, length: int | None = None):
        """(K, V) in the cache dtype, [B, HKV, length, DH]: positions
        [0, length) read back through the library's dequantizer."""
        n = self.offset if length is None else length

        def deq(t):
            sl = tuple(x[:, :, :n].contiguous() for x in t)
            return kva.dequant(*sl, self.bits)

        return deq(self.keys), deq(self.values)


class FullPrecisionKVCache:
    """The third arm: an fp16 (or fp32) cache [B, HKV, capacity, DH]."""

    def __init__(self, batch: int, n_kv_heads: int, head_dim: int, capacity: int, dtype=None,
                 device="cuda"):
        torch = _torch()
        dtype = torch.float16 if dtype is None else dtype
        shape = (batch, n_kv_heads, capacity, head_dim)
        self.k = torch.zeros(shape, dtype=dtype, device=device)
        self.v = torch.zeros(shape, dtype=dtype, device=device)
        self.capacity, self.offset, self.dtype = capacity, 0, dtype

    def append_at(self, keys, values, positions):
        """Write keys / values [B, HKV, 1, DH] at each sequence's row
        positions[b] (int32 [B] device tensor); no host bookkeeping."""
        torch = _torch()
        rows = torch.arange(keys.shape[0], device=keys.device)
        idx = positions.long()
        self.k[rows, :, idx] = keys[:, :, 0]
        self.v[rows, :, idx] = values[:, :, 0]

    def update_and_fetch(self, keys, values):
        n = keys.shape[2]
        if self.offset + n > self.capacity:
            raise ValueError(f"cache full: {self.offset} + {n} positions > capacity "
                             f"{self.capacity}")
        self.k[:, :, self.offset:self.offset + n] = keys
        self.v[:, :, self.offset:self.offset + n] = values
        self.offset += n
        return self.k[:, :, :self.offset], self.v[:, :, :self.offset]


def _causal_mask(n_q: int, n_kv: int, device):
    """Bottom-right aligned causal mask: query i (the last n_q positions of
    n_kv) sees keys j <= n_kv - n_q + i. None when every key is visible."""
    if n_q == 1:
        return None
    torch = _torch()
    i = torch.arange(n_q, device=device)[:, None]
    j = torch.arange(n_kv, device=device)[None, :]
    return j <= (n_kv - n_q + i)


def stock_attention(queries, cache, scale: float, mask=None):
    """The incumbent: torch scaled-dot-product attention over the cache as the
    framework holds it -- the dequantized packed cache (the step's own entry
    included, read back quantized) or the full-precision one.
    queries [B, H, L, DH] -> [B, H, L, DH]."""
    torch = _torch()
    F = torch.nn.functional
    if isinstance(cache, QuantizedKVCache):
        k, v = cache.dequantized()
        k, v = k.to(queries.dtype), v.to(queries.dtype)
    else:
        k, v = cache.k[:, :, :cache.offset], cache.v[:, :, :cache.offset]
    n_q, n_kv = queries.shape[2], k.shape[2]
    causal = isinstance(mask, str) and mask == "causal"
    if causal and n_q == n_kv and n_q > 1:
        # a first chunk: top-left and bottom-right alignment agree, and the
        # flag keeps torch on its fused causal kernels (no [L, L] mask)
        return F.scaled_dot_product_attention(queries, k, v, is_causal=True, scale=scale,
                                              enable_gqa=k.shape[1] != queries.shape[1])
    attn_mask = _causal_mask(n_q, n_kv, queries.device) if causal else mask
    return F.scaled_dot_product_attention(queries, k, v, attn_mask=attn_mask, scale=scale,
                                          enable_gqa=k.shape[1] != queries.shape[1])


def contract_reference(queries, cache):
    """fp64 composition of the kernel's contract on the dequantized cache: the
    shadow yardstick separating "the wiring is wrong" from "the stock path's
    own arithmetic sits far from the contract" (the reference's _shadow_ref,
    spike_mlx_e2e.py:174-198). queries [B, H, 1, DH] -> [B, H, DH] fp64."""
    torch = _torch()
    b, h, _, d = queries.shape
    tc = cache.offset - 1
    r = h // cache.n_kv_heads
    kk, vv = cache.dequantized(tc)
    kk = kk.double().repeat_interleave(r, dim=1)
    vv = vv.double().repeat_interleave(r, dim=1)
    q = queries[:, :, 0].double()
    nk = cache.new_keys[:, :, -1].double().repeat_interleave(r, dim=1)
    nv = cache.new_values[:, :, -1].double().repeat_interleave(r, dim=1)
    sc = torch.cat([torch.einsum("bhd,bhtd->bht", q, kk),
                    (q * nk).sum(-1, keepdim=True)], dim=-1) * d ** -0.5
    p = torch.softmax(sc, dim=-1)
    return torch.einsum("bht,bhtd->bhd", p[..., :tc], vv) + p[..., tc:] * nv


@dataclass
class RouterStats:
    calls: int = 0
    fallback: dict = field(default_factory=dict)
    kernels: dict = field(default_factory=dict)   # fused calls by the kernel that served them
    shadow_fused_ref: float = 0.0
    shadow_stock_ref: float = 0.0
    shadow_ref_mag: float = 0.0

    def hard_fallbacks(self) -> dict:
        """Fallbacks that mean the fused arm stopped being the fused arm;
        prefill chunks route to stock by design (spike_mlx_e2e.py:107-112)."""
        return {k: v for k, v in self.fallback.items() if not k.startswith("prefill-")}


class DecodeRouter:
    """The attention call of a decode loop: `router(queries, keys, values,
    cache=..., scale=..., mask=..., sinks=...)` -> [B, H, L, DH].

    fused=False routes everything to stock (the incumbent arm). shadow=True
    runs the fused step AND stock on eligible calls, records each one's
    largest distance to the fp64 contract composition, and returns stock (the
    wiring check of spike_mlx_e2e.py:205-224)."""

    def __init__(self, fused: bool = True, shadow: bool = False):
        self.fused, self.shadow = fused, shadow
        self.stats = RouterStats()
        self.workspace = kva.Workspace()

    def reset(self) -> None:
        self.stats = RouterStats()

    @staticmethod
    def ineligible(queries, cache, scale, mask=None, sinks=None):
        """None when the fused kernel takes this call, else the reason. The
        query length is checked first so prefill chunks are labelled as
        prefill whatever the cache's state (spike_mlx_e2e.py:126-152)."""
        b, h, n, d = queries.shape
        if n != 1:
            return f"prefill-L{n}"
        if not isinstance(cache, QuantizedKVCache):
            return "cache-not-quantized"
        if cache.new_keys is None:
            return "no-stashed-new-entry"
        if cache.new_keys.shape[2] != 1:
            return f"stash-L{cache.new_keys.shape[2]}"
        if d not in kva.SUPPORTED_DH or d != cache.head_dim:
            return f"head-dim-{d}"
        if cache.bits not in kva.SUPPORTED_BITS or cache.group_size not in kva.SUPPORTED_GROUPS:
            return f"quant-{cache.bits}b-gs{cache.group_size}"
        if queries.dtype != cache.dtype:
            return f"dtype-{str(queries.dtype).replace('torch.', '')}"
        if b != cache.batch or h % cache.n_kv_heads:
            return f"heads-B{b}-H{h}-over-HKV{cache.n_kv_heads}"
        if mask is not None and not (isinstance(mask, str) and mask == "causal"):
            return "mask-array"
        if sinks is not None:
            return "sinks"
        if abs(scale * math.sqrt(d) - 1.0) > 1e-6:
            return "nonstandard-scale"
        tc = cache.offset - 1
        if tc < 0 or not kva.should_dispatch(tc):
            return f"t-{tc}-outside-dispatch"
        return None

    def fused_step(self, queries, cache):
        """The one fused step on the padded buffers, logical length
        offset - 1 (the new entry enters at full precision)."""
        b, h, _, d = queries.shape
        q = queries.reshape(b, h, d).contiguous()
        nk = cache.new_keys.reshape(b, cache.n_kv_heads, d)
        nv = cache.new_values.reshape(b, cache.n_kv_heads, d)
        # the kernel depends on the cache's geometry and format only: plan once
        kernel = getattr(cache, "planned_kernel", None)
        if kernel is None:
            kernel = cache.planned_kernel = kva.plan_kernel(
                q, *cache.keys, *cache.values, nk, nv, bits=cache.bits, t_cached=cache.offset - 1)
        self.stats.kernels[kernel] = self.stats.kernels.get(kernel, 0) + 1
        out = kva.decode(q, *cache.keys, *cache.values, nk, nv, bits=cache.bits,
                         t_cached=cache.offset - 1, workspace=self.workspace)
        return out.reshape(b, h, 1, d)

    def __call__(self, queries, keys=None, values=None, *, cache=None, scale=1.0, mask=None,
                 sinks=None):
        st = self.stats
        if self.fused:
            why = self.ineligible(queries, cache, scale, mask, sinks)
            if why is None:
                st.calls += 1
                out = self.fused_step(queries, cache)
                if self.shadow:
                    ref = contract_reference(queries, cache)
                    stock = stock_attention(queries, cache, scale, mask)
                    st.shadow_fused_ref = max(st.shadow_fused_ref,
                                              float((out[:, :, 0].double() - ref).abs().max()))
                    st.shadow_stock_ref = max(st.shadow_stock_ref,
                                              float((stock[:, :, 0].double() - ref).abs().max()))
                    st.shadow_ref_mag = max(st.shadow_ref_mag, float(ref.abs().max()))
                    return stock
                return out
            st.fallback[why] = st.fallback.get(why, 0) + 1
        if sinks is not None:
            raise NotImplementedError("attention sinks are not served by the stock composition")
        return stock_attention(queries, cache, scale, mask)
