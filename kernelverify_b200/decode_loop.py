"""End-to-end decode tokens/s with the fused kernel in the loop.

The B200 form of the reference's end-to-end A/B (bench/spike_mlx_e2e.py):
does routing the decode-step attention to the fused quantized-KV kernel move
decode tokens/s? A Qwen3-4B-shaped decoder (36 layers, hidden 2560, 32 query /
8 cache heads of 128, SwiGLU 9728, q/k RMSNorm, RoPE theta 1e6, tied
embeddings; random-initialised fp16 weights -- no checkpoint is available
offline -- so tokens/s transfers and the text does not) runs greedy
generation in three arms, interleaved within every round:

  A  fused kernel, quantized KV cache (the candidate)
  B  stock composition, quantized KV cache (the incumbent; primary ratio A/B)
  C  stock attention, fp16 cache (the third arm; if C beats A the result is
     demoted whatever A/B says, spike_mlx_e2e.py:25-30)

Decode tokens/s excludes prefill and the first token (spike_mlx_e2e.py:
276-297) and counts tokens of every sequence in the batch. Prefill goes
through stock in every arm (the router whitelists it). The reference model ran
4-bit weights under MLX on an M-series GPU; here the weights are fp16 under
torch/cuBLAS, so only the attention arm differs between A and B.

    python -m kernelverify_b200.decode_loop --smoke
    python -m kernelverify_b200.decode_loop --ab [--bits 4 8] [--prompt 512 896]
"""

from __future__ import annotations

import argparse
import json
import statistics
import sys
import time
from dataclasses import dataclass

from kernelverify_b200.pack import kv_attention as kva
from kernelverify_b200.serving import (DecodeRouter, FullPrecisionKVCache, QuantizedKVCache)

GROUP_SIZE = 64


def _torch():
    import torch
    return torch


@dataclass(frozen=True)
class DecoderShape:
    n_layers: int = 36
    hidden: int = 2560
    n_heads: int = 32
    n_kv_heads: int = 8
    head_dim: int = 128
    intermediate: int = 9728
    vocab: int = 151936
    rope_theta: float = 1_000_000.0
    eps: float = 1e-6


QWEN3_4B = DecoderShape()
TINY = DecoderShape(n_layers=2, hidden=256, n_heads=8, n_kv_heads=2, head_dim=64,
                    intermediate=512, vocab=1024)

# prompt length -> generated tokens, as the reference's A/B (spike_mlx_e2e.py:84-88)
GEN_TOKENS = {512: 480, 896: 120}


class Decoder:
    """Random-initialised decoder of `shape` in `dtype` on `device`. Weights
    are N(0, 1/fan_in); norms are ones. q/k/v and gate/up projections are one
    matmul each."""

    def __init__(self, shape: DecoderShape, device="cuda", dtype=None, seed: int = 0):
        torch = _torch()
        dtype = torch.float16 if dtype is None else dtype
        self.shape, self.device, self.dtype = shape, torch.device(device), dtype
        g = torch.Generator(device=self.device)
        g.manual_seed(seed)
        s = shape
        qkv = (s.n_heads + 2 * s.n_kv_heads) * s.head_dim

        def w(rows, cols):
            t = torch.empty((rows, cols), dtype=dtype, device=self.device)
            return t.normal_(0.0, cols ** -0.5, generator=g)

        self.embed = w(s.vocab, s.hidden)
        self.layers = []
        for _ in range(s.n_layers):
            self.layers.append({
                "wqkv": w(qkv, s.hidden),
                "wo": w(s.hidden, s.n_heads * s.head_dim),
                "wgu": w(2 * s.intermediate, s.hidden),
                "wd": w(s.hidden, s.intermediate),
                "n_in": torch.ones(s.hidden, dtype=dtype, device=self.device),
                "n_post": torch.ones(s.hidden, dtype=dtype, device=self.device),
                "n_q": torch.ones(s.head_dim, dtype=dtype, device=self.device),
                "n_k": torch.ones(s.head_dim, dtype=dtype, device=self.device),
            })
        self.n_final = torch.ones(s.hidden, dtype=dtype, device=self.device)
        half = s.head_dim // 2
        self.inv_freq = 1.0 / (s.rope_theta ** (torch.arange(half, device=self.device,
                                                             dtype=torch.float32) / half))

    def rope_tables(self, positions):
        """cos, sin [B or 1, 1, L, DH] for float32 positions [B or 1, L]."""
        torch = _torch()
        ang = positions[..., None] * self.inv_freq
        cos = torch.cat([ang.cos(), ang.cos()], dim=-1).to(self.dtype)[:, None]
        sin = torch.cat([ang.sin(), ang.sin()], dim=-1).to(self.dtype)[:, None]
        return cos, sin

    @staticmethod
    def _rope(x, cos, sin):
        """Rotate-half RoPE on x [B, heads, L, DH]."""
        torch = _torch()
        x1, x2 = x.chunk(2, dim=-1)
        return x * cos + torch.cat([-x2, x1], dim=-1) * sin

    def run(self, tokens, cos, sin, attend):
        """tokens [B, L] -> last-position logits [B, vocab]. attend(i, q, k, v)
        is layer i's attention on post-RoPE q [B, H, L, DH], k / v
        [B, HKV, L, DH] (it owns the cache update)."""
        torch = _torch()
        F = torch.nn.functional
        s = self.shape
        b, n = tokens.shape
        x = F.embedding(tokens, self.embed)
        for i, lw in enumerate(self.layers):
            h = F.rms_norm(x, (s.hidden,), lw["n_in"], s.eps)
            qkv = F.linear(h, lw["wqkv"]).view(b, n, s.n_heads + 2 * s.n_kv_heads, s.head_dim)
            q, k, v = qkv.split([s.n_heads, s.n_kv_heads, s.n_kv_heads], dim=2)
            q = F.rms_norm(q, (s.head_dim,), lw["n_q"], s.eps).transpose(1, 2)
            k = F.rms_norm(k, (s.head_dim,), lw["n_k"], s.eps).transpose(1, 2)
            v = v.transpose(1, 2)
            a = attend(i, self._rope(q, cos, sin), self._rope(k, cos, sin), v)
            x = x + F.linear(a.transpose(1, 2).reshape(b, n, s.n_heads * s.head_dim), lw["wo"])
            h = F.rms_norm(x, (s.hidden,), lw["n_post"], s.eps)
            gate, up = F.linear(h, lw["wgu"]).chunk(2, dim=-1)
            x = x + F.linear(F.silu(gate) * up, lw["wd"])
        x = F.rms_norm(x[:, -1], (s.hidden,), self.n_final, s.eps)
        return F.linear(x, self.embed)

    def forward(self, tokens, caches, router):
        """tokens [B, L] -> last-position logits [B, vocab]; appends L
        positions to every layer's cache through its update step and routes
        the attention call (the eager decode loop)."""
        torch = _torch()
        n = tokens.shape[1]
        pos0 = caches[0].offset
        t = torch.arange(pos0, pos0 + n, device=self.device, dtype=torch.float32)[None]
        cos, sin = self.rope_tables(t)
        scale = self.shape.head_dim ** -0.5

        def attend(i, q, k, v):
            keys, values = caches[i].update_and_fetch(k, v)
            return router(q, keys, values, cache=caches[i], scale=scale,
                          mask="causal" if n > 1 else None)

        return self.run(tokens, cos, sin, attend)

    def caches(self, batch: int, capacity: int, kv_bits: int | None):
        s = self.shape
        if kv_bits is None:
            return [FullPrecisionKVCache(batch, s.n_kv_heads, s.head_dim, capacity, self.dtype,
                                         self.device) for _ in range(s.n_layers)]
        return [QuantizedKVCache(batch, s.n_kv_heads, s.head_dim, capacity, kv_bits, GROUP_SIZE,
                                 self.dtype, self.device) for _ in range(s.n_layers)]


def generate(model: Decoder, prompt, gen_tokens: int, kv_bits: int | None, router: DecodeRouter):
    """Greedy generation of gen_tokens tokens after prompt [B, P]; returns
    (tokens [B, gen_tokens], decode tokens/s over the gen_tokens - 1 steps
    after the first token, wall clock with the device synchronised)."""
    torch = _torch()
    b, p = prompt.shape
    caches = model.caches(b, p + gen_tokens, kv_bits)
    out = []

    def sync():
        if model.device.type == "cuda":
            torch.cuda.synchronize(model.device)

    with torch.inference_mode():
        logits = model.forward(prompt, caches, router)          # prefill + first token
        tok = logits.argmax(dim=-1, keepdim=True)
        out.append(tok)
        sync()
        t0 = time.perf_counter()
        for _ in range(gen_tokens - 1):
            logits = model.forward(tok, caches, router)
            tok = logits.argmax(dim=-1, keepdim=True)
            out.append(tok)
        sync()
        dt = time.perf_counter() - t0
    steps = gen_tokens - 1
    return torch.cat(out, dim=1), (steps * b / dt if steps else 0.0)


class CapturedDecode:
    """One decode step of every sequence, captured as a CUDA graph: token,
    RoPE position, cache append, attention and the greedy pick all read and
    write device buffers, so a replay needs nothing from the host and
    tokens/s measures the GPU rather than the Python launch loop.

    arm "fused": quantized cache, appends at the device positions and the
      fused kernel over the padded buffers with `seq_lens` = positions (the
      library's ragged-length form, planned for the capacity);
    arm "stock": quantized cache, every position of the capacity dequantized
      and torch attention with a length mask (what the stock composition can
      do without a host length);
    arm "fp16": full-precision cache and torch attention with the same mask.
    The capacity should be the final length (prompt + generated), so the
    stock arms' reads past the current length stay small."""

    ARMS = ("fused", "stock", "fp16")

    def __init__(self, model: Decoder, batch: int, capacity: int, arm: str, bits: int = 4):
        torch = _torch()
        if arm not in self.ARMS:
            raise ValueError(f"arm {arm!r} not in {self.ARMS}")
        self.model, self.batch, self.capacity, self.arm, self.bits = (model, batch, capacity, arm,
                                                                      bits)
        self.caches = model.caches(batch, capacity, None if arm == "fp16" else bits)
        self.tok = torch.zeros((batch, 1), dtype=torch.long, device=model.device)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=model.device)
        self.workspace = kva.Workspace()
        self.graph = None
        self.length = 0
        self.fused_kernel = None

    def prefill_synthetic(self, length: int, seed: int = 0, chunk: int = 1024) -> None:
        """Fill positions [0, length) of every layer with N(0, 1) keys and
        values (the work of a decode step does not depend on the values);
        every arm built with the same seed holds the same values, quantized or
        not."""
        torch = _torch()
        s = self.model.shape
        g = torch.Generator(device=self.model.device)
        g.manual_seed(seed)
        for cache in self.caches:
            for c0 in range(0, length, chunk):
                n = min(chunk, length - c0)
                shape = (self.batch, s.n_kv_heads, n, s.head_dim)
                k = torch.randn(shape, generator=g, device=self.model.device).to(self.model.dtype)
                v = torch.randn(shape, generator=g, device=self.model.device).to(self.model.dtype)
                if isinstance(cache, QuantizedKVCache):
                    kva.cache_append(k.contiguous(), *cache.keys, cache.bits, position=c0)
                    kva.cache_append(v.contiguous(), *cache.values, cache.bits, position=c0)
                else:
                    cache.k[:, :, c0:c0 + n] = k
                    cache.v[:, :, c0:c0 + n] = v
            cache.offset = length
        self.pos.fill_(length)
        self.length = length

    def _attend(self, i, q, k, v):
        torch = _torch()
        F = torch.nn.functional
        cache = self.caches[i]
        s = self.model.shape
        scale = s.head_dim ** -0.5
        b = q.shape[0]
        if self.arm == "fused":
            cache.append_at(k, v, self.pos)
            if self.fused_kernel is None:
                self.fused_kernel = kva.plan_kernel(
                    q.reshape(b, s.n_heads, s.head_dim).contiguous(), *cache.keys, *cache.values,
                    cache.new_keys.reshape(b, s.n_kv_heads, s.head_dim),
                    cache.new_values.reshape(b, s.n_kv_heads, s.head_dim), bits=cache.bits,
                    t_cached=self.capacity - 1, seq_lens=self.pos)
            out = kva.decode(q.reshape(b, s.n_heads, s.head_dim).contiguous(), *cache.keys,
                             *cache.values, cache.new_keys.reshape(b, s.n_kv_heads, s.head_dim),
                             cache.new_values.reshape(b, s.n_kv_heads, s.head_dim),
                             bits=cache.bits, t_cached=self.capacity - 1, seq_lens=self.pos,
                             workspace=self.workspace)
            return out.reshape(b, s.n_heads, 1, s.head_dim)
        cache.append_at(k, v, self.pos)
        if self.arm == "stock":
            kk = kva.dequant(*cache.keys, cache.bits).to(q.dtype)
            vv = kva.dequant(*cache.values, cache.bits).to(q.dtype)
        else:
            kk, vv = cache.k, cache.v
        rows = kk.shape[2]
        live = (torch.arange(rows, device=q.device)[None, :]
                <= self.pos[:, None]).view(b, 1, 1, rows)
        # the R query heads of a cache head ride as R query rows (contiguous
        # GQA blocks), so torch's masked kernel reads each cache head once
        r = s.n_heads // s.n_kv_heads
        out = F.scaled_dot_product_attention(q.reshape(b, s.n_kv_heads, r, s.head_dim), kk, vv,
                                             attn_mask=live, scale=scale)
        return out.reshape(b, s.n_heads, 1, s.head_dim)

    def _step(self):
        torch = _torch()
        cos, sin = self.model.rope_tables(self.pos.float()[:, None])
        logits = self.model.run(self.tok, cos, sin, self._attend)
        self.tok.copy_(logits.argmax(dim=-1, keepdim=True))
        self.pos.add_(1)

    def capture(self, warmup: int = 2) -> None:
        """Run `warmup` eager steps on a side stream (allocations, library
        attribute lookups), rewind, then capture one step."""
        torch = _torch()
        start, tok0 = self.pos.clone(), self.tok.clone()
        side = torch.cuda.Stream(self.model.device)
        side.wait_stream(torch.cuda.current_stream(self.model.device))
        with torch.inference_mode(), torch.cuda.stream(side):
            for _ in range(warmup):
                self._step()
        torch.cuda.current_stream(self.model.device).wait_stream(side)
        self.pos.copy_(start)
        self.tok.copy_(tok0)
        self.graph = torch.cuda.CUDAGraph()
        with torch.inference_mode(), torch.cuda.graph(self.graph):
            self._step()
        torch.cuda.synchronize(self.model.device)

    def run(self, steps: int) -> float:
        """Replay `steps` decode steps; decode tokens/s of the batch, timed
        with CUDA events around the replays."""
        torch = _torch()
        if self.graph is None:
            self.capture()
        if self.length + steps >= self.capacity:
            raise ValueError(f"{steps} steps from length {self.length} overrun capacity "
                             f"{self.capacity}")
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            self.graph.replay()
        stop.record()
        stop.synchronize()
        self.length += steps
        return steps * self.batch / (start.elapsed_time(stop) / 1e3)

    def rewind(self, length: int) -> None:
        """Back to `length` cached positions (the entries past it are
        overwritten by the next steps)."""
        self.pos.fill_(length)
        self.length = length


def ab_graph(model: Decoder, batch: int, prompt: int, steps: int, bits: int = 4,
             rounds: int = 3, arms=CapturedDecode.ARMS) -> dict:
    """Interleaved rounds of the captured step per arm at one (batch, prompt
    length): median decode tokens/s per arm, spreads, A/B and the demotion
    flag."""
    capacity = prompt + steps + 2
    runs = {}
    for arm in arms:
        d = CapturedDecode(model, batch, capacity, arm, bits)
        d.prefill_synthetic(prompt, seed=prompt + bits)
        d.capture()
        runs[arm] = d
    vals = {arm: [] for arm in arms}
    for _ in range(rounds):
        for arm in arms:
            runs[arm].rewind(prompt)
            vals[arm].append(runs[arm].run(steps))
    med = statistics.median
    row = {"mode": "graph", "bits": bits, "batch": batch, "prompt": prompt, "steps": steps,
           "rounds": rounds}
    if "fused" in arms:
        row["fused_kernel"] = runs["fused"].fused_kernel
    for arm in arms:
        row[f"{arm}_tps"] = round(med(vals[arm]), 1)
        row[f"{arm}_spread_pct"] = round(spread_pct(vals[arm]), 2)
    if "fused" in arms and "stock" in arms:
        row["ratio_AB"] = round(med(vals["fused"]) / med(vals["stock"]), 4)
    if "fused" in arms and "fp16" in arms:
        row["ratio_AC"] = round(med(vals["fused"]) / med(vals["fp16"]), 4)
        row["demotion_C_beats_A"] = med(vals["fp16"]) > med(vals["fused"])
    for d in runs.values():
        d.graph = None
    return row


def make_prompt(model: Decoder, batch: int, length: int, seed: int = 0):
    torch = _torch()
    g = torch.Generator(device="cpu")
    g.manual_seed(seed)
    return torch.randint(0, model.shape.vocab, (batch, length), generator=g).to(model.device)


def spread_pct(xs) -> float:
    """(max - min) / median, in percent."""
    m = statistics.median(xs)
    return 100.0 * (max(xs) - min(xs)) / m if m else 0.0


def smoke(model: Decoder, prompt_len: int = 64, gen: int = 8, bits=(8, 4)) -> dict:
    """Wiring check, no timing: every decode-shaped call goes fused, no hard
    fallback, and in a shadow round the fused output sits within 4 fp16 ulps
    of the output magnitude of the fp64 contract composition
    (spike_mlx_e2e.py:299-340)."""
    n_layers = model.shape.n_layers
    prompt = make_prompt(model, 1, prompt_len)
    router = DecodeRouter(fused=True, shadow=True)
    generate(model, prompt, gen, bits[0], router)
    st = router.stats
    bound = 4e-3 * max(1.0, st.shadow_ref_mag)
    report = {"shadow_calls": st.calls, "decode_steps": st.calls // n_layers,
              "fallbacks": dict(st.fallback), "hard_fallbacks": st.hard_fallbacks(),
              "fused_gap": st.shadow_fused_ref, "stock_gap": st.shadow_stock_ref,
              "gate": bound, "ref_mag": st.shadow_ref_mag}
    ok = (st.calls > 0 and st.calls % n_layers == 0 and not st.hard_fallbacks()
          and st.shadow_fused_ref < bound)
    router = DecodeRouter(fused=True)
    generate(model, prompt, gen, bits[1], router)
    report["fused_calls"] = router.stats.calls
    report["fused_kernels"] = dict(router.stats.kernels)
    ok = ok and router.stats.calls == (gen - 1) * n_layers and not router.stats.hard_fallbacks()
    report["ok"] = bool(ok)
    return report


def ab(model: Decoder, bits_list, prompts, rounds: int | None = None, batch: int = 1,
       gen_tokens: dict | None = None) -> list:
    """Interleaved A/B/C rounds per (bits, prompt length); medians and
    spreads per arm, the A/B ratio, and the demotion flag."""
    rows = []
    gen_tokens = gen_tokens or GEN_TOKENS
    for bits in bits_list:
        for p in prompts:
            prompt = make_prompt(model, batch, p, seed=p + bits)
            g = gen_tokens.get(p, 128)
            n = rounds or (5 if g >= 400 else 9)
            a_r, b_r, c_r = DecodeRouter(fused=True), DecodeRouter(fused=False), \
                DecodeRouter(fused=False)
            generate(model, prompt, min(g, 16), bits, a_r)    # warm every arm once
            generate(model, prompt, min(g, 16), bits, b_r)
            generate(model, prompt, min(g, 16), None, c_r)
            a_r.reset()
            a_v, b_v, c_v = [], [], []
            for _ in range(n):
                a_v.append(generate(model, prompt, g, bits, a_r)[1])
                b_v.append(generate(model, prompt, g, bits, b_r)[1])
                c_v.append(generate(model, prompt, g, None, c_r)[1])
            med = statistics.median
            rows.append({
                "bits": bits, "prompt": p, "gen": g, "batch": batch, "rounds": n,
                "fused_calls": a_r.stats.calls, "hard_fallbacks": a_r.stats.hard_fallbacks(),
                "fused_kernels": dict(a_r.stats.kernels),
                "armA_tps": round(med(a_v), 2), "armB_tps": round(med(b_v), 2),
                "armC_fp16_tps": round(med(c_v), 2),
                "armA_spread_pct": round(spread_pct(a_v), 2),
                "armB_spread_pct": round(spread_pct(b_v), 2),
                "armC_spread_pct": round(spread_pct(c_v), 2),
                "ratio_AB": round(med(a_v) / med(b_v), 4),
                "demotion_C_beats_A": med(c_v) > med(a_v)})
    return rows


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    mode = ap.add_mutually_exclusive_group(required=True)
    mode.add_argument("--smoke", action="store_true")
    mode.add_argument("--ab", action="store_true")
    mode.add_argument("--ab-graph", action="store_true",
                      help="the captured-step A/B (GPU-bound tokens/s)")
    ap.add_argument("--tiny", action="store_true", help="a 2-layer decoder instead of Qwen3-4B")
    ap.add_argument("--bits", type=int, nargs="*", default=[4, 8])
    ap.add_argument("--prompt", type=int, nargs="*", default=[512, 896])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--rounds", type=int, default=None)
    ap.add_argument("--steps", type=int, default=64, help="decode steps per round (--ab-graph)")
    args = ap.parse_args(argv)
    model = Decoder(TINY if args.tiny else QWEN3_4B)
    if args.smoke:
        report = smoke(model)
        print(json.dumps(report))
        return 0 if report["ok"] else 1
    if args.ab_graph:
        for bits in args.bits:
            for p in args.prompt:
                print(json.dumps(ab_graph(model, args.batch, p, args.steps, bits,
                                          args.rounds or 3)), flush=True)
        return 0
    rows = ab(model, args.bits, args.prompt, args.rounds, args.batch)
    for row in rows:
        print(json.dumps(row))
    return 1 if any(r["hard_fallbacks"] for r in rows) else 0


if __name__ == "__main__":
    sys.exit(main())
