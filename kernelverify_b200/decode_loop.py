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

    def _rope(self, x, pos0: int):
        """Rotate-half RoPE on x [B, heads, L, DH] at positions pos0 + [0, L)."""
        torch = _torch()
        n = x.shape[2]
        t = torch.arange(pos0, pos0 + n, device=self.device, dtype=torch.float32)
        ang = t[:, None] * self.inv_freq[None, :]
        cos = torch.cat([ang.cos(), ang.cos()], dim=-1).to(x.dtype)
        sin = torch.cat([ang.sin(), ang.sin()], dim=-1).to(x.dtype)
        x1, x2 = x.chunk(2, dim=-1)
        return x * cos + torch.cat([-x2, x1], dim=-1) * sin

    def forward(self, tokens, caches, router):
        """tokens [B, L] -> last-position logits [B, vocab]; appends L
        positions to every layer's cache."""
        torch = _torch()
        F = torch.nn.functional
        s = self.shape
        b, n = tokens.shape
        pos0 = caches[0].offset
        x = F.embedding(tokens, self.embed)
        for lw, cache in zip(self.layers, caches):
            h = F.rms_norm(x, (s.hidden,), lw["n_in"], s.eps)
            qkv = F.linear(h, lw["wqkv"]).view(b, n, s.n_heads + 2 * s.n_kv_heads, s.head_dim)
            q, k, v = qkv.split([s.n_heads, s.n_kv_heads, s.n_kv_heads], dim=2)
            q = F.rms_norm(q, (s.head_dim,), lw["n_q"], s.eps).transpose(1, 2)
            k = F.rms_norm(k, (s.head_dim,), lw["n_k"], s.eps).transpose(1, 2)
            v = v.transpose(1, 2)
            q, k = self._rope(q, pos0), self._rope(k, pos0)
            keys, values = cache.update_and_fetch(k, v)
            a = router(q, keys, values, cache=cache, scale=s.head_dim ** -0.5,
                       mask="causal" if n > 1 else None)
            x = x + F.linear(a.transpose(1, 2).reshape(b, n, s.n_heads * s.head_dim), lw["wo"])
            h = F.rms_norm(x, (s.hidden,), lw["n_post"], s.eps)
            gate, up = F.linear(h, lw["wgu"]).chunk(2, dim=-1)
            x = x + F.linear(F.silu(gate) * up, lw["wd"])
        x = F.rms_norm(x[:, -1], (s.hidden,), self.n_final, s.eps)
        return F.linear(x, self.embed)

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
    ap.add_argument("--tiny", action="store_true", help="a 2-layer decoder instead of Qwen3-4B")
    ap.add_argument("--bits", type=int, nargs="*", default=[4, 8])
    ap.add_argument("--prompt", type=int, nargs="*", default=[512, 896])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--rounds", type=int, default=None)
    args = ap.parse_args(argv)
    model = Decoder(TINY if args.tiny else QWEN3_4B)
    if args.smoke:
        report = smoke(model)
        print(json.dumps(report))
        return 0 if report["ok"] else 1
    rows = ab(model, args.bits, args.prompt, args.rounds, args.batch)
    for row in rows:
        print(json.dumps(row))
    return 1 if any(r["hard_fallbacks"] for r in rows) else 0


if __name__ == "__main__":
    sys.exit(main())
