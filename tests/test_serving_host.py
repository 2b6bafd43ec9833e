"""Host logic of the serving hook, on CPU: the router's eligibility reasons
(bench/spike_mlx_e2e.py:126-152 labels each fallback), fallback counting,
and the decode loop's cache bookkeeping (incremental decode through the
stock path equals one full forward: RoPE positions and the bottom-right
causal mask of a chunk with prior context)."""

from __future__ import annotations

import math

import pytest
import torch

from kernelverify_b200 import decode_loop as dl
from kernelverify_b200.serving import (DecodeRouter, FullPrecisionKVCache, QuantizedKVCache,
                                       _causal_mask, stock_attention)


def _qcache(b=1, hkv=2, dh=64, cap=16, bits=4, group=64, offset=5, stash_len=1):
    c = QuantizedKVCache(b, hkv, dh, cap, bits, group, torch.float16, device="cpu")
    c.offset = offset
    if stash_len:
        c.new_keys = torch.zeros(b, hkv, stash_len, dh, dtype=torch.float16)
        c.new_values = torch.zeros_like(c.new_keys)
    return c


def _q(b=1, h=8, n=1, dh=64, dtype=torch.float16):
    return torch.zeros(b, h, n, dh, dtype=dtype)


def test_eligible_decode_call():
    c = _qcache()
    assert DecodeRouter.ineligible(_q(), c, 64 ** -0.5) is None
    assert DecodeRouter.ineligible(_q(), c, 64 ** -0.5, mask="causal") is None


@pytest.mark.parametrize("case, reason", [
    (dict(q=dict(n=7)), "prefill-L7"),
    (dict(cache="full"), "cache-not-quantized"),
    (dict(c=dict(stash_len=0)), "no-stashed-new-entry"),
    (dict(c=dict(stash_len=3)), "stash-L3"),
    (dict(q=dict(dtype=torch.float32)), "dtype-float32"),
    (dict(q=dict(h=7)), "heads-B1-H7-over-HKV2"),
    (dict(q=dict(b=2)), "heads-B2-H8-over-HKV2"),
    (dict(mask=torch.ones(1, 1, dtype=torch.bool)), "mask-array"),
    (dict(sinks=torch.zeros(8)), "sinks"),
    (dict(scale=1.0), "nonstandard-scale"),
    (dict(c=dict(offset=0)), "t--1-outside-dispatch"),
])
def test_ineligible_reasons(case, reason):
    c = _qcache(**case.get("c", {}))
    if case.get("cache") == "full":
        c = FullPrecisionKVCache(1, 2, 64, 16, torch.float16, device="cpu")
    q = _q(**case.get("q", {}))
    why = DecodeRouter.ineligible(q, c, case.get("scale", 64 ** -0.5), case.get("mask"),
                                  case.get("sinks"))
    assert why == reason


def test_prefill_label_wins_over_cache_state():
    """The query length is checked first: a prefill chunk over a cache with
    no stash is still a prefill fallback, not a hard one."""
    c = _qcache(stash_len=0)
    assert DecodeRouter.ineligible(_q(n=4), c, 64 ** -0.5) == "prefill-L4"


def test_fallbacks_are_counted_and_prefill_whitelisted():
    r = DecodeRouter(fused=True)
    c = FullPrecisionKVCache(1, 2, 64, 16, torch.float32, device="cpu")
    k = torch.randn(1, 2, 4, 64)
    c.update_and_fetch(k, k)
    r(torch.randn(1, 8, 4, 64), cache=c, scale=0.125, mask="causal")
    c.update_and_fetch(k[:, :, :1], k[:, :, :1])
    r(torch.randn(1, 8, 1, 64), cache=c, scale=0.125)
    assert r.stats.calls == 0
    assert r.stats.fallback == {"prefill-L4": 1, "cache-not-quantized": 1}
    assert r.stats.hard_fallbacks() == {"cache-not-quantized": 1}


def test_causal_mask_is_bottom_right_aligned():
    m = _causal_mask(3, 5, "cpu")
    assert m.tolist() == [[True, True, True, False, False],
                          [True, True, True, True, False],
                          [True, True, True, True, True]]
    assert _causal_mask(1, 5, "cpu") is None


def test_stock_attention_matches_explicit_softmax():
    torch.manual_seed(0)
    c = FullPrecisionKVCache(2, 2, 64, 16, torch.float64, device="cpu")
    k, v = torch.randn(2, 2, 9, 64, dtype=torch.float64), torch.randn(2, 2, 9, 64,
                                                                     dtype=torch.float64)
    c.update_and_fetch(k, v)
    q = torch.randn(2, 8, 1, 64, dtype=torch.float64)
    out = stock_attention(q, c, 64 ** -0.5)
    kk, vv = k.repeat_interleave(4, dim=1), v.repeat_interleave(4, dim=1)
    p = torch.softmax(torch.einsum("bhqd,bhtd->bhqt", q, kk) / math.sqrt(64), dim=-1)
    assert torch.allclose(out, torch.einsum("bhqt,bhtd->bhqd", p, vv), atol=1e-12)


def test_cache_capacity_is_enforced():
    c = FullPrecisionKVCache(1, 2, 64, 4, torch.float32, device="cpu")
    c.update_and_fetch(torch.zeros(1, 2, 3, 64), torch.zeros(1, 2, 3, 64))
    with pytest.raises(ValueError, match="cache full"):
        c.update_and_fetch(torch.zeros(1, 2, 2, 64), torch.zeros(1, 2, 2, 64))


def test_incremental_decode_equals_full_forward():
    """Prefill 6 tokens then decode 3 one at a time through the stock path:
    each step's logits equal those of one forward over the whole prefix."""
    model = dl.Decoder(dl.TINY, device="cpu", dtype=torch.float32, seed=1)
    toks = torch.randint(0, dl.TINY.vocab, (2, 9), generator=torch.Generator().manual_seed(2))
    router = DecodeRouter(fused=False)
    caches = model.caches(2, 9, None)
    with torch.inference_mode():
        got = [model.forward(toks[:, :6], caches, router)]
        for i in range(6, 9):
            got.append(model.forward(toks[:, i:i + 1], caches, router))
        for j, n in enumerate(range(6, 10)):
            want = model.forward(toks[:, :n], model.caches(2, 9, None), router)
            assert torch.allclose(got[j], want, atol=2e-4, rtol=1e-4), n


def test_generate_counts_decode_tokens_per_sequence():
    model = dl.Decoder(dl.TINY, device="cpu", dtype=torch.float32)
    prompt = dl.make_prompt(model, 3, 5)
    toks, tps = dl.generate(model, prompt, 4, None, DecodeRouter(fused=False))
    assert toks.shape == (3, 4) and tps > 0
