"""The serving hook on the device: the cache append is the canonical
quantizer written into cache slots (bit-exact, positions from the host or the
device, rows past the buffer not written), the fused step reached through the
router passes the oracle's verdict on the padded cache it built itself, and
the decode loop's wiring check (every decode call fused, shadow gap inside the
gate) holds on a small decoder."""

from __future__ import annotations

import numpy as np
import pytest

from oracle import quant
from tests.kvq_cases import judge_per_sequence, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch_cuda(native):
    import torch
    return torch


def _empty_cache(torch, b, hkv, cap, dh, bits, group, dtype):
    words = torch.zeros((b, hkv, cap, dh * bits // 32), dtype=torch.int32, device="cuda")
    scales = torch.zeros((b, hkv, cap, dh // group), dtype=dtype, device="cuda")
    return words, scales, torch.zeros_like(scales)


def _expect(w, bits, group):
    codes, s, b = quant.canonical_quantize(w.reshape(-1, w.shape[-1]), bits, group)
    return quant.pack_codes(codes, bits), s, b


@pytest.mark.parametrize("bits", [2, 3, 4, 6, 8])
@pytest.mark.parametrize("group", [32, 64, 128])
@pytest.mark.parametrize("dtype", ["float16", "float32"])
def test_append_at_host_position_is_the_canonical_quantizer(torch_cuda, bits, group, dtype):
    torch = torch_cuda
    from kernelverify_b200.pack import kv_attention as kva
    rng = np.random.default_rng(bits * 100 + group)
    b, hkv, n, cap, dh, pos = 3, 2, 5, 16, 128, 4
    w = rng.standard_normal((b, hkv, n, dh)).astype(dtype)
    w[rng.random(w.shape) < 0.02] *= 30
    cache = _empty_cache(torch, b, hkv, cap, dh, bits, group, getattr(torch, dtype))
    kva.cache_append(to_dev(w), *cache, bits, position=pos)
    torch.cuda.synchronize()
    words, scales, biases = (t.cpu().numpy() for t in cache)
    ew, es, eb = _expect(w, bits, group)
    got_w = words[:, :, pos:pos + n].reshape(-1, words.shape[-1]).view(np.uint32)
    assert np.array_equal(got_w, ew)
    assert np.array_equal(scales[:, :, pos:pos + n].reshape(es.shape).view(np.uint8),
                          es.view(np.uint8))
    assert np.array_equal(biases[:, :, pos:pos + n].reshape(eb.shape).view(np.uint8),
                          eb.view(np.uint8))
    untouched = np.ones(cap, dtype=bool)
    untouched[pos:pos + n] = False
    assert not words[:, :, untouched].any() and not scales[:, :, untouched].any()


def test_append_at_device_positions_per_sequence(torch_cuda):
    """Each sequence at its own device position; the last one runs past the
    buffer, whose rows are not written (the rest of that run is)."""
    torch = torch_cuda
    from kernelverify_b200.pack import kv_attention as kva
    rng = np.random.default_rng(11)
    b, hkv, n, cap, dh, bits = 4, 2, 3, 12, 64, 4
    w = rng.standard_normal((b, hkv, n, dh)).astype(np.float16)
    pos = np.array([0, 5, 9, 10], dtype=np.int32)
    cache = _empty_cache(torch, b, hkv, cap, dh, bits, 64, torch.float16)
    kva.cache_append(to_dev(w), *cache, bits, positions=to_dev(pos))
    torch.cuda.synchronize()
    words = cache[0].cpu().numpy().view(np.uint32)
    scales = cache[1].cpu().numpy()
    for s in range(b):
        ew, es, _ = _expect(w[s], bits, 64)
        ew, es = ew.reshape(hkv, n, -1), es.reshape(hkv, n, -1)
        for j in range(n):
            t = pos[s] + j
            if t < cap:
                assert np.array_equal(words[s, :, t], ew[:, j])
                assert np.array_equal(scales[s, :, t].view(np.uint16), es[:, j].view(np.uint16))
        written = set(int(pos[s]) + j for j in range(n) if pos[s] + j < cap)
        for t in set(range(cap)) - written:
            assert not words[s, :, t].any()


def test_append_rejects_host_overrun_and_shared_batch(torch_cuda):
    torch = torch_cuda
    from kernelverify_b200 import _native
    from kernelverify_b200.pack import kv_attention as kva
    cache = _empty_cache(torch, 2, 2, 8, 64, 4, 64, torch.float16)
    w = torch.zeros((2, 2, 3, 64), dtype=torch.float16, device="cuda")
    with pytest.raises(_native.KvqError, match="runs past t_stride"):
        kva.cache_append(w, *cache, 4, position=6)
    shared = tuple(t[0] for t in cache)         # [HKV, T, ...]: one cache for all rows
    with pytest.raises(ValueError):
        kva.cache_append(w, *shared, 4, position=0)


@pytest.mark.parametrize("bits", [4, 8, 3])
def test_router_fused_step_passes_the_oracle(torch_cuda, bits):
    """Prefill through update_and_fetch, one decode update, the fused step
    through the router on the padded cache (capacity past the logical
    length): judged per sequence against the fp64 contract reference of the
    raw values the cache was filled from."""
    torch = torch_cuda
    from kernelverify_b200.serving import DecodeRouter, QuantizedKVCache
    rng = np.random.default_rng(40 + bits)
    b, h, hkv, dh, p, cap = 2, 16, 4, 128, 300, 512
    kc = rng.standard_normal((b, hkv, p, dh)).astype(np.float16)
    vc = rng.standard_normal((b, hkv, p, dh)).astype(np.float16)
    nk = rng.standard_normal((b, hkv, 1, dh)).astype(np.float16)
    nv = rng.standard_normal((b, hkv, 1, dh)).astype(np.float16)
    q = (rng.standard_normal((b, h, 1, dh)) * 0.6).astype(np.float16)
    cache = QuantizedKVCache(b, hkv, dh, cap, bits, 64, torch.float16, "cuda")
    cache.update_and_fetch(to_dev(kc), to_dev(vc))
    keys, values = cache.update_and_fetch(to_dev(nk), to_dev(nv))
    router = DecodeRouter(fused=True)
    out = router(to_dev(q), keys, values, cache=cache, scale=dh ** -0.5)
    torch.cuda.synchronize()
    assert router.stats.calls == 1 and not router.stats.fallback
    assert tuple(out.shape) == (b, h, 1, dh)
    verdicts = judge_per_sequence(q[:, :, 0], kc, vc, nk[:, :, 0], nv[:, :, 0], bits,
                                  out[:, :, 0].cpu().numpy(), group=64)
    assert all(v.ok for v in verdicts), verdicts


def test_router_shadow_and_stock_agree_with_contract(torch_cuda):
    torch = torch_cuda
    from kernelverify_b200.serving import DecodeRouter, QuantizedKVCache
    rng = np.random.default_rng(5)
    b, h, hkv, dh, p = 1, 8, 2, 64, 200
    cache = QuantizedKVCache(b, hkv, dh, 256, 8, 64, torch.float16, "cuda")
    cache.update_and_fetch(to_dev(rng.standard_normal((b, hkv, p, dh)).astype(np.float16)),
                           to_dev(rng.standard_normal((b, hkv, p, dh)).astype(np.float16)))
    cache.update_and_fetch(to_dev(rng.standard_normal((b, hkv, 1, dh)).astype(np.float16)),
                           to_dev(rng.standard_normal((b, hkv, 1, dh)).astype(np.float16)))
    q = to_dev((rng.standard_normal((b, h, 1, dh)) * 0.6).astype(np.float16))
    router = DecodeRouter(fused=True, shadow=True)
    router(q, cache=cache, scale=dh ** -0.5)
    st = router.stats
    assert st.calls == 1
    assert st.shadow_fused_ref < 4e-3 * max(1.0, st.shadow_ref_mag)
    # stock reads the new entry back quantized at 8 bits: near, not at, the contract
    assert st.shadow_stock_ref < 5e-2 * max(1.0, st.shadow_ref_mag)


def test_decode_loop_wiring_smoke(torch_cuda):
    from kernelverify_b200 import decode_loop as dl
    model = dl.Decoder(dl.TINY)
    report = dl.smoke(model, prompt_len=40, gen=6)
    assert report["ok"], report
    assert report["decode_steps"] == 5 and report["fused_calls"] == 5 * dl.TINY.n_layers


def test_decode_loop_arms_agree_on_first_token(torch_cuda):
    """Prefill is stock in every arm, so the first generated token of the
    fused and the stock quantized arm is the same token."""
    from kernelverify_b200 import decode_loop as dl
    from kernelverify_b200.serving import DecodeRouter
    model = dl.Decoder(dl.TINY, seed=3)
    prompt = dl.make_prompt(model, 2, 33)
    ta, _ = dl.generate(model, prompt, 4, 4, DecodeRouter(fused=True))
    tb, _ = dl.generate(model, prompt, 4, 4, DecodeRouter(fused=False))
    assert bool((ta[:, 0] == tb[:, 0]).all())


@pytest.mark.parametrize("arm", ["fused", "stock", "fp16"])
def test_captured_step_replays_the_eager_step(torch_cuda, arm):
    """The captured decode step (device positions, device-side append, the
    fused kernel with seq_lens) replays exactly what the same step computes
    eagerly, token for token, and advances the device positions."""
    torch = torch_cuda
    from kernelverify_b200 import decode_loop as dl
    model = dl.Decoder(dl.TINY, seed=4)
    d = dl.CapturedDecode(model, batch=3, capacity=56, arm=arm, bits=4)
    d.prefill_synthetic(40, seed=1)
    d.tok.fill_(7)
    d.capture()
    replayed = []
    for _ in range(4):
        d.graph.replay()
        replayed.append(d.tok.clone())
    assert d.pos.tolist() == [44, 44, 44]
    d.rewind(40)
    d.tok.fill_(7)
    eager = []
    with torch.inference_mode():
        for _ in range(4):
            d._step()
            eager.append(d.tok.clone())
    torch.cuda.synchronize()
    for a, b in zip(replayed, eager):
        assert torch.equal(a, b)


def test_captured_ab_reports_every_arm(torch_cuda):
    from kernelverify_b200 import decode_loop as dl
    model = dl.Decoder(dl.TINY)
    row = dl.ab_graph(model, batch=2, prompt=64, steps=8, bits=4, rounds=2)
    for arm in dl.CapturedDecode.ARMS:
        assert row[f"{arm}_tps"] > 0
    assert "ratio_AB" in row and "demotion_C_beats_A" in row


def test_serving_caches_keep_the_tensor_core_kernels(torch_cuda):
    """Any capacity: the cache pads its rows so 4-bit DH-128 fp16 steps plan
    the tensor-core kernels, in the router and in the captured step."""
    torch = torch_cuda
    from kernelverify_b200 import decode_loop as dl
    from kernelverify_b200.serving import DecodeRouter, QuantizedKVCache
    cache = QuantizedKVCache(2, 2, 128, 1001, 4, 64, torch.float16, "cuda")
    assert cache.t_stride % 64 == 0 and cache.t_stride >= 1001
    k = torch.randn(2, 2, 37, 128, device="cuda", dtype=torch.float16)
    cache.update_and_fetch(k, k)
    cache.update_and_fetch(k[:, :, :1].contiguous(), k[:, :, :1].contiguous())
    router = DecodeRouter()
    router(torch.randn(2, 8, 1, 128, device="cuda", dtype=torch.float16), cache=cache,
           scale=128 ** -0.5)
    assert router.stats.kernels == {"tensor-core": 1}
    shape = dl.DecoderShape(n_layers=1, hidden=512, n_heads=4, n_kv_heads=2, head_dim=128,
                            intermediate=512, vocab=256)
    d = dl.CapturedDecode(dl.Decoder(shape), batch=2, capacity=8258, arm="fused", bits=4)
    d.prefill_synthetic(100)
    d.capture()
    assert d.fused_kernel == "tensor-core"
