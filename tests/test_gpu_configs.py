"""Every BASELINE configuration at its own geometry and split plan, on a B200.

The workload is built the way bench.py builds the one it times: N(0,1) fp32
draws on the device (config 3: 1 % of the entries x20), cast to fp16,
quantized on the device by the library's canonical quantizer, one cache per
sequence (config 4: rows padded to a multiple of 64, ragged `seq_lens` on the
device). The step then runs through the public call the bench times --
`kv_attention.decode` (kvq_decode: the library's own split plan for that
geometry), and for config 5 also the sequence-split decoder on one rank -- so
the split plan under test is the timed one.

The oracle (fp64 reference, the reference's floored four-member tolerance)
judges a seeded sample of (sequence, cache head) units from their raw fp16
rows, which it quantizes itself; each unit is its own case, which is stricter
than a whole-batch tolerance (per-case max|ref|). Units are judged in a
spawned process pool. Test infrastructure: the oracle is the checker, never
the thing measured.
"""

from __future__ import annotations

import numpy as np
import pytest

from tests.kvq_cases import judge_units

pytestmark = pytest.mark.gpu

CONFIG1 = dict(B=1, H=8, HKV=2, T=2048, bits=4, group=64)
CONFIG2 = dict(B=32, H=32, HKV=8, T=8192, bits=4, group=64)
CONFIG3 = dict(B=16, H=32, HKV=8, T=16384)
CONFIG4 = dict(B=64, H=28, HKV=4, T=32768, bits=8, group=64)
CONFIG5 = dict(B=1, H=64, HKV=8, T=131072, bits=4, group=64)
DH = 128


@pytest.fixture(scope="module")
def kva(native):
    from kernelverify_b200.pack import kv_attention
    return kv_attention


def _raw(shape, seed, outliers=0.0):
    """N(0,1) fp32 on the device, a fraction `outliers` of entries x20, as fp16."""
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    raw = torch.randn(shape, dtype=torch.float32, device="cuda", generator=g)
    if outliers:
        hit = torch.rand(shape, device="cuda", generator=g) < outliers
        raw = torch.where(hit, raw * 20.0, raw)
    return raw.half()


def _inputs(b, h, hkv, seed):
    import torch
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    q = torch.randn((b, h, DH), generator=g, device="cuda").half()
    nk = torch.randn((b, hkv, DH), generator=g, device="cuda").half()
    nv = torch.randn((b, hkv, DH), generator=g, device="cuda").half()
    return q, nk, nv


def _payloads(units, q, k_raw, v_raw, nk, nv, outs, bits, group, lens=None, tag=""):
    """Host copies of each judged unit's rows (b, hk) -- q rows hk*r..(hk+1)*r
    -- with the same rows of every candidate output in `outs` ({tag: out}, or
    one output tensor)."""
    r = q.shape[1] // k_raw.shape[1]
    if not isinstance(outs, dict):
        outs = {"": outs}
    res = []
    for b, hk in units:
        t = int(lens[b]) if lens is not None else k_raw.shape[2]
        res.append((f"{tag}b{b}/hk{hk}/T{t}",
                    q[b, hk * r:(hk + 1) * r].cpu().numpy(),
                    k_raw[b, hk, :t].cpu().numpy(), v_raw[b, hk, :t].cpu().numpy(),
                    nk[b, hk].cpu().numpy(), nv[b, hk].cpu().numpy(), bits, group,
                    {k: o[b, hk * r:(hk + 1) * r].cpu().numpy() for k, o in outs.items()}))
    return res


def _assert_all(verdicts):
    bad = [f"{label}: {v}" for label, v in verdicts if not v.ok]
    worst = max((v.err / v.tol if v.tol else 0.0) for _, v in verdicts)
    print(f"{len(verdicts)} units judged, worst err/tol {worst:.3f}")
    assert not bad, "\n".join(bad)


def _run(kva, cfg, seed, outliers=0.0, lens=None):
    """Raw caches, their packed artefacts and the decoded output of one config."""
    import torch
    b, h, hkv, t = cfg["B"], cfg["H"], cfg["HKV"], cfg["T"]
    q, nk, nv = _inputs(b, h, hkv, seed)
    k_raw = _raw((b, hkv, t, DH), 2 * seed + 1, outliers)
    v_raw = _raw((b, hkv, t, DH), 2 * seed + 2, outliers)
    k_art = kva.quantize(k_raw, cfg["bits"], cfg["group"])
    v_art = kva.quantize(v_raw, cfg["bits"], cfg["group"])
    sl = torch.from_numpy(np.asarray(lens, dtype=np.int32)).cuda() if lens is not None else None
    out = kva.decode(q, *k_art, *v_art, nk, nv, bits=cfg["bits"], seq_lens=sl)
    torch.cuda.synchronize()
    return q, nk, nv, k_raw, v_raw, k_art, v_art, out


def test_config1_whole(kva):
    """Config 1: one sequence, 8 query heads on 2 cache heads, T=2048, 4-bit."""
    cfg = CONFIG1
    q, nk, nv, k_raw, v_raw, _, _, out = _run(kva, cfg, seed=11)
    units = [(0, hk) for hk in range(cfg["HKV"])]
    _assert_all(judge_units(_payloads(units, q, k_raw, v_raw, nk, nv, out, 4, 64)))


def test_config2_sampled_sequences(kva):
    """Config 2 (B=32, 32/8 heads, T=8192, 4-bit g64) at its own split plan:
    four sequences, every cache head of each."""
    cfg = CONFIG2
    q, nk, nv, k_raw, v_raw, k_art, v_art, out = _run(kva, cfg, seed=21)
    a = kva._args(q, *k_art, *v_art, nk, nv, bits=4)
    print(f"config 2: {kva.KERNEL_NAMES[kva._native.lib().kvq_plan_kernel(a)]} kernel, "
          f"{kva._native.lib().kvq_split_count(a)} splits")
    units = [(b, hk) for b in (0, 11, 22, 31) for hk in range(cfg["HKV"])]
    _assert_all(judge_units(_payloads(units, q, k_raw, v_raw, nk, nv, out, 4, 64)))


@pytest.mark.parametrize("bits", [2, 3, 4, 6, 8])
def test_config3_sweep(kva, bits):
    """Config 3 (B=16, 32/8 heads, T=16384, 1 % of entries x20): every group
    at this width, two units each (first and last sequence and cache head)."""
    import torch
    cfg = CONFIG3
    b, h, hkv, t = cfg["B"], cfg["H"], cfg["HKV"], cfg["T"]
    q, nk, nv = _inputs(b, h, hkv, 31)
    k_raw = _raw((b, hkv, t, DH), 61, 0.01)
    v_raw = _raw((b, hkv, t, DH), 62, 0.01)
    payloads = []
    for group in (32, 64, 128):
        k_art = kva.quantize(k_raw, bits, group)
        v_art = kva.quantize(v_raw, bits, group)
        out = kva.decode(q, *k_art, *v_art, nk, nv, bits=bits)
        torch.cuda.synchronize()
        payloads += _payloads([(0, 0), (b - 1, hkv - 1)], q, k_raw, v_raw, nk, nv, out, bits,
                              group, tag=f"g{group} ")
        del k_art, v_art
    _assert_all(judge_units(payloads))


def test_config4_ragged(kva):
    """Config 4 (B=64, 28/4 heads, 8-bit g64, lengths seeded U[256, 32768]):
    the shortest and the longest sequence and two others."""
    import importlib.util
    from pathlib import Path
    spec = importlib.util.spec_from_file_location("bench", Path(__file__).resolve().parents[1] / "bench.py")
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    lens = bench.ragged_lengths(CONFIG4["B"], 256, 32768, 0)
    assert int(lens.sum()) == 1_077_211 and int(lens.min()) == 345 and int(lens.max()) == 32678
    cfg = dict(CONFIG4, T=-(-int(lens.max()) // 64) * 64)
    q, nk, nv, k_raw, v_raw, _, _, out = _run(kva, cfg, seed=41, lens=lens)
    lo, hi = int(np.argmin(lens)), int(np.argmax(lens))
    units = [(lo, 0), (hi, 3), (17, 1), (40, 2)]
    _assert_all(judge_units(_payloads(units, q, k_raw, v_raw, nk, nv, out, 8, 64, lens=lens)))


def test_config5_long_context(kva):
    """Config 5 (B=1, 64/8 heads, T=131072, 4-bit g64) on one GPU, both
    through kvq_decode and through the sequence-split decoder the bench runs
    at N=1: the first and the last cache head (8 query heads each; the oracle
    holds one cache head tiled 8x at a time)."""
    import torch
    from kernelverify_b200.pack.tsplit import SequenceSplitDecoder
    cfg = CONFIG5
    q, nk, nv, k_raw, v_raw, k_art, v_art, out = _run(kva, cfg, seed=51)
    dec = SequenceSplitDecoder(1, cfg["H"], DH, torch.device("cuda"), group=None)
    out_split = torch.empty_like(out)
    dec.step(q, *k_art, *v_art, nk, nv, bits=4, t_local=cfg["T"], out=out_split)
    torch.cuda.synchronize()
    units = [(0, 0), (0, cfg["HKV"] - 1)]
    payloads = _payloads(units, q, k_raw, v_raw, nk, nv,
                         {"decode ": out, "tsplit ": out_split}, 4, 64)
    _assert_all(judge_units(payloads, processes=2))
