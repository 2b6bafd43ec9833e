"""Test helpers: pack a numpy case with the oracle's quantizer, upload it, run
it through the CUDA door, and judge it with the oracle. Test infrastructure."""

from __future__ import annotations

import numpy as np

from oracle import kv, quant


def to_dev(a, device="cuda"):
    import torch
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(np.ascontiguousarray(a)).to(device)


def pack(cache, bits, group=64):
    """(words, scales, biases) numpy for an (H, T, DH) or (B, H, T, DH) cache."""
    if cache.ndim == 4:
        parts = [quant.quantize_cache(c, bits, group) for c in cache]
        return tuple(np.stack([p[i] for p in parts]) for i in range(3))
    return quant.quantize_cache(cache, bits, group)


def run_decode(q, k_cache, v_cache, new_k, new_v, bits, group=64, *, t_cached=None,
               seq_lens=None, k_art=None, v_art=None):
    """CUDA output (numpy) for raw numpy caches packed by the oracle quantizer."""
    import torch
    from kernelverify_b200.pack import kv_attention as kva

    kw, ks, kb = k_art if k_art is not None else pack(k_cache, bits, group)
    vw, vs, vb = v_art if v_art is not None else pack(v_cache, bits, group)
    args = [to_dev(x) for x in (q, kw, ks, kb, vw, vs, vb, new_k, new_v)]
    sl = to_dev(np.asarray(seq_lens, dtype=np.int32)) if seq_lens is not None else None
    out = kva.decode(*args, bits=bits, t_cached=t_cached, seq_lens=sl)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def judge_gqa(q, k_cache, v_cache, new_k, new_v, bits, out, group=64, dtype="float16"):
    """Verdict of a shared-cache (possibly GQA) case against the oracle."""
    inputs = kv.gqa_tiled_inputs(q, k_cache, v_cache, new_k, new_v, bits, group)
    return kv.verify_output(inputs, out, dtype)


def judge_per_sequence(q, k_caches, v_caches, new_k, new_v, bits, out, lens=None, group=64,
                       dtype="float16", rows=None):
    """Each sequence judged as its own B=1 case (rows are independent; a
    per-case max|ref| makes this stricter than one whole-batch tolerance)."""
    verdicts = []
    for b in (range(q.shape[0]) if rows is None else rows):
        t = k_caches.shape[2] if lens is None else int(lens[b])
        verdicts.append(judge_gqa(q[b:b + 1], k_caches[b, :, :t], v_caches[b, :, :t],
                                  new_k[b:b + 1], new_v[b:b + 1], bits, out[b:b + 1], group,
                                  dtype))
    return verdicts


def judge_unit(payload):
    """Verdicts of one (sequence, cache head) unit from its raw fp16 rows: q
    [r, DH] of the unit's query heads, k/v rows [T, DH], new_k/new_v [DH], and
    one or more candidate outputs [r, DH] ({tag: out}) judged against one
    reference and tolerance. A module-level function so a spawned process
    pool can run it (the oracle is CPU numpy; the judged units are
    independent)."""
    label, q, k_rows, v_rows, new_k, new_v, bits, group, outs = payload
    inputs = kv.gqa_tiled_inputs(q[None], k_rows[None], v_rows[None], new_k[None, None],
                                 new_v[None, None], bits, group)
    ref, tol = kv.reference_and_tolerance(inputs)
    return [(f"{tag}{label}", kv.judge(out[None], ref, tol)) for tag, out in outs.items()]


def judge_units(payloads, processes: int | None = None):
    """[(label, Verdict)] of every unit and candidate, judged in a spawned
    pool (never forked: the caller has a CUDA context)."""
    import multiprocessing as mp
    import os
    n = max(1, min(len(payloads), processes or os.cpu_count() or 1))
    if n == 1:
        res = [judge_unit(p) for p in payloads]
    else:
        with mp.get_context("spawn").Pool(n) as pool:
            res = pool.map(judge_unit, payloads, chunksize=1)
    return [v for unit in res for v in unit]
