"""bench.py's host arithmetic on the CPU: the algorithmic bytes a step reads
for every BASELINE config, config 4's seeded lengths (the same draw as the
oracle's case maker), and the variant selection of the sweep."""

from __future__ import annotations

import bench
from oracle import cases


def test_kv_bytes_per_config():
    c2 = bench.CONFIG2
    # 2 (K, V) x 8 heads x 32 x 8192 rows x (64 code bytes + 2 groups x 4 bytes)
    assert bench.kv_bytes(c2) == 2 * 8 * 32 * 8192 * (64 + 8)
    c3 = dict(bench.CONFIG3, bits=3, group=32)
    assert bench.kv_bytes(c3) == 2 * 8 * 16 * 16384 * (48 + 16)
    lens = bench.ragged_lengths(*((bench.CONFIG4["B"],) + bench.CONFIG4["lens"]))
    assert int(lens.sum()) == 1_077_211 and lens.min() == 345 and lens.max() == 32678
    assert bench.kv_bytes(bench.CONFIG4, int(lens.sum())) == 2 * 4 * 1_077_211 * (128 + 8)


def test_config4_lengths_are_the_oracle_draw():
    lo, hi, seed = bench.CONFIG4["lens"]
    assert (bench.ragged_lengths(64, lo, hi, seed) == cases.ragged_lengths(64, lo, hi, seed)).all()


def test_sweep_arguments():
    a = bench.parse_args(["--config", "3", "--bits", "6", "--group", "32"])
    assert (a.config, a.bits, a.group) == (3, 6, 32)
    assert bench.SWEEP_BITS == (2, 3, 4, 6, 8) and bench.SWEEP_GROUPS == (32, 64, 128)
    # the default is the metric's 1/2/4/8-GPU configuration, the sequence split
    assert bench.parse_args([]).config == 5


def test_cpu_shards_and_parity_unpack():
    """The CPU baseline's shard of a unit, and the bench's library-independent
    code unpack against the oracle's packer (every width, straddling codes)."""
    import numpy as np
    import torch
    from oracle import quant
    assert bench.cpu_shard_positions(bench.CONFIG5) == 8192
    assert bench.cpu_shard_positions(bench.CONFIG2) == 512
    rng = np.random.default_rng(3)
    for bits in (2, 3, 4, 6, 8):
        codes = rng.integers(0, 1 << bits, size=(5, 128))
        words = quant.pack_codes(codes, bits)
        got = bench._unpack_codes(torch.from_numpy(words.view(np.int32)), bits, 128)
        assert np.array_equal(got.numpy().astype(np.int64), codes)


def test_parity_unit_matches_the_oracle_reference():
    """The bench's fp64 device reference, run on the CPU here, equals the
    oracle's fp64 reference on the same packed rows."""
    import numpy as np
    import torch
    from oracle import cases, kv, quant
    q, kc, vc, nk, nv = cases.make_case(1, 4, 300, 128, seed=5)
    kc, vc, nk, nv = kc[:1], vc[:1], nk[:, :1], nv[:, :1]
    kw, ks, kb = quant.quantize_cache(kc, 4)
    vw, vs, vb = quant.quantize_cache(vc, 4)
    art = tuple(torch.from_numpy(np.ascontiguousarray(a.view(np.int32) if a.dtype == np.uint32 else a))[0]
                for a in (kw, ks, kb, vw, vs, vb))
    ref = kv.kv_reference(kv.gqa_tiled_inputs(q, kc, vc, nk, nv, 4))[0]
    res = bench.parity_unit(torch.from_numpy(ref), torch.from_numpy(q[0]), torch.from_numpy(nk[0, 0]),
                            torch.from_numpy(nv[0, 0]), art, 4)
    assert res["ok"] and res["max_abs"] < 1e-12, res
