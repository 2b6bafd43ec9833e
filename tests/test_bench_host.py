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
    assert bench.parse_args([]).config == 2
