"""Decode steps in flight on several streams at once: without a caller's
workspace each stream gets its own default scratch, so two steps launched
back to back on two streams (no synchronisation between them) return exactly
what each returns alone."""

from __future__ import annotations

import pytest

from oracle import cases
from tests.kvq_cases import pack, to_dev

pytestmark = pytest.mark.gpu


def test_default_workspaces_are_per_stream(native):
    import torch
    from kernelverify_b200.pack import kv_attention as kva
    dev = torch.device("cuda", torch.cuda.current_device())
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    b1, _ = kva._workspace(dev, 1 << 20, None, s1)
    b2, _ = kva._workspace(dev, 1 << 20, None, s2)
    again, _ = kva._workspace(dev, 1 << 20, None, s1)
    assert b1.data_ptr() != b2.data_ptr() and again.data_ptr() == b1.data_ptr()


def test_concurrent_steps_on_two_streams_match_their_solo_runs(native):
    import torch
    from kernelverify_b200.pack import kv_attention as kva
    steps = []
    for seed, (b, h, t) in ((1, (4, 32, 4096)), (2, (2, 16, 9000))):
        q, kc, vc, nk, nv = cases.make_case(b, h, t, 128, seed=seed)
        hkv = h // 4
        kc, vc, nk, nv = kc[:hkv], vc[:hkv], nk[:, :hkv], nv[:, :hkv]
        steps.append([to_dev(x) for x in (q, *pack(kc, 4), *pack(vc, 4), nk, nv)])
    solo = []
    for args in steps:
        solo.append(kva.decode(*args, bits=4).clone())
        torch.cuda.synchronize()
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    outs = []
    for _ in range(3):
        for args, s in zip(steps, streams):
            with torch.cuda.stream(s):
                outs.append(kva.decode(*args, bits=4, stream=s))
    torch.cuda.synchronize()
    for i, out in enumerate(outs):
        assert torch.equal(out, solo[i % 2]), i
