"""The framework door's argument checks on a machine without a GPU: every
tensor the library reaches through its raw address alone is checked for
shape, dtype and contiguity before an address is taken, so a wrong buffer is
a ValueError on the host, never a kernel indexing memory the tensor does not
own. No device call is made."""

from __future__ import annotations

import pytest

torch = pytest.importorskip("torch")

from kernelverify_b200.pack import kv_attention as kva  # noqa: E402


def f32(*shape):
    return torch.zeros(shape, dtype=torch.float32)


@pytest.mark.parametrize("over,needle", [
    (dict(part_o=f32(2, 1, 4, 64, 1)), "part_o must be"),
    (dict(part_m=f32(2, 1, 5)), "part_m has shape"),
    (dict(part_l=torch.zeros((2, 1, 4), dtype=torch.float16)), "part_l is"),
    (dict(part_m=f32(2, 1, 8)[:, :, ::2]), "part_m must be contiguous"),
    (dict(out=f32(1, 4, 32)), "out has shape"),
    (dict(out_dtype=torch.bfloat16), "not float16 or float32"),
    (dict(), "CUDA tensor"),
])
def test_lse_merge_checks_every_buffer(over, needle):
    args = dict(part_o=f32(2, 1, 4, 64), part_m=f32(2, 1, 4), part_l=f32(2, 1, 4),
                out_dtype=torch.float32, out=None)
    args.update(over)
    with pytest.raises(ValueError, match=needle):
        kva.lse_merge(args["part_o"], args["part_m"], args["part_l"], args["out_dtype"],
                      out=args["out"])


def test_lse_merge_records_checks_out():
    rows, dh = 4, 64
    records = f32(3, kva.record_floats(rows, dh))
    with pytest.raises(ValueError, match="out has shape"):
        kva.lse_merge_records(records, 1, rows, dh, torch.float16,
                              out=torch.zeros((1, rows, dh + 1), dtype=torch.float16))
    with pytest.raises(ValueError, match="out is"):
        kva.lse_merge_records(records, 1, rows, dh, torch.float16, out=f32(1, rows, dh))
    with pytest.raises(ValueError, match="records must be"):
        kva.lse_merge_records(records[:, :-1], 1, rows, dh, torch.float16)


@pytest.mark.parametrize("over,needle", [
    (dict(words=torch.zeros((2, 16), dtype=torch.int16)), "int32/uint32"),
    (dict(words=torch.zeros((2, 13), dtype=torch.int32), bits=3), "not a packed artefact"),
    (dict(scales=torch.zeros((2, 3), dtype=torch.float16)), "groups per row"),
    (dict(biases=torch.zeros((2, 2), dtype=torch.float32)), "biases is"),
    (dict(bits=5), "not a packed artefact"),
])
def test_dequant_checks_the_artefact(over, needle):
    args = dict(words=torch.zeros((2, 16), dtype=torch.int32),
                scales=torch.zeros((2, 2), dtype=torch.float16),
                biases=torch.zeros((2, 2), dtype=torch.float16), bits=4)
    args.update(over)
    with pytest.raises(ValueError, match=needle):
        kva.dequant(args["words"], args["scales"], args["biases"], args["bits"])


def test_dequant_of_a_host_tensor_is_refused():
    w = torch.zeros((2, 16), dtype=torch.int32)
    s = torch.zeros((2, 2), dtype=torch.float16)
    with pytest.raises(ValueError, match="CUDA"):
        kva.dequant(w, s, s.clone(), 4)


def test_launch_config_is_the_cuda_core_plan():
    """One split of 256 positions below a wave; more splits as T grows; the
    grid's y covers the cache heads x head tiles."""
    (splits, y, z), block = kva.launch_config(1, 8, 2, 256)
    assert (splits, y, z) == (1, 2, 1) and block == (256, 1, 1)
    (splits, y, z), _ = kva.launch_config(32, 32, 8, 8192)
    assert splits > 1 and y == 8 and z == 32
