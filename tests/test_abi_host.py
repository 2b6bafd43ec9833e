"""The C-ABI library on a machine without a GPU: it loads, exports every
symbol include/kvq_b200.h declares, and rejects bad arguments (or the missing
device) with a status and a message -- no compute call is made."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest

from kernelverify_b200 import _native

HEADER = Path(__file__).resolve().parents[1] / "include" / "kvq_b200.h"


@pytest.fixture(scope="module")
def lib():
    from kernelverify_b200 import build
    build.build()
    return _native.lib()


def declared_functions() -> set:
    text = HEADER.read_text()
    return set(re.findall(r"^\s*(?:const\s+)?\w+\**\s+\**(kvq_\w+)\s*\(", text, re.M))


def test_header_and_binding_agree():
    assert declared_functions() == set(_native.EXPORTS)


def _prototypes() -> dict:
    """name -> (return type, [parameter types]) of every prototype in the
    header, comments stripped."""
    text = re.sub(r"/\*.*?\*/", "", HEADER.read_text(), flags=re.S)
    protos = {}
    for ret, name, params in re.findall(r"((?:const\s+)?\w+\s*\**)\s*(kvq_\w+)\s*\(([^)]*)\)\s*;",
                                        text):
        params = " ".join(params.split())
        plist = [] if params in ("", "void") else [p.strip() for p in params.split(",")]
        protos[name] = (" ".join(ret.split()), plist)
    return protos


def _ctype_of(decl: str):
    """The ctypes type a C parameter or return declaration binds to."""
    decl = " ".join(decl.replace("*", " * ").split())
    if decl.count("*") == 2:
        return ctypes.POINTER(ctypes.c_void_p)
    if decl == "uint32_t * status" or decl.endswith("uint32_t * status"):
        return ctypes.POINTER(ctypes.c_uint32)
    if decl.startswith("const char *"):
        return ctypes.c_char_p
    if "kvq_args" in decl:
        return ctypes.POINTER(_native.KvqArgs)
    if "*" in decl:
        return ctypes.c_void_p
    base = decl.replace("const ", "").split()[0]
    return {"int": ctypes.c_int, "uint32_t": ctypes.c_uint32, "uint64_t": ctypes.c_uint64,
            "size_t": ctypes.c_size_t}[base]


def test_binding_signatures_match_the_header_prototypes(lib):
    """Every ctypes declaration has the header prototype's arity and types, so
    a binding can never pass an argument the C side reads as something else."""
    for name, (ret, params) in _prototypes().items():
        fn = getattr(lib, name)
        assert fn.restype == _ctype_of(ret), (name, ret, fn.restype)
        want = [_ctype_of(p) for p in params]
        assert len(fn.argtypes) == len(want), (name, len(fn.argtypes), len(want))
        for i, (got, exp) in enumerate(zip(fn.argtypes, want)):
            if "*" in params[i] and got is ctypes.c_void_p:
                continue          # any pointer may travel as a plain address
            assert got == exp, (name, i, params[i], got, exp)


def test_library_exports_every_declared_symbol(lib):
    handle = ctypes.CDLL(str(_native.LIB_PATH))
    for name in declared_functions():
        assert hasattr(handle, name), name
    assert lib.kvq_abi_version() == _native.ABI_VERSION


def test_supports_reports_the_instantiated_formats(lib):
    for dh in (64, 128):
        for bits in (2, 3, 4, 6, 8):
            for g in (32, 64, 128):
                for dt in (0, 1):
                    assert lib.kvq_supports(dh, bits, g, dt) == (dh % g == 0)
    assert not lib.kvq_supports(96, 4, 32, 0)
    assert not lib.kvq_supports(128, 5, 64, 0)
    assert not lib.kvq_supports(128, 4, 64, 2)


def _args(**over):
    a = _native.KvqArgs()
    for name in ("q", "k_wq", "k_scales", "k_biases", "v_wq", "v_scales", "v_biases",
                 "new_k", "new_v"):
        setattr(a, name, 4096)
    a.b_rows, a.n_heads, a.n_kv_heads = 1, 8, 2
    a.t_cached, a.t_stride, a.head_dim = 100, 128, 128
    a.bits, a.group_size, a.dtype, a.has_new_entry = 4, 64, 0, 1
    a.t_begin, a.t_end = 0, _native.KVQ_T_END_ALL
    for k, v in over.items():
        setattr(a, k, v)
    return a


@pytest.mark.parametrize("over,needle", [
    (dict(head_dim=96), b"head_dim"),
    (dict(bits=5), b"bits"),
    (dict(group_size=48), b"group_size"),
    (dict(dtype=3), b"dtype"),
    (dict(n_heads=7), b"multiple"),
    (dict(t_cached=200), b"t_stride"),
    (dict(q=0), b"NULL"),
    (dict(q=4097), b"aligned"),
    (dict(t_begin=10, t_end=5), b"t_begin"),
])
def test_invalid_arguments_return_a_status_and_message(lib, over, needle):
    a = _args(**over)
    status = lib.kvq_decode(ctypes.byref(a), 8192, None, 0, None)
    assert status == _native.KVQ_ERR_INVALID
    assert needle in lib.kvq_last_error()


def test_workspace_is_sized_and_checked(lib):
    a = _args()
    need = lib.kvq_workspace_bytes(ctypes.byref(a))
    assert need > 0 and need % 256 == 0
    status = lib.kvq_decode(ctypes.byref(a), 8192, None, 0, None)
    assert status == _native.KVQ_ERR_INVALID and b"workspace" in lib.kvq_last_error()


def test_missing_device_is_unsupported_not_a_crash(lib):
    """Valid arguments on a machine with no GPU: the call reports UNSUPPORTED."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    a = _args()
    need = lib.kvq_workspace_bytes(ctypes.byref(a))
    status = lib.kvq_decode(ctypes.byref(a), 8192, 1 << 20, need, None)
    assert status == _native.KVQ_ERR_UNSUPPORTED
    assert lib.kvq_last_error()


@pytest.mark.parametrize("over,needle", [
    (dict(position=6), b"runs past t_stride"),
    (dict(b_rows=2, batch_stride=0), b"one cache per sequence"),
    (dict(b_rows=2, batch_stride=8), b"overlaps"),
    (dict(bits=5), b"bits"),
    (dict(w=0), b"NULL"),
])
def test_cache_append_rejects_bad_destinations(lib, over, needle):
    """Host checks of kvq_cache_append, before any device work: a host
    position past the buffer, a shared cache under several sequences, a batch
    stride that overlaps, a bad width, a NULL pointer."""
    a = dict(w=4096, b_rows=1, n_kv_heads=2, n_new=3, head_dim=64, bits=4, group=64, dtype=0,
             positions=None, position=0, t_stride=8, batch_stride=16, wq=8192, scales=8192,
             biases=8192)
    a.update(over)
    status = lib.kvq_cache_append(a["w"], a["b_rows"], a["n_kv_heads"], a["n_new"],
                                  a["head_dim"], a["bits"], a["group"], a["dtype"],
                                  a["positions"], a["position"], a["t_stride"],
                                  a["batch_stride"], a["wq"], a["scales"], a["biases"], None)
    assert status == _native.KVQ_ERR_INVALID
    assert needle in lib.kvq_last_error()


def test_plan_kernel_names_the_kernel_without_a_device(lib):
    """Aligned fp16 DH-128 geometry plans the tensor-core kernels at every
    width and group; a t_stride that is not a multiple of 8, head_dim 64, fp32
    or more than 8 query heads per cache head the CUDA-core one; invalid
    arguments a negative status."""
    TC, CC = _native.KVQ_KERNEL_TENSOR_CORE, _native.KVQ_KERNEL_CUDA_CORE
    for bits in (2, 3, 4, 6, 8):
        for group in (32, 64, 128):
            assert lib.kvq_plan_kernel(ctypes.byref(_args(bits=bits, group_size=group))) == TC
    assert lib.kvq_plan_kernel(ctypes.byref(_args(head_dim=64))) == CC
    assert lib.kvq_plan_kernel(ctypes.byref(_args(dtype=1))) == CC
    assert lib.kvq_plan_kernel(ctypes.byref(_args(t_stride=130))) == CC
    assert lib.kvq_plan_kernel(ctypes.byref(_args(n_heads=32, n_kv_heads=2))) == CC
    assert lib.kvq_plan_kernel(ctypes.byref(_args(bits=5))) == _native.KVQ_ERR_INVALID


def test_tsplit_region_layout_and_format_gate_without_a_device(lib):
    """The one-kernel sequence split: its region is the 256-byte control
    block, a per-row u32 array (step counts), a partial store of
    min(64 rows, max(16384, 2 rows))
    rows and two parities x world records of rows, each row head_dim + 2
    tagged 8-byte words, each block 256-aligned; it serves the 4-bit group-64
    tensor-core format only, and refuses other formats and bad ranks before
    any device work."""
    def a256(x):
        return (x + 255) // 256 * 256
    for rows, world in [(64, 8), (64, 1), (3, 2), (2048, 4), (9000, 2)]:
        part = min(64 * rows, max(16384, 2 * rows))
        want = 256 + a256(4 * rows) + a256(8 * 130 * part) + 2 * world * a256(8 * 130 * rows)
        assert lib.kvq_tsplit_region_bytes(rows, 128, world) == want
    assert lib.kvq_tsplit_region_bytes(64, 128, 0) == 0
    assert lib.kvq_tsplit_region_bytes(64, 128, 9) == 0
    assert lib.kvq_tsplit_region_bytes(64, 64, 1) == 0
    assert lib.kvq_tsplit_supported(ctypes.byref(_args())) == 1
    assert lib.kvq_tsplit_supported(ctypes.byref(_args(n_heads=64, n_kv_heads=8))) == 1
    # config 5 on one rank without a device: 8 units planned for two CTAs on
    # each of the fallback 148 SMs -> 37 splits
    c5 = _args(n_heads=64, n_kv_heads=8, t_cached=131072, t_stride=131072)
    assert lib.kvq_tsplit_split_count(ctypes.byref(c5)) == 37
    assert lib.kvq_tsplit_split_count(ctypes.byref(_args(bits=8))) == 0
    for over in (dict(bits=8), dict(group_size=32), dict(head_dim=64), dict(dtype=1),
                 dict(t_stride=130), dict(bits=5)):
        assert lib.kvq_tsplit_supported(ctypes.byref(_args(**over))) == 0, over
    a = _args()
    regions = (ctypes.c_void_p * 1)(1 << 20)
    nbytes = lib.kvq_tsplit_region_bytes(8, 128, 1)
    st = lib.kvq_tsplit_decode(ctypes.byref(_args(bits=8)), regions, nbytes, 1, 0, 8192, 0, None)
    assert st == _native.KVQ_ERR_UNSUPPORTED and b"4-bit group-64" in lib.kvq_last_error()
    st = lib.kvq_tsplit_decode(ctypes.byref(a), regions, nbytes, 2, 2, 8192, 0, None)
    assert st == _native.KVQ_ERR_INVALID and b"rank" in lib.kvq_last_error()
    st = lib.kvq_tsplit_decode(ctypes.byref(a), regions, nbytes - 256, 1, 0, 8192, 0, None)
    assert st == _native.KVQ_ERR_INVALID and b"kvq_tsplit_region_bytes" in lib.kvq_last_error()
