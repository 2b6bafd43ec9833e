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
