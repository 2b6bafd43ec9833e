"""ctypes binding of the C ABI in include/kvq_b200.h.

The library is the in-tree kernelverify_b200/_lib/libkvq_b200.so (built by
`python -m kernelverify_b200.build`). There is no fallback: when the library
is missing or will not load, every entry point raises `NativeUnavailable`.
"""

from __future__ import annotations

import ctypes
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libkvq_b200.so"
ABI_VERSION = 1

KVQ_OK, KVQ_ERR_INVALID, KVQ_ERR_LAUNCH, KVQ_ERR_UNSUPPORTED = 0, -1, -2, -3
KVQ_F16, KVQ_F32 = 0, 1
KVQ_T_END_ALL = 0xFFFFFFFF
KVQ_NOALLOC_SCRATCH_BYTES = 16 << 20
KVQ_KERNEL_CUDA_CORE, KVQ_KERNEL_TENSOR_CORE, KVQ_KERNEL_TCGEN05 = 0, 1, 2
KVQ_PEER_MAX_RANKS = 8
KVQ_PEER_HANDLE_BYTES = 64

# Every symbol include/kvq_b200.h declares.
EXPORTS = ("kvq_workspace_bytes", "kvq_decode", "kvq_decode_partial", "kvq_split_count",
           "kvq_decode_splits", "kvq_lse_merge", "kvq_lse_merge_records", "kvq_decode_noalloc",
           "kvq_dequant", "kvq_quantize", "kvq_cache_append", "kvq_supports", "kvq_plan_kernel", "kvq_last_error", "kvq_abi_version",
           "kvq_peer_region_bytes", "kvq_peer_record_offset", "kvq_peer_alloc", "kvq_peer_open",
           "kvq_peer_close", "kvq_peer_free", "kvq_peer_merge", "kvq_peer_status",
           "kvq_peer_last_error", "kvq_tsplit_region_bytes", "kvq_tsplit_supported", "kvq_tsplit_split_count",
           "kvq_tsplit_decode", "kvq_stage_copy")


class NativeUnavailable(RuntimeError):
    """The CUDA library is absent or unloadable; the CUDA path cannot run."""


class KvqError(RuntimeError):
    """A kvq entry point returned a failure status."""

    def __init__(self, status: int, message: str):
        super().__init__(f"kvq status {status}: {message}")
        self.status = status
        self.message = message


class KvqArgs(ctypes.Structure):
    _fields_ = [
        ("q", ctypes.c_void_p), ("k_wq", ctypes.c_void_p), ("k_scales", ctypes.c_void_p),
        ("k_biases", ctypes.c_void_p), ("v_wq", ctypes.c_void_p), ("v_scales", ctypes.c_void_p),
        ("v_biases", ctypes.c_void_p), ("new_k", ctypes.c_void_p), ("new_v", ctypes.c_void_p),
        ("seq_lens", ctypes.c_void_p),
        ("b_rows", ctypes.c_uint32), ("n_heads", ctypes.c_uint32), ("n_kv_heads", ctypes.c_uint32),
        ("t_cached", ctypes.c_uint32), ("t_stride", ctypes.c_uint32), ("head_dim", ctypes.c_uint32),
        ("bits", ctypes.c_uint32), ("group_size", ctypes.c_uint32), ("dtype", ctypes.c_uint32),
        ("has_new_entry", ctypes.c_uint32), ("cache_batch_stride", ctypes.c_uint64),
        ("t_begin", ctypes.c_uint32), ("t_end", ctypes.c_uint32),
    ]


_lock = threading.Lock()
_lib = None


def _declare(lib) -> None:
    P, U32, U64, SZ, I = (ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_size_t,
                          ctypes.c_int)
    AP = ctypes.POINTER(KvqArgs)
    sig = {
        "kvq_workspace_bytes": (SZ, [AP]),
        "kvq_decode": (I, [AP, P, P, SZ, P]),
        "kvq_decode_partial": (I, [AP, P, P, P, P, SZ, P]),
        "kvq_split_count": (U32, [AP]),
        "kvq_plan_kernel": (I, [AP]),
        "kvq_decode_splits": (I, [AP, P, P, P, P]),
        "kvq_lse_merge": (I, [P, P, P, U32, U32, U32, U32, P, P]),
        "kvq_lse_merge_records": (I, [P, U32, U32, U32, U32, P, P]),
        "kvq_decode_noalloc": (I, [AP, P, P]),
        "kvq_dequant": (I, [P, P, P, U64, U32, U32, U32, U32, P, P]),
        "kvq_quantize": (I, [P, U64, U32, U32, U32, U32, P, P, P, P]),
        "kvq_cache_append": (I, [P, U32, U32, U32, U32, U32, U32, U32, P, U32, U32, U64, P, P,
                                 P, P]),
        "kvq_supports": (I, [U32, U32, U32, U32]),
        "kvq_last_error": (ctypes.c_char_p, []),
        "kvq_abi_version": (I, []),
        "kvq_peer_region_bytes": (SZ, [U32, U32]),
        "kvq_peer_record_offset": (SZ, [U32, U32, U32]),
        "kvq_peer_alloc": (I, [SZ, ctypes.POINTER(ctypes.c_void_p), P]),
        "kvq_peer_open": (I, [P, ctypes.POINTER(ctypes.c_void_p)]),
        "kvq_peer_close": (I, [P]),
        "kvq_peer_free": (I, [P]),
        "kvq_peer_merge": (I, [P, U32, U32, U32, U32, U32, U32, P, U64, P]),
        "kvq_peer_status": (I, [P, ctypes.POINTER(ctypes.c_uint32), P]),
        "kvq_peer_last_error": (ctypes.c_char_p, []),
        "kvq_tsplit_region_bytes": (SZ, [U32, U32, U32]),
        "kvq_tsplit_supported": (I, [AP]),
        "kvq_tsplit_split_count": (U32, [AP]),
        "kvq_tsplit_decode": (I, [AP, P, SZ, U32, U32, P, U64, P]),
        "kvq_stage_copy": (I, [P, P, SZ, P]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args


def lib():
    """The loaded library (loaded once per process)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise NativeUnavailable(
                    f"{LIB_PATH} is missing; build it with `python -m kernelverify_b200.build`")
            try:
                handle = ctypes.CDLL(str(LIB_PATH))
            except OSError as error:
                raise NativeUnavailable(f"{LIB_PATH} will not load: {error}") from error
            _declare(handle)
            version = handle.kvq_abi_version()
            if version != ABI_VERSION:
                raise NativeUnavailable(f"{LIB_PATH} has ABI {version}, this binding speaks {ABI_VERSION}")
            _lib = handle
    return _lib


def check(status: int) -> None:
    if status != KVQ_OK:
        raise KvqError(status, lib().kvq_last_error().decode(errors="replace"))


def check_peer(status: int) -> None:
    """check() for the kvq_peer_* entries, which keep their own last error."""
    if status != KVQ_OK:
        raise KvqError(status, lib().kvq_peer_last_error().decode(errors="replace"))
