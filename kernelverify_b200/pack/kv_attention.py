"""CUDA build of kernelverify's quantized-KV attention decode pack.

Mirrors the reference pack module (kernelverify/pack/kv_attention.py) name
for name, with the Metal kernel replaced by the sm_100a library behind the C
ABI of include/kvq_b200.h:

* `build(torch)`    -- the framework door (the reference's `build(mx)`,
  kernelverify/pack/kv_attention.py:369-393): a callable taking the nine
  tensor inputs in the reference's order plus the LOGICAL cached length.
* `kernel_spec()`   -- the runner door (kernelverify/pack/kv_attention.py:
  292-352) for `kernelverify_b200.runners.CudaRunner`.
* `quantize_cache`  -- packed artefact triplet of an (H, T, DH) cache, computed
  on the device by the library's bit-exact canonical quantizer
  (kernelverify/pack/kv_attention.py:270-283).
* `require_capacity`, `should_dispatch`, `launch_config`, `SUPPORTED_BITS`,
  `SUPPORTED_DH`, `KERNEL_NAME`, `INPUT_NAMES`, `OUTPUT_NAMES`.

Differences from the Metal kernel, all extensions:
* no capacity bound: T is split into chunks with a log-sum-exp merge, so the
  reference's TCAP = 1024 (kernelverify/pack/kv_attention.py:53-65) is gone;
  `require_capacity` keeps only the physical bound (the logical length must
  fit the buffer it indexes);
* bits 6 and groups 32/128 besides the reference's {2,3,4,8} x 64;
* per-sequence caches ([B, HKV, T_stride, ...]) and ragged lengths besides the
  reference's cache shared by all batch rows;
* T-range shards (`decode_partial`) for sequence-split multi-GPU decode.
"""

from __future__ import annotations

from kernelverify_b200 import _native
from kernelverify_b200._native import KVQ_F16, KVQ_F32, KVQ_T_END_ALL, KvqArgs

KERNEL_NAME = "kv_attn_decode"
SUPPORTED_BITS = (2, 3, 4, 6, 8)
SUPPORTED_DH = (64, 128)
SUPPORTED_GROUPS = (32, 64, 128)
INPUT_NAMES = ["q", "k_wq", "k_scales", "k_biases",
               "v_wq", "v_scales", "v_biases", "new_k", "new_v", "t_cached"]
OUTPUT_NAMES = ["out"]
THREADS_PER_CTA = 256
MAX_T = 0xFFFFFFFE  # positions are uint32 in the ABI


def _torch():
    import torch
    return torch


def _dtype_code(dt) -> int:
    torch = _torch()
    if dt == torch.float16:
        return KVQ_F16
    if dt == torch.float32:
        return KVQ_F32
    raise ValueError(f"kv_attention: dtype {dt} is not float16 or float32")


def require_capacity(t: int, t_stride: int | None = None) -> None:
    """Reject a logical length the call cannot serve, loudly.

    There is no compile-time capacity here (the reference's TCAP check,
    kernelverify/pack/kv_attention.py:242-256, guarded a threadgroup buffer
    this kernel does not have). What remains is the physical bound: the
    logical length indexes the cache buffer, so it may not exceed its rows."""
    if t < 0 or t > MAX_T:
        raise ValueError(f"t={t} is outside the supported range [0, {MAX_T}]")
    if t_stride is not None and t > t_stride:
        raise ValueError(f"t_cached={t} exceeds the cache buffer's {t_stride} rows per head")


def should_dispatch(t: int) -> bool:
    """Every length is served (kernelverify/pack/kv_attention.py:259-267 deferred
    T > 1024 to MLX; nothing is deferred here)."""
    return 0 <= t <= MAX_T


def launch_config(b: int, h: int, n_kv_heads: int | None = None, t: int = 0):
    """(grid, block) of the CUDA-core partial kernel for B=b, H=h at length
    t: grid (T splits, cache heads x head tiles, b), 256 threads.
    Informational only -- the library plans its own launch, and the
    tensor-core kernels (`plan_kernel` names which one runs) size their T
    splits by whole waves of resident CTAs instead."""
    hkv = n_kv_heads or h
    r = h // hkv
    ht = 1 if r == 1 else (4 if r <= 4 else 8)
    tiles = -(-r // ht)
    units = b * hkv * tiles
    chunk = -(-t * units // (148 * 4 * 2))          # ceil: fill ~2 waves of 4 CTAs/SM
    chunk = max(THREADS_PER_CTA, -(-chunk // THREADS_PER_CTA) * THREADS_PER_CTA)
    splits = max(1, -(-t // chunk)) if t else 1
    return (splits, hkv * tiles, b), (THREADS_PER_CTA, 1, 1)


def _check_buffers(device, *entries) -> None:
    """Tensors the library reads or writes through their raw addresses alone,
    as (name, tensor, shape, dtype) entries: each must have exactly this
    shape and dtype and be contiguous (all checked first), then live on
    `device` -- or the kernel would index memory the tensor does not own."""
    for name, ten, shape, dtype in entries:
        if tuple(ten.shape) != tuple(shape):
            raise ValueError(f"{name} has shape {tuple(ten.shape)}, expected {tuple(shape)}")
        if ten.dtype != dtype:
            raise ValueError(f"{name} is {ten.dtype}, expected {dtype}")
        if not ten.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
    torch = _torch()
    device = torch.device(device)
    if device.type == "cuda" and device.index is None and torch.cuda.is_available():
        device = torch.device("cuda", torch.cuda.current_device())
    for name, ten, _, _ in entries:
        if not ten.is_cuda or ten.device != device:
            raise ValueError(f"{name} must be a CUDA tensor on {device}")


def _check_words(name, ten) -> None:
    torch = _torch()
    if ten.dtype not in (torch.int32, torch.uint32):
        raise ValueError(f"{name}: packed words must be int32/uint32 tensors, got {ten.dtype}")


def _args(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *, bits,
          t_cached=None, seq_lens=None, t_begin=0, t_end=None, has_new_entry=True) -> KvqArgs:
    """Validate shapes and build the C argument block."""
    if q.dim() != 3:
        raise ValueError(f"q must be [B, H, DH], got {tuple(q.shape)}")
    b, h, dh = q.shape
    if k_wq.dim() == 3:
        per_seq, (hkv, t_stride, words) = False, k_wq.shape
    elif k_wq.dim() == 4:
        per_seq = True
        bk, hkv, t_stride, words = k_wq.shape
        if bk != b:
            raise ValueError(f"per-sequence cache has {bk} rows, q has {b}")
    else:
        raise ValueError(f"k_wq must be [HKV, T, W] or [B, HKV, T, W], got {tuple(k_wq.shape)}")
    if dh not in SUPPORTED_DH:
        raise ValueError(f"head_dim {dh} not in {SUPPORTED_DH}")
    if bits not in SUPPORTED_BITS:
        raise ValueError(f"bits {bits} not in {SUPPORTED_BITS}")
    if words * 32 != dh * bits:
        raise ValueError(f"k_wq rows hold {words} words; {dh} codes of {bits} bits need {dh * bits // 32}")
    groups = k_scales.shape[-1]
    if groups == 0 or dh % groups:
        raise ValueError(f"scales carry {groups} groups per row, which does not divide {dh}")
    group = dh // groups
    if h % hkv:
        raise ValueError(f"{h} query heads do not divide into {hkv} cache heads")
    for name, ten, shape in (("k_wq", k_wq, tuple(k_wq.shape)), ("v_wq", v_wq, tuple(k_wq.shape)),
                             ("k_scales", k_scales, tuple(k_wq.shape[:-1]) + (groups,)),
                             ("k_biases", k_biases, tuple(k_wq.shape[:-1]) + (groups,)),
                             ("v_scales", v_scales, tuple(k_wq.shape[:-1]) + (groups,)),
                             ("v_biases", v_biases, tuple(k_wq.shape[:-1]) + (groups,)),
                             ("new_k", new_k, (b, hkv, dh)), ("new_v", new_v, (b, hkv, dh))):
        if tuple(ten.shape) != shape:
            raise ValueError(f"{name} has shape {tuple(ten.shape)}, expected {shape}")
        if not ten.is_contiguous():
            raise ValueError(f"{name} must be contiguous")
        if not ten.is_cuda or ten.device != q.device:
            raise ValueError(f"{name} must be a CUDA tensor on {q.device}")
    torch = _torch()
    code = _dtype_code(q.dtype)
    for name, ten in (("new_k", new_k), ("new_v", new_v), ("k_scales", k_scales),
                      ("k_biases", k_biases), ("v_scales", v_scales), ("v_biases", v_biases)):
        if ten.dtype != q.dtype:
            raise ValueError(f"{name} is {ten.dtype}; every float input must be {q.dtype}")
    if k_wq.dtype not in (torch.int32, torch.uint32) or v_wq.dtype != k_wq.dtype:
        raise ValueError("packed words must be int32/uint32 tensors")
    if not q.is_contiguous():
        raise ValueError("q must be contiguous")
    if t_cached is None:
        t_cached = t_stride
    require_capacity(int(t_cached), t_stride)
    if seq_lens is not None:
        _check_buffers(q.device, ("seq_lens", seq_lens, (b,), torch.int32))
    a = KvqArgs()
    a.q, a.k_wq, a.k_scales, a.k_biases = (q.data_ptr(), k_wq.data_ptr(), k_scales.data_ptr(),
                                           k_biases.data_ptr())
    a.v_wq, a.v_scales, a.v_biases = v_wq.data_ptr(), v_scales.data_ptr(), v_biases.data_ptr()
    a.new_k, a.new_v = new_k.data_ptr(), new_v.data_ptr()
    a.seq_lens = seq_lens.data_ptr() if seq_lens is not None else None
    a.b_rows, a.n_heads, a.n_kv_heads = b, h, hkv
    a.t_cached, a.t_stride, a.head_dim = int(t_cached), t_stride, dh
    a.bits, a.group_size, a.dtype = bits, group, code
    a.has_new_entry = 1 if has_new_entry else 0
    a.cache_batch_stride = hkv * t_stride if per_seq else 0
    a.t_begin = int(t_begin)
    a.t_end = KVQ_T_END_ALL if t_end is None else int(t_end)
    return a


KERNEL_NAMES = {0: "cuda-core", 1: "tensor-core", 2: "tcgen05"}


def plan_kernel(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *, bits,
                t_cached=None, seq_lens=None) -> str:
    """Which kernel `decode` would run on these arguments ("tensor-core",
    "tcgen05" or "cuda-core"); host only, nothing is launched."""
    a = _args(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, bits=bits,
              t_cached=t_cached, seq_lens=seq_lens)
    kind = _native.lib().kvq_plan_kernel(a)
    _native.check(min(kind, 0))
    return KERNEL_NAMES[kind]


class Workspace:
    """A reusable, growing scratch buffer on one device (the library never
    allocates; this is the caller-side allocation it asks for)."""

    def __init__(self):
        self._buf = None

    def get(self, nbytes: int, device, stream=None):
        """(buffer, bytes) of at least `nbytes`; a new buffer is allocated on
        `stream` (default: the current one), so the caching allocator orders
        the old buffer's reuse after that stream's work."""
        if nbytes == 0:
            return None, 0
        buf = self._buf
        if buf is None or buf.numel() < nbytes or buf.device != device:
            torch = _torch()
            self._buf = None
            if stream is None:
                self._buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
            else:
                with torch.cuda.stream(stream):
                    self._buf = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8,
                                            device=device)
        return self._buf, self._buf.numel()


_default_ws: dict = {}


def _workspace(device, nbytes, ws: Workspace | None, stream):
    """The scratch for one call on `stream`. Without a caller's workspace each
    stream has its own default one, so calls in flight on different streams
    never share partials; a buffer is allocated on the stream that uses it."""
    if ws is None:
        key = (device.type, device.index, stream.cuda_stream)
        ws = _default_ws.get(key)
        if ws is None:
            ws = _default_ws[key] = Workspace()
    return ws.get(nbytes, device, stream)


def decode(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *, bits,
           t_cached=None, seq_lens=None, out=None, workspace: Workspace | None = None,
           stream=None):
    """One decode step on the current CUDA stream: out [B, H, DH] in q's dtype.

    Caches are [HKV, T_stride, ...] (shared by every batch row, the reference
    layout) or [B, HKV, T_stride, ...] (one per sequence); `t_cached` is the
    logical length (default: all rows), `seq_lens` an optional int32 [B]
    tensor of ragged lengths (then `t_cached` bounds them)."""
    torch = _torch()
    a = _args(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, bits=bits,
              t_cached=t_cached, seq_lens=seq_lens)
    lib = _native.lib()
    if out is None:
        out = torch.empty_like(q)
    else:
        _check_buffers(q.device, ("out", out, q.shape, q.dtype))
    need = lib.kvq_workspace_bytes(a)
    s = stream if stream is not None else torch.cuda.current_stream(q.device)
    buf, have = _workspace(q.device, need, workspace, s)
    _native.check(lib.kvq_decode(a, out.data_ptr(), buf.data_ptr() if buf is not None else None,
                                 have, s.cuda_stream))
    return out


def decode_launch(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *, bits,
                  out, t_cached=None, seq_lens=None, workspace: Workspace | None = None):
    """The step of `decode` on these exact tensors, validated and planned
    once: returns launch(stream) that enqueues kvq_decode with the argument
    block built here (the tensors' contents may change between calls, not
    their addresses). For serving loops that call the same step every token
    (`HostStep`)."""
    torch = _torch()
    a = _args(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, bits=bits,
              t_cached=t_cached, seq_lens=seq_lens)
    _check_buffers(q.device, ("out", out, q.shape, q.dtype))
    lib = _native.lib()
    need = lib.kvq_workspace_bytes(a)
    ws = workspace if workspace is not None else Workspace()
    buf, have = ws.get(need, q.device)
    ws_ptr = buf.data_ptr() if buf is not None else None
    out_ptr = out.data_ptr()
    keep = (q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, out, seq_lens, buf)

    def launch(stream=None):
        s = stream if stream is not None else torch.cuda.current_stream(q.device)
        _native.check(lib.kvq_decode(a, out_ptr, ws_ptr, have, s.cuda_stream))
        return keep[9]

    return launch


_cuda_driver = None


def _graph_launcher(graph, stream):
    """A call that launches `graph` on `stream` and waits for it through the
    CUDA driver directly (cuGraphLaunch, cuStreamSynchronize: the executable
    graph is a driver object whichever runtime made it), or None when the
    driver or the graph's handle cannot be had -- the caller then replays
    through torch."""
    import ctypes
    global _cuda_driver
    try:
        if _cuda_driver is None:
            drv = ctypes.CDLL("libcuda.so.1")
            drv.cuGraphLaunch.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
            drv.cuGraphLaunch.restype = ctypes.c_int
            drv.cuStreamSynchronize.argtypes = [ctypes.c_void_p]
            drv.cuStreamSynchronize.restype = ctypes.c_int
            _cuda_driver = drv
        exec_handle = graph.raw_cuda_graph_exec()
        exec_handle = ctypes.c_void_p(int(exec_handle) if not isinstance(exec_handle, int)
                                      else exec_handle)
    except (OSError, AttributeError, TypeError, RuntimeError):
        return None
    drv, s = _cuda_driver, ctypes.c_void_p(stream.cuda_stream)

    def launch():
        rc = drv.cuGraphLaunch(exec_handle, s)
        if rc == 0:
            rc = drv.cuStreamSynchronize(s)
        if rc != 0:
            raise RuntimeError(f"CUDA driver error {rc} launching a captured decode step")

    return launch


class HostStep:
    """A decode step fed from host memory and returning to it -- the serving
    loop's shape, where each token's q, new_k and new_v arrive on the host
    and its output is wanted back there.

    The three inputs share one pinned staging buffer (`q`, `new_k`, `new_v`
    are views the caller may write into directly) and one device buffer, so a
    step makes one host-to-device copy; the output comes back with one
    device-to-host copy into the pinned `out` (both are `kvq_stage_copy`
    kernels, cheaper than copy-engine transfers at these sizes). `make_launch(q_dev, new_k_dev,
    new_v_dev, out_dev)` is called once with the device views and returns
    launch(stream), which enqueues the device step on them (`decode_launch`,
    or a sequence-split decoder's `launch`). With `graph=True` the copies and the step are captured once as
    a CUDA graph after one eager step, so each call is one graph launch and
    one wait. A call returns once the output is in `out`: its duration is the
    token's latency."""

    def __init__(self, make_launch, q_shape, kv_shape, dtype, device, graph: bool = True):
        import math
        torch = _torch()
        self.device = torch.device(device)
        esz = torch.empty((), dtype=dtype).element_size()
        align = 16 // esz                      # each segment starts on 16 bytes
        n_q, n_kv = math.prod(q_shape), math.prod(kv_shape)
        off_k = -(-n_q // align) * align
        off_v = off_k + -(-n_kv // align) * align
        total = off_v + n_kv
        self._host = torch.empty(total, dtype=dtype, pin_memory=True)
        self._dev = torch.empty(total, dtype=dtype, device=self.device)
        self.q = self._host[:n_q].view(q_shape)
        self.new_k = self._host[off_k:off_k + n_kv].view(kv_shape)
        self.new_v = self._host[off_v:off_v + n_kv].view(kv_shape)
        self.out = torch.empty(q_shape, dtype=dtype, pin_memory=True)
        dq = self._dev[:n_q].view(q_shape)
        dk = self._dev[off_k:off_k + n_kv].view(kv_shape)
        dv = self._dev[off_v:off_v + n_kv].view(kv_shape)
        self._dout = torch.empty(q_shape, dtype=dtype, device=self.device)
        self.h2d_bytes = total * esz
        self.d2h_bytes = self.out.numel() * esz
        self._stream = torch.cuda.Stream(self.device)
        self._done = torch.cuda.Event()
        with torch.cuda.stream(self._stream):
            launch = make_launch(dq, dk, dv, self._dout)

        lib = _native.lib()
        h_in, d_in, n_in = self._host.data_ptr(), self._dev.data_ptr(), self.h2d_bytes
        h_out, d_out, n_out = self.out.data_ptr(), self._dout.data_ptr(), self.d2h_bytes

        def body():
            # the staging copies are kernels reading / writing the pinned
            # buffers through their mapping (kvq_stage_copy): a few KB each,
            # where a copy engine's fixed latency would dominate
            s = self._stream.cuda_stream
            _native.check(lib.kvq_stage_copy(d_in, h_in, n_in, s))
            launch(self._stream)
            _native.check(lib.kvq_stage_copy(h_out, d_out, n_out, s))

        self._body = body
        with torch.cuda.stream(self._stream):
            body()                            # sets the kernels' attributes
        self._stream.synchronize()
        self._graph = None
        self._launch_graph = None
        if graph:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=self._stream):
                body()
            self._graph = g
            self._launch_graph = _graph_launcher(g, self._stream)
        # numpy views of the pinned staging: a host copy into them costs a
        # memcpy, not a torch dispatch
        self._np = (self.q.numpy(), self.new_k.numpy(), self.new_v.numpy())

    def __call__(self, q=None, new_k=None, new_v=None):
        """One step; q / new_k / new_v (host tensors or arrays), when given,
        are copied into the staging views first. Returns the pinned `out`,
        valid until the next call."""
        import numpy as np
        for src, dst in zip((q, new_k, new_v), self._np):
            if src is not None:
                np.copyto(dst, src if isinstance(src, np.ndarray) else src.numpy(), casting="no")
        if self._launch_graph is not None:
            self._launch_graph()
            return self.out
        torch = _torch()
        with torch.cuda.stream(self._stream):
            if self._graph is not None:
                self._graph.replay()
            else:
                self._body()
            self._done.record(self._stream)
        self._done.synchronize()
        return self.out

    def close(self) -> None:
        """Release the captured graph (before the tensors it uses go)."""
        self._launch_graph = None
        self._graph = None


def decode_partial(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, *,
                   bits, t_begin, t_end, has_new_entry, t_cached=None, seq_lens=None,
                   part_o=None, part_m=None, part_l=None, workspace: Workspace | None = None,
                   stream=None):
    """One T-range shard: (O [B,H,DH] fp32 unnormalised, m [B,H], l [B,H])."""
    torch = _torch()
    a = _args(q, k_wq, k_scales, k_biases, v_wq, v_scales, v_biases, new_k, new_v, bits=bits,
              t_cached=t_cached, seq_lens=seq_lens, t_begin=t_begin, t_end=t_end,
              has_new_entry=has_new_entry)
    lib = _native.lib()
    b, h, dh = q.shape
    if part_o is None:
        part_o = torch.empty((b, h, dh), dtype=torch.float32, device=q.device)
    if part_m is None:
        part_m = torch.empty((b, h), dtype=torch.float32, device=q.device)
    if part_l is None:
        part_l = torch.empty((b, h), dtype=torch.float32, device=q.device)
    _check_buffers(q.device, ("part_o", part_o, (b, h, dh), torch.float32),
                   ("part_m", part_m, (b, h), torch.float32),
                   ("part_l", part_l, (b, h), torch.float32))
    need = lib.kvq_workspace_bytes(a)
    s = stream if stream is not None else torch.cuda.current_stream(q.device)
    buf, have = _workspace(q.device, need, workspace, s)
    _native.check(lib.kvq_decode_partial(a, part_o.data_ptr(), part_m.data_ptr(),
                                         part_l.data_ptr(),
                                         buf.data_ptr() if buf is not None else None, have,
                                         s.cuda_stream))
    return part_o, part_m, part_l


def lse_merge(part_o, part_m, part_l, out_dtype, out=None, stream=None):
    """Merge stacked partials part_o [P, B, H, DH], part_m/part_l [P, B, H]
    into out [B, H, DH] (the sequence-split merge)."""
    torch = _torch()
    if part_o.dim() != 4:
        raise ValueError(f"part_o must be [P, B, H, DH], got {tuple(part_o.shape)}")
    n, b, h, dh = part_o.shape
    dev = part_o.device
    _dtype_code(out_dtype)
    bufs = [("part_o", part_o, (n, b, h, dh), torch.float32),
            ("part_m", part_m, (n, b, h), torch.float32),
            ("part_l", part_l, (n, b, h), torch.float32)]
    if out is not None:
        bufs.append(("out", out, (b, h, dh), out_dtype))
    _check_buffers(dev, *bufs)
    if out is None:
        out = torch.empty((b, h, dh), dtype=out_dtype, device=dev)
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    lib = _native.lib()
    _native.check(lib.kvq_lse_merge(part_o.data_ptr(), part_m.data_ptr(), part_l.data_ptr(), n,
                                    b * h, dh, _dtype_code(out_dtype), out.data_ptr(),
                                    s.cuda_stream))
    return out


def record_floats(rows: int, head_dim: int) -> int:
    """Floats in one partial record: O [rows, DH], then m [rows], then l [rows]."""
    return rows * (head_dim + 2)


def record_views(record, b_rows: int, n_heads: int, head_dim: int):
    """(part_o [B, H, DH], part_m [B, H], part_l [B, H]) views into one fp32
    partial record, for `decode_partial` to write in place."""
    rows = b_rows * n_heads
    if record.dtype != _torch().float32 or record.numel() != record_floats(rows, head_dim):
        raise ValueError(f"a record of {rows} rows x DH {head_dim} is "
                         f"{record_floats(rows, head_dim)} fp32 values")
    o = record[:rows * head_dim].view(b_rows, n_heads, head_dim)
    m = record[rows * head_dim:rows * (head_dim + 1)].view(b_rows, n_heads)
    l = record[rows * (head_dim + 1):].view(b_rows, n_heads)
    return o, m, l


def lse_merge_records(records, b_rows: int, n_heads: int, head_dim: int, out_dtype, out=None,
                      stream=None):
    """Merge partial records laid end to end (records [P, record_floats]) --
    what an all-gather of every rank's record produces -- into out [B, H, DH]."""
    torch = _torch()
    rows = b_rows * n_heads
    if (records.dim() != 2 or records.shape[1] != record_floats(rows, head_dim)
            or records.dtype != torch.float32 or not records.is_contiguous()):
        raise ValueError(f"records must be contiguous fp32 [P, {record_floats(rows, head_dim)}]")
    _dtype_code(out_dtype)
    if out is None:
        out = torch.empty((b_rows, n_heads, head_dim), dtype=out_dtype, device=records.device)
    else:
        _check_buffers(records.device, ("out", out, (b_rows, n_heads, head_dim), out_dtype))
    s = stream if stream is not None else torch.cuda.current_stream(records.device)
    _native.check(_native.lib().kvq_lse_merge_records(records.data_ptr(), records.shape[0], rows,
                                                      head_dim, _dtype_code(out_dtype),
                                                      out.data_ptr(), s.cuda_stream))
    return out


def quantize(w, bits: int, group_size: int = 64, stream=None):
    """Canonical quantizer on the device: w [..., DH] (fp16/fp32, contiguous)
    -> (words uint32-as-int32 [..., DH*bits/32], scales [..., DH/g], biases)."""
    torch = _torch()
    if not w.is_cuda or not w.is_contiguous():
        raise ValueError("w must be a contiguous CUDA tensor")
    dh = w.shape[-1]
    rows = w.numel() // dh if dh else 0
    lead = tuple(w.shape[:-1])
    words = torch.empty(lead + (dh * bits // 32,), dtype=torch.int32, device=w.device)
    scales = torch.empty(lead + (dh // group_size,), dtype=w.dtype, device=w.device)
    biases = torch.empty_like(scales)
    s = stream if stream is not None else torch.cuda.current_stream(w.device)
    _native.check(_native.lib().kvq_quantize(w.data_ptr(), rows, dh, bits, group_size,
                                             _dtype_code(w.dtype), words.data_ptr(),
                                             scales.data_ptr(), biases.data_ptr(),
                                             s.cuda_stream))
    return words, scales, biases


def cache_append(w, words, scales, biases, bits: int, *, position: int = 0, positions=None,
                 stream=None):
    """Quantize w [B, HKV, L, DH] into positions [pos_b, pos_b + L) of a
    per-sequence packed cache (words [B, HKV, T_stride, DH*bits/32], scales and
    biases [B, HKV, T_stride, DH/g]) -- or of a shared [HKV, T_stride, ...]
    cache when B == 1. pos_b = positions[b] (an int32 [B] CUDA tensor, read on
    the device) or `position`. Bit-identical to `quantize` of the same rows."""
    torch = _torch()
    if w.dim() != 4 or not w.is_cuda or not w.is_contiguous():
        raise ValueError("w must be a contiguous CUDA tensor [B, HKV, L, DH]")
    b, hkv, n_new, dh = w.shape
    per_seq = words.dim() == 4
    lead = tuple(words.shape[:-2]) if per_seq else (1,) + tuple(words.shape[:-2])
    if lead != (b, hkv):
        raise ValueError(f"cache leads with {tuple(words.shape[:-2])}; w is [{b}, {hkv}, ...]")
    t_stride = words.shape[-2]
    groups = scales.shape[-1]
    _check_words("words", words)
    if groups == 0 or dh % groups or words.shape[-1] * 32 != dh * bits:
        raise ValueError(f"cache rows do not hold {dh} codes of {bits} bits")
    for name, ten in (("words", words), ("scales", scales), ("biases", biases)):
        if not ten.is_cuda or not ten.is_contiguous() or ten.device != w.device:
            raise ValueError(f"{name} must be a contiguous CUDA tensor on {w.device}")
        if tuple(ten.shape[:-1]) != tuple(words.shape[:-1]):
            raise ValueError(f"{name} has shape {tuple(ten.shape)}")
    if scales.dtype != w.dtype or biases.dtype != w.dtype:
        raise ValueError("scales and biases must have w's dtype")
    if positions is not None:
        if positions.dtype != torch.int32 or tuple(positions.shape) != (b,) or not positions.is_cuda:
            raise ValueError("positions must be a CUDA int32 tensor [B]")
    s = stream if stream is not None else torch.cuda.current_stream(w.device)
    _native.check(_native.lib().kvq_cache_append(
        w.data_ptr(), b, hkv, n_new, dh, bits, dh // groups, _dtype_code(w.dtype),
        positions.data_ptr() if positions is not None else None, int(position), t_stride,
        hkv * t_stride if per_seq else 0, words.data_ptr(), scales.data_ptr(),
        biases.data_ptr(), s.cuda_stream))


def quantize_cache(cache, bits: int, group_size: int = 64):
    """Packed artefact triplet for an (H, T, DH) -- or (B, H, T, DH) -- cache,
    quantized row by row on the device (kernelverify/pack/kv_attention.py:270-283)."""
    return quantize(cache.contiguous(), bits, group_size)


def dequant(words, scales, biases, bits: int, stream=None):
    """fp32 dequantized values of a packed artefact, same leading shape."""
    torch = _torch()
    if (words.dim() < 1 or words.shape[-1] == 0 or bits not in SUPPORTED_BITS
            or words.shape[-1] * 32 % bits):
        raise ValueError(f"words {tuple(words.shape)} at {bits} bits is not a packed artefact")
    _check_words("words", words)
    groups = scales.shape[-1]
    dh = words.shape[-1] * 32 // bits
    if groups == 0 or dh % groups:
        raise ValueError(f"scales carry {groups} groups per row, which does not divide {dh}")
    _dtype_code(scales.dtype)
    lead = tuple(words.shape[:-1])
    _check_buffers(words.device, ("words", words, words.shape, words.dtype),
                   ("scales", scales, lead + (groups,), scales.dtype),
                   ("biases", biases, lead + (groups,), scales.dtype))
    rows = words.numel() // words.shape[-1]
    out = torch.empty(tuple(words.shape[:-1]) + (dh,), dtype=torch.float32, device=words.device)
    s = stream if stream is not None else torch.cuda.current_stream(words.device)
    _native.check(_native.lib().kvq_dequant(words.data_ptr(), scales.data_ptr(),
                                            biases.data_ptr(), rows, dh, bits, dh // groups,
                                            _dtype_code(scales.dtype), out.data_ptr(),
                                            s.cuda_stream))
    return out


def build(torch_module=None):
    """The framework door: a callable in the reference's MLX-door spelling
    (kernelverify/pack/kv_attention.py:369-393).

        kernel = build(torch)
        [out] = kernel(inputs=[q, k_wq, k_scales, k_biases, v_wq, v_scales,
                               v_biases, new_k, new_v],
                       t_cached=t, template=[("T", torch.float16),
                                             ("BITS", bits), ("DH", dh)])

    Padded caches are passed whole with the logical length as a scalar;
    `output_shapes`/`output_dtypes`, when given, are checked against what the
    step produces; `grid`/`threadgroup` are accepted and ignored (the library
    plans its own launch)."""
    def guarded(*, inputs, t_cached, template=(), output_shapes=None, output_dtypes=None,
                grid=None, threadgroup=None, seq_lens=None):
        tmpl = dict(template)
        q = inputs[0]
        bits = int(tmpl.get("BITS", 0)) or None
        if bits is None:
            raise ValueError("template must carry BITS")
        if "DH" in tmpl and int(tmpl["DH"]) != q.shape[-1]:
            raise ValueError(f"template DH={tmpl['DH']} but q has head_dim {q.shape[-1]}")
        if "T" in tmpl and tmpl["T"] != q.dtype:
            raise ValueError(f"template T={tmpl['T']} but q is {q.dtype}")
        if output_shapes is not None and [tuple(s) for s in output_shapes] != [tuple(q.shape)]:
            raise ValueError(f"output_shapes {output_shapes} != [{tuple(q.shape)}]")
        if output_dtypes is not None and list(output_dtypes) != [q.dtype]:
            raise ValueError(f"output_dtypes {output_dtypes} != [{q.dtype}]")
        return [decode(*inputs, bits=bits, t_cached=t_cached, seq_lens=seq_lens)]

    return guarded


def kernel_spec(ragged: bool = False):
    """The runner-door template (kernelverify/pack/kv_attention.py:292-352),
    for `kernelverify_b200.runners.CudaRunner`. `specialize()` fills `$T`,
    `$BITS`, `$DH` (and optionally `$GROUP`); the source names the library
    entry point and the instantiation it selects, the bindings keep the
    reference's names and order. ragged=True adds an int32 input `seq_lens`
    [b_rows] after new_v: per-sequence logical lengths, each at most the
    case's t_cached (one cache per sequence: params cache_batch_stride)."""
    from kernelverify_b200.runners import Binding, BindingKind, KernelSpec, LaunchSpec

    source = (
        "// kvq-b200 library translation unit: libkvq_b200.so, entry kvq_decode\n"
        "#pragma kvq library kvq_decode\n"
        "#pragma kvq instantiate T=$T BITS=$BITS DH=$DH\n"
    )
    return KernelSpec(
        source=source,
        entry_point=KERNEL_NAME,
        name=f"{KERNEL_NAME}-$BITS bit-DH$DH-$T",
        bindings=(Binding(BindingKind.INPUT, "q"),
                  Binding(BindingKind.INPUT, "k_wq"),
                  Binding(BindingKind.INPUT, "k_scales"),
                  Binding(BindingKind.INPUT, "k_biases"),
                  Binding(BindingKind.INPUT, "v_wq"),
                  Binding(BindingKind.INPUT, "v_scales"),
                  Binding(BindingKind.INPUT, "v_biases"),
                  Binding(BindingKind.INPUT, "new_k"),
                  Binding(BindingKind.INPUT, "new_v"),
                  *((Binding(BindingKind.INPUT, "seq_lens"),) if ragged else ()),
                  Binding(BindingKind.OUTPUT),
                  Binding(BindingKind.SCALAR, "n_heads", "uint32"),
                  Binding(BindingKind.SCALAR, "t_cached", "uint32"),
                  Binding(BindingKind.SCALAR, "n_kv_heads", "uint32"),
                  Binding(BindingKind.SCALAR, "t_stride", "uint32")),
        launch=LaunchSpec(grid=(THREADS_PER_CTA, 1, ["b_rows", "n_heads"]),
                          threadgroup=(THREADS_PER_CTA, 1, 1)),
    )
