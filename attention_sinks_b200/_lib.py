"""ctypes binding of the C ABI in include/sinkcache_b200.h, plus torch-tensor wrappers.

Every GPU operation of this package goes through these wrappers into the sm_100a library
`lib/libsinkcache_b200.so`.  There is no other implementation: if the library is missing,
the first call raises, it never falls back to PyTorch or the CPU.
"""

import ctypes
import os
import threading

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libsinkcache_b200.so")

DTYPE_F32, DTYPE_BF16, DTYPE_F16 = 0, 1, 2
OP_APPEND, OP_EVICT, OP_ATTEND, OP_FUSED_STEP = 0, 1, 2, 3
STATUS_WAIT_TIMEOUT = 1

_DTYPE_CODE = {torch.float32: DTYPE_F32, torch.bfloat16: DTYPE_BF16, torch.float16: DTYPE_F16}

EXPORTED_SYMBOLS = (
    "sink_abi_version", "sink_strerror", "sink_workspace_bytes", "sink_plan", "sink_append",
    "sink_evict_rerotate", "sink_decode_attention", "sink_fused_decode_step", "sink_read_status",
    "sink_decode_attention_noalloc", "sink_v2_place", "sink_v2_decode_step", "sink_prepare_device",
    "sink_debug_fail_next_wait", "sink_plan_launch", "sink_evict_rerotate_keycopy", "sink_v2_gather",
    "sink_debug_cluster_capacity", "sink_launch_count",
)
LAUNCH_SPLIT, LAUNCH_CLUSTER, LAUNCH_TENSOR = 0, 1, 2
NOALLOC_SCRATCH_BYTES = 16 << 20
# argument errors (negative return codes of the C ABI)
EINVAL, EDTYPE, EHEADDIM, EGROUP, ELAYOUT, EWORKSPACE, EDEVICE, ESCRATCH = -1, -2, -3, -4, -5, -6, -7, -8


class KVBuffers(ctypes.Structure):
    """sink_kv_buffers_t"""
    _fields_ = [
        ("k", ctypes.c_void_p), ("v", ctypes.c_void_p),
        ("k_dtype", ctypes.c_int32), ("v_dtype", ctypes.c_int32),
        ("batch", ctypes.c_int32), ("heads_kv", ctypes.c_int32),
        ("slots", ctypes.c_int32), ("head_dim", ctypes.c_int32),
        ("k_stride_b", ctypes.c_int64), ("k_stride_h", ctypes.c_int64),
        ("v_stride_b", ctypes.c_int64), ("v_stride_h", ctypes.c_int64),
    ]


class Rows(ctypes.Structure):
    """sink_rows_t"""
    _fields_ = [
        ("data", ctypes.c_void_p), ("dtype", ctypes.c_int32), ("heads", ctypes.c_int32),
        ("n", ctypes.c_int32), ("pad_", ctypes.c_int32),
        ("stride_b", ctypes.c_int64), ("stride_h", ctypes.c_int64), ("stride_t", ctypes.c_int64),
    ]


_lib = None
_lock = threading.Lock()


def _declare(lib):
    i32, i64, sz, vp, fp = ctypes.c_int32, ctypes.c_int64, ctypes.c_size_t, ctypes.c_void_p, ctypes.c_void_p
    pkv, prows = ctypes.POINTER(KVBuffers), ctypes.POINTER(Rows)
    pi32 = ctypes.POINTER(ctypes.c_int32)
    sig = {
        "sink_abi_version": (i32, []),
        "sink_launch_count": (ctypes.c_uint64, []),
        "sink_strerror": (ctypes.c_char_p, [i32]),
        "sink_workspace_bytes": (sz, [i32] * 12),
        "sink_plan": (i32, [i32] * 12 + [pi32] * 6),
        "sink_plan_launch": (i32, [i32] * 12 + [pi32] * 2),
        "sink_append": (i32, [pkv, prows, prows, i32, vp]),
        "sink_evict_rerotate": (i32, [pkv, i32, i32, i32, fp, fp, i32, vp, sz, vp]),
        "sink_evict_rerotate_keycopy": (i32, [pkv, i32, i32, i32, fp, fp, i32, prows, vp, sz, vp]),
        "sink_decode_attention": (i32, [prows, pkv, i32, ctypes.c_float, vp, i64, vp, i64, i64, vp, sz, vp]),
        "sink_fused_decode_step": (i32, [pkv, prows, prows, prows, i32, i32, i32, i32, fp, fp, i32,
                                         ctypes.c_float, vp, i64, vp, i64, i64, vp, sz, vp]),
        "sink_read_status": (i32, [vp, vp, pi32]),
        "sink_prepare_device": (i32, []),
        "sink_debug_fail_next_wait": (i32, [i32, i32]),
        "sink_debug_cluster_capacity": (i32, [i32]),
        "sink_decode_attention_noalloc": (i32, [prows, pkv, i32, ctypes.c_float, vp, i64, vp, i64, i64, vp]),
        "sink_v2_place": (i32, [pkv, prows, prows, prows, vp, i32, prows, vp, i64, i32, i32, vp, i32, vp]),
        "sink_v2_gather": (i32, [pkv, i32, i32, i32, i64, i64, prows, prows, prows, prows, vp]),
        "sink_v2_decode_step": (i32, [pkv, prows, prows, prows, vp, i32, vp, i32, i32, vp, i32, prows,
                                      ctypes.c_float, vp, i64, vp, i64, i64, vp, sz, vp]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args


def lib():
    """The loaded library.  Raises if it has not been built (there is no fallback)."""
    global _lib
    if _lib is None:
        with _lock:
            if _lib is None:
                if not os.path.exists(LIB_PATH):
                    raise RuntimeError(
                        f"sinkcache_b200 CUDA library not found at {LIB_PATH}; build it with "
                        "`python -m attention_sinks_b200.build`")
                handle = ctypes.CDLL(LIB_PATH)
                _declare(handle)
                _lib = handle
    return _lib


def strerror(code: int) -> str:
    return lib().sink_strerror(int(code)).decode()


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} failed ({rc}): {strerror(rc)}")


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPE_CODE[dtype]
    except KeyError:
        raise TypeError(f"sinkcache_b200 supports float32 / bfloat16 / float16, got {dtype}") from None


def check_device(device: torch.device) -> None:
    """The kernels run on CUDA devices only; there is no CPU implementation."""
    if device.type != "cuda":
        raise RuntimeError(f"sinkcache_b200 runs on CUDA devices only (got {device})")


def _require_cuda(*tensors: torch.Tensor) -> None:
    for t in tensors:
        check_device(t.device)


def kv_desc(kbuf: torch.Tensor, vbuf: torch.Tensor) -> KVBuffers:
    """Descriptor of [B, Hkv, slots, D] cache buffers (rows must be contiguous)."""
    _require_cuda(kbuf, vbuf)
    if kbuf.shape != vbuf.shape or kbuf.dim() != 4:
        raise ValueError(f"K/V buffers must be [B, H, slots, D] of one shape, got {tuple(kbuf.shape)}, "
                         f"{tuple(vbuf.shape)}")
    d = kbuf.shape[-1]
    for t in (kbuf, vbuf):  # a single row has no row stride to check
        if t.stride(-1) != 1 or (t.shape[-2] > 1 and t.stride(-2) != d):
            raise ValueError("cache buffers need contiguous rows (stride[-2] == head_dim, stride[-1] == 1)")
    b, h, s, _ = kbuf.shape
    return KVBuffers(kbuf.data_ptr(), vbuf.data_ptr(), dtype_code(kbuf.dtype), dtype_code(vbuf.dtype),
                     b, h, s, d, kbuf.stride(0), kbuf.stride(1), vbuf.stride(0), vbuf.stride(1))


def rows_desc(t: torch.Tensor) -> Rows:
    """Descriptor of a [B, H, n, D] tensor with a unit last stride."""
    _require_cuda(t)
    if t.dim() != 4 or t.stride(-1) != 1:
        raise ValueError(f"expected a [B, H, n, D] tensor with unit last stride, got {tuple(t.shape)} "
                         f"strides {t.stride()}")
    return Rows(t.data_ptr(), dtype_code(t.dtype), t.shape[1], t.shape[2], 0,
                t.stride(0), t.stride(1), t.stride(2))


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


_sm_count = {}


_prepared: set[int] = set()


def prepare_device(device: torch.device) -> None:
    """The library's one-time set-up of `device` (kernel shared-memory opt-ins, the tensor-map
    encoder lookup): must run outside any CUDA-graph capture, so the caches call it at lazy
    initialisation."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx in _prepared:
        return
    with torch.cuda.device(idx):
        _check(lib().sink_prepare_device(), "sink_prepare_device")
    _prepared.add(idx)


def sm_count(device: torch.device) -> int:
    idx = device.index if device.index is not None else torch.cuda.current_device()
    if idx not in _sm_count:
        _sm_count[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _sm_count[idx]


def workspace_bytes(op: int, batch: int, heads_kv: int, heads_q: int, head_dim: int,
                    k_dtype: torch.dtype, v_dtype: torch.dtype, rows: int, n_sink: int,
                    window: int, drop: int, num_sms: int) -> int:
    n = lib().sink_workspace_bytes(op, batch, heads_kv, heads_q, head_dim, dtype_code(k_dtype),
                                   dtype_code(v_dtype), rows, n_sink, window, drop, num_sms)
    if n == 0:
        raise ValueError("sinkcache_b200: unsupported shapes for the workspace query "
                         f"(op={op}, B={batch}, Hkv={heads_kv}, Hq={heads_q}, D={head_dim}, "
                         f"K={k_dtype}, V={v_dtype}, rows={rows})")
    return int(n)


def plan(op: int, batch: int, heads_kv: int, heads_q: int, head_dim: int, k_dtype: torch.dtype,
         v_dtype: torch.dtype, rows: int, n_sink: int, window: int, drop: int, num_sms: int) -> dict:
    out = [ctypes.c_int32() for _ in range(6)]
    rc = lib().sink_plan(op, batch, heads_kv, heads_q, head_dim, dtype_code(k_dtype), dtype_code(v_dtype),
                         rows, n_sink, window, drop, num_sms, *[ctypes.byref(o) for o in out])
    _check(rc, "sink_plan")
    keys = ("splits", "rows_per_split", "chunk_rows", "stages", "smem_bytes", "cluster_ctas")
    res = {k: o.value for k, o in zip(keys, out)}
    mode, ctas = ctypes.c_int32(), ctypes.c_int32()
    rc = lib().sink_plan_launch(op, batch, heads_kv, heads_q, head_dim, dtype_code(k_dtype), dtype_code(v_dtype),
                                rows, n_sink, window, drop, num_sms, ctypes.byref(mode), ctypes.byref(ctas))
    _check(rc, "sink_plan_launch")
    res["launch"], res["ctas"] = mode.value, ctas.value
    return res


class Workspace:
    """Device scratch for the kernels (split partials, halo rows, status word), grown on
    demand and reused.  A step captured in a CUDA graph keeps the pointer it saw, so
    size it before capture (SinkLayer does, at lazy initialisation)."""

    def __init__(self):
        self.buf = None

    def get(self, nbytes: int, device: torch.device) -> torch.Tensor:
        if self.buf is None or self.buf.numel() < nbytes or self.buf.device != device:
            self.buf = torch.zeros(max(nbytes, 256), dtype=torch.uint8, device=device)
        return self.buf

    def read_status(self) -> int:
        """Status bits set by kernels since the last read (synchronises the stream)."""
        if self.buf is None:
            return 0
        st = ctypes.c_int32(0)
        _check(lib().sink_read_status(self.buf.data_ptr(), stream_handle(self.buf.device),
                                      ctypes.byref(st)), "sink_read_status")
        return st.value

    def check(self) -> None:
        """Raise if a kernel reported a failure since the last read (synchronises the stream).
        A bounded wait that ran out means the launches since then produced no valid result
        and may have left an in-place eviction partly applied."""
        status = self.read_status()
        if status:
            what = "a bounded wait for a bulk copy ran out" if status & STATUS_WAIT_TIMEOUT else "unknown failure"
            raise RuntimeError(f"sinkcache_b200 kernel status 0x{status:x}: {what}; the results of the launches "
                               "since the last check are void")


# ---------------------------------------------------------------------------- operations


def fail_next_wait(chunk: int, polls: int) -> None:
    """Failure-detection test hook (sink_debug_fail_next_wait): the next stream-kernel launch
    leaves chunk `chunk` of every split unissued, with every wait bounded by `polls` polls,
    so that wait runs out and the launch reports SINK_STATUS_WAIT_TIMEOUT."""
    _check(lib().sink_debug_fail_next_wait(int(chunk), int(polls)), "sink_debug_fail_next_wait")


def launch_count() -> int:
    """Kernel launches the library has issued in this process (sink_launch_count)."""
    return int(lib().sink_launch_count())


def force_cluster_capacity(clusters: int) -> None:
    """Cluster-fallback test hook (sink_debug_cluster_capacity): clusters >= 0 is taken as the
    device's capacity for every clustered stream launch (0: clustered plans run as split
    launches); -1 asks the device again."""
    _check(lib().sink_debug_cluster_capacity(int(clusters)), "sink_debug_cluster_capacity")


def append(kbuf: torch.Tensor, vbuf: torch.Tensor, k: torch.Tensor, v: torch.Tensor, row: int) -> None:
    """kbuf[:, :, row:row+n] = k; vbuf[:, :, row:row+n] = v (cache.py:159-160)."""
    kv = kv_desc(kbuf, vbuf)
    rc = lib().sink_append(ctypes.byref(kv), ctypes.byref(rows_desc(k)), ctypes.byref(rows_desc(v)),
                           int(row), stream_handle(kbuf.device))
    _check(rc, "sink_append")


def evict_rerotate(kbuf: torch.Tensor, vbuf: torch.Tensor, n_sink: int, window: int, drop: int,
                   cos: torch.Tensor | None, sin: torch.Tensor | None, ws: Workspace) -> None:
    """In-place shift of the window by `drop` rows, keys rotated by -drop (kernels.py:59-73)."""
    kv = kv_desc(kbuf, vbuf)
    b, h, _, d = kbuf.shape
    need = workspace_bytes(OP_EVICT, b, h, h, d, kbuf.dtype, vbuf.dtype, 0, n_sink, window, drop,
                           sm_count(kbuf.device))
    buf = ws.get(need, kbuf.device)
    rotate = cos is not None
    rc = lib().sink_evict_rerotate(ctypes.byref(kv), n_sink, window, drop,
                                   cos.data_ptr() if rotate else None, sin.data_ptr() if rotate else None,
                                   1 if rotate else 0, buf.data_ptr(), buf.numel(),
                                   stream_handle(kbuf.device))
    _check(rc, "sink_evict_rerotate")


def evict_rerotate_keycopy(kbuf: torch.Tensor, vbuf: torch.Tensor, n_sink: int, window: int, drop: int,
                           cos: torch.Tensor | None, sin: torch.Tensor | None, k_copy: torch.Tensor,
                           ws: Workspace) -> None:
    """evict_rerotate (nothing moves when drop == 0) that also writes the window rows' final
    keys, rounded to the value dtype, into k_copy rows [n_sink, n_sink + window)."""
    kv = kv_desc(kbuf, vbuf)
    b, h, _, d = kbuf.shape
    need = workspace_bytes(OP_EVICT, b, h, h, d, kbuf.dtype, vbuf.dtype, 0, n_sink, window, drop,
                           sm_count(kbuf.device))
    buf = ws.get(need, kbuf.device)
    rotate = cos is not None and drop > 0
    rc = lib().sink_evict_rerotate_keycopy(ctypes.byref(kv), n_sink, window, drop,
                                           cos.data_ptr() if rotate else None, sin.data_ptr() if rotate else None,
                                           1 if rotate else 0, ctypes.byref(rows_desc(k_copy)), buf.data_ptr(),
                                           buf.numel(), stream_handle(kbuf.device))
    _check(rc, "sink_evict_rerotate_keycopy")


def mask_arg(mask: torch.Tensor | None, batch: int, rows: int) -> tuple[int | None, int, torch.Tensor | None]:
    """(pointer, batch stride in bytes, tensor to keep alive until the launch) of a boolean
    [B or 1, 1, 1, rows] attention mask for a one-token query (True = attend), as the
    kernels take it."""
    if mask is None:
        return None, 0, None
    if (mask.dtype != torch.bool or mask.dim() != 4 or mask.shape[1] != 1 or mask.shape[2] != 1
            or mask.shape[3] != rows or mask.shape[0] not in (1, batch)):
        raise ValueError(f"kernel masks are boolean [B, 1, 1, {rows}], got {mask.dtype} {tuple(mask.shape)}")
    _require_cuda(mask)
    if mask.stride(-1) != 1:
        mask = mask.contiguous()
    return mask.data_ptr(), (mask.stride(0) if mask.shape[0] > 1 else 0), mask


def decode_attention(q: torch.Tensor, kbuf: torch.Tensor, vbuf: torch.Tensor, rows: int, scale: float,
                     out: torch.Tensor, ws: Workspace, mask: torch.Tensor | None = None) -> torch.Tensor:
    """out[B, 1, Hq, D] = attention of q[B, Hq, 1, D] over kbuf/vbuf rows [0, rows), rows
    with a False `mask` entry left out."""
    kv = kv_desc(kbuf, vbuf)
    b, h, _, d = kbuf.shape
    need = workspace_bytes(OP_ATTEND, b, h, q.shape[1], d, kbuf.dtype, vbuf.dtype, rows, 0, 1, 0,
                           sm_count(kbuf.device))
    buf = ws.get(need, kbuf.device)
    mptr, msb, _keep = mask_arg(mask, b, rows)
    rc = lib().sink_decode_attention(ctypes.byref(rows_desc(q)), ctypes.byref(kv), int(rows), float(scale),
                                     mptr, msb, out.data_ptr(), out.stride(0), out.stride(2), buf.data_ptr(),
                                     buf.numel(), stream_handle(kbuf.device))
    _check(rc, "sink_decode_attention")
    return out


def fused_decode_step(kbuf: torch.Tensor, vbuf: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                      q: torch.Tensor, n_sink: int, window: int, drop: int, append_row: int,
                      cos: torch.Tensor | None, sin: torch.Tensor | None, scale: float,
                      out: torch.Tensor, ws: Workspace, mask: torch.Tensor | None = None) -> torch.Tensor:
    """Evict `drop` rows (re-rotating keys), append (k, v) at `append_row`, attend q over rows
    [0, append_row] -- one pass over the cache."""
    kv = kv_desc(kbuf, vbuf)
    b, h, _, d = kbuf.shape
    need = workspace_bytes(OP_FUSED_STEP, b, h, q.shape[1], d, kbuf.dtype, vbuf.dtype, append_row + 1,
                           n_sink, window, drop, sm_count(kbuf.device))
    buf = ws.get(need, kbuf.device)
    rotate = cos is not None
    mptr, msb, _keep = mask_arg(mask, b, append_row + 1)
    rc = lib().sink_fused_decode_step(
        ctypes.byref(kv), ctypes.byref(rows_desc(k)), ctypes.byref(rows_desc(v)), ctypes.byref(rows_desc(q)),
        n_sink, window, drop, append_row, cos.data_ptr() if rotate else None,
        sin.data_ptr() if rotate else None, 1 if rotate else 0, float(scale), mptr, msb, out.data_ptr(),
        out.stride(0), out.stride(2), buf.data_ptr(), buf.numel(), stream_handle(kbuf.device))
    _check(rc, "sink_fused_decode_step")
    return out


def decode_attention_noalloc(q: torch.Tensor, kbuf: torch.Tensor, vbuf: torch.Tensor, rows: int, scale: float,
                             out: torch.Tensor, mask: torch.Tensor | None = None) -> int:
    """decode_attention without a workspace, for callers that cannot allocate device memory:
    the library's static 16 MiB device scratch holds the split partials instead.  Returns
    the library's code (0, or ESCRATCH when the request needs more scratch than that)."""
    kv = kv_desc(kbuf, vbuf)
    mptr, msb, _keep = mask_arg(mask, kbuf.shape[0], rows)
    return lib().sink_decode_attention_noalloc(ctypes.byref(rows_desc(q)), ctypes.byref(kv), int(rows),
                                               float(scale), mptr, msb, out.data_ptr(), out.stride(0),
                                               out.stride(2), stream_handle(kbuf.device))


# ------------------------------------------------------------------ ring-buffer (v2) layer


def _region_args(reg_k: torch.Tensor | None, reg_pos: torch.Tensor | None, R: int,
                 inv_freq: torch.Tensor | None):
    if R == 0:
        return None, None, None, 0
    _require_cuda(reg_k, reg_pos, inv_freq)
    if reg_pos.dtype != torch.int64 or inv_freq.dtype != torch.float64:
        raise TypeError("region positions are int64 and inv_freq float64 on the device")
    if not reg_pos.is_contiguous() or not inv_freq.is_contiguous():
        raise ValueError("region positions and inv_freq must be contiguous")
    return ctypes.byref(rows_desc(reg_k)), reg_pos.data_ptr(), inv_freq.data_ptr(), inv_freq.numel()


def _position_arg(position: torch.Tensor | None):
    if position is None:
        return None
    _require_cuda(position)
    if position.dtype != torch.int64 or position.numel() != 2 or not position.is_contiguous():
        raise ValueError("position is a contiguous device int64 tensor {t, 0}")
    return position.data_ptr()


def v2_place(kbuf: torch.Tensor, vbuf: torch.Tensor, k: torch.Tensor | None, v: torch.Tensor | None,
             reg_k: torch.Tensor | None, reg_pos: torch.Tensor | None, R: int,
             region_out: torch.Tensor | None, position: torch.Tensor | None, t: int, n_sink: int,
             window: int, inv_freq: torch.Tensor | None) -> None:
    """Ring-buffer layer place step (cache_v2.py:171-176, :101-116): (k, v) into ring slot
    (t - n_sink) mod (window + 1); region keys reg_k[:, :, :R] (original rotations, positions
    reg_pos[:R]) rotated to sit just before the window, into `region_out` rows [0, R) or,
    when it is None, the cache rows after the ring.  t comes from the device tensor
    `position` = {t, 0} (advanced by one) or, when that is None, from the host int `t`."""
    kv = kv_desc(kbuf, vbuf)
    rk, rp, inv, rot_half = _region_args(reg_k, reg_pos, R, inv_freq)
    kd = ctypes.byref(rows_desc(k)) if k is not None else None
    vd = ctypes.byref(rows_desc(v)) if v is not None else None
    od = ctypes.byref(rows_desc(region_out)) if region_out is not None else None
    rc = lib().sink_v2_place(ctypes.byref(kv), kd, vd, rk, rp, int(R), od, _position_arg(position),
                             int(t), int(n_sink), int(window), inv, int(rot_half), stream_handle(kbuf.device))
    _check(rc, "sink_v2_place")


def v2_decode_step(kbuf: torch.Tensor, vbuf: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   reg_k: torch.Tensor | None, reg_pos: torch.Tensor | None, R: int,
                   position: torch.Tensor, n_sink: int, window: int, inv_freq: torch.Tensor | None,
                   q: torch.Tensor, scale: float, out: torch.Tensor, ws: Workspace,
                   mask: torch.Tensor | None = None) -> torch.Tensor:
    """Ring-buffer layer decode step (cache_v2.py:167-181) fused with its attention over the
    window + 1 + R rows: place as v2_place, then split-K decode attention."""
    kv = kv_desc(kbuf, vbuf)
    b, h, _, d = kbuf.shape
    rows = window + 1 + R
    need = workspace_bytes(OP_ATTEND, b, h, q.shape[1], d, kbuf.dtype, vbuf.dtype, rows, 0, 1, 0,
                           sm_count(kbuf.device))
    buf = ws.get(need, kbuf.device)
    rk, rp, inv, rot_half = _region_args(reg_k, reg_pos, R, inv_freq)
    mptr, msb, _keep = mask_arg(mask, b, rows)
    rc = lib().sink_v2_decode_step(
        ctypes.byref(kv), ctypes.byref(rows_desc(k)), ctypes.byref(rows_desc(v)), rk, rp, int(R),
        _position_arg(position), int(n_sink), int(window), inv, int(rot_half), ctypes.byref(rows_desc(q)),
        float(scale), mptr, msb, out.data_ptr(), out.stride(0), out.stride(2), buf.data_ptr(), buf.numel(),
        stream_handle(kbuf.device))
    _check(rc, "sink_v2_decode_step")
    return out


def v2_gather(kbuf: torch.Tensor, vbuf: torch.Tensor, n_sink: int, window: int, R: int, lo: int, hi: int,
              k: torch.Tensor | None, v: torch.Tensor | None, out_k: torch.Tensor, out_v: torch.Tensor) -> None:
    """[region, window by position, chunk] rows of a ring-buffer layer into out_k / out_v:
    out_v rows [0, R) from the region's values (out_k's are the place kernel's), rows
    [R, R + hi - lo) from the ring slots of positions lo .. hi - 1, then the chunk (k, v)."""
    kv = kv_desc(kbuf, vbuf)
    kd = ctypes.byref(rows_desc(k)) if k is not None else None
    vd = ctypes.byref(rows_desc(v)) if v is not None else None
    rc = lib().sink_v2_gather(ctypes.byref(kv), int(n_sink), int(window), int(R), int(lo), int(hi), kd, vd,
                              ctypes.byref(rows_desc(out_k)), ctypes.byref(rows_desc(out_v)),
                              stream_handle(kbuf.device))
    _check(rc, "sink_v2_gather")
