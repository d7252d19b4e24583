"""ctypes binding of ``libpaged_decode.so`` -- the C ABI declared in ``include/paged_decode.h``.

This module is the only place Python touches the native library. It loads the .so built by
``llm-serving_b200/build.py`` (never a JIT cache), declares every entry point's signature,
and offers thin typed helpers that pass ``tensor.data_ptr()`` values, element strides and
the current torch stream. There is no Python or CPU implementation of any kernel here: if
the library cannot be loaded, :data:`AVAILABLE` is False and every caller raises.
"""

from __future__ import annotations

import ctypes
import math
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().parent.parent / "libpaged_decode.so"

PD_OK = 0
PD_ERR_INVALID = 1
PD_ERR_UNSUPPORTED = 2
PD_ERR_CUDA = 3
PD_ERR_WORKSPACE = 4

PD_F32, PD_F16, PD_BF16 = 0, 1, 2
PD_SLOT_I32, PD_SLOT_I64 = 0, 1
DEVERR_WAIT_TIMEOUT = 1
DEVERR_APPEND_RANGE = 2

_DTYPES = {torch.float32: PD_F32, torch.float16: PD_F16, torch.bfloat16: PD_BF16}

_c_i32 = ctypes.c_int32
_c_i64 = ctypes.c_int64
_c_ptr = ctypes.c_void_p
_c_i64p = ctypes.POINTER(ctypes.c_int64)
_c_size = ctypes.c_size_t
_c_float = ctypes.c_float

_SIGNATURES = {
    "pd_status_string": (ctypes.c_char_p, [ctypes.c_int]),
    "pd_abi_version": (ctypes.c_int, []),
    "pd_launch_count": (ctypes.c_uint64, []),
    "pd_last_error_string": (ctypes.c_char_p, []),
    "pd_device_error": (ctypes.c_int, [ctypes.POINTER(ctypes.c_uint), ctypes.c_int]),
    "pd_decode_workspace_bytes": (_c_size, [_c_i32, _c_i32, _c_i32, _c_i32, _c_i32]),
    "pd_decode": (
        ctypes.c_int,
        [_c_ptr, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_i64, _c_i32, _c_i64p, _c_i64p, _c_ptr, _c_i64,
         _c_i32, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_float,
         _c_ptr, _c_size, _c_ptr],
    ),
    "pd_prefill": (
        ctypes.c_int,
        [_c_ptr, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_i64, _c_i32, _c_i64p, _c_i64p, _c_ptr, _c_i64,
         _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
         _c_i32, _c_float, _c_ptr],
    ),
    "pd_decode_noalloc": (
        ctypes.c_int,
        [_c_ptr, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_i64, _c_i32, _c_i64p, _c_i64p, _c_ptr, _c_i64,
         _c_i32, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32, _c_float,
         _c_ptr],
    ),
    "pd_decode_partials": (
        ctypes.c_int,
        [_c_ptr, _c_i64, _c_i64, _c_ptr, _c_ptr, _c_i64, _c_i32, _c_i64p, _c_i64p, _c_ptr, _c_i64,
         _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_ptr, _c_i32, _c_i32, _c_i32, _c_i32, _c_i32,
         _c_float, _c_ptr, _c_size, _c_ptr],
    ),
    "pd_lse_merge": (
        ctypes.c_int,
        [_c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_i32, _c_i32, _c_i32, _c_i32, _c_ptr, _c_i64,
         _c_i64, _c_i32, _c_ptr],
    ),
    "pd_plan_create": (
        ctypes.c_int,
        [ctypes.POINTER(_c_ptr), _c_i32, ctypes.POINTER(_c_ptr), ctypes.POINTER(_c_ptr), _c_i64,
         _c_i32, _c_i64p, _c_i64p, _c_ptr, _c_i64, _c_i32, _c_ptr, _c_i32, _c_i32, _c_i32, _c_i32,
         _c_i32, _c_float, _c_ptr, _c_size],
    ),
    "pd_plan_run": (ctypes.c_int, [_c_ptr, _c_i32, _c_ptr, _c_ptr, _c_ptr]),
    "pd_plan_run_append": (
        ctypes.c_int,
        [_c_ptr, _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_ptr, _c_i64, _c_i64, _c_ptr, _c_ptr],
    ),
    "pd_plan_run_append_rope": (
        ctypes.c_int,
        [_c_ptr, _c_i32, _c_ptr, _c_ptr, _c_ptr, _c_i64, _c_i64, _c_ptr, _c_i64, _c_i64, _c_ptr, _c_ptr,
         _c_ptr, _c_i64, _c_i32, _c_ptr],
    ),
    "pd_plan_destroy": (None, [_c_ptr]),
    "pd_plan_set_overlap": (ctypes.c_int, [_c_ptr, _c_i32]),
    "pd_plan_set_static_table": (ctypes.c_int, [_c_ptr, _c_i32]),
    "pd_kv_append_slots": (
        ctypes.c_int,
        [_c_ptr, _c_ptr, _c_i64, _c_i32, _c_i64p, _c_i64p, _c_i32, _c_ptr, _c_i32, _c_ptr, _c_i64p,
         _c_ptr, _c_i64p, _c_i32, _c_i64, _c_i32, _c_i32, _c_ptr],
    ),
    "pd_kv_append_table": (
        ctypes.c_int,
        [_c_ptr, _c_ptr, _c_i64, _c_i32, _c_i64p, _c_i64p, _c_i32, _c_ptr, _c_i64, _c_i32, _c_ptr,
         _c_ptr, _c_i64p, _c_ptr, _c_i64p, _c_i32, _c_i32, _c_i32, _c_i32, _c_ptr],
    ),
    "pd_kv_append_table_rope": (
        ctypes.c_int,
        [_c_ptr, _c_ptr, _c_i64, _c_i32, _c_i64p, _c_i64p, _c_i32, _c_ptr, _c_i64, _c_i32, _c_ptr,
         _c_ptr, _c_i64p, _c_ptr, _c_i64p, _c_i32, _c_i32, _c_i32, _c_i32, _c_ptr, _c_ptr, _c_i64, _c_i32,
         _c_ptr],
    ),
    "pd_set_decode_tuning": (ctypes.c_int, [_c_i32, _c_i32, _c_i32, _c_i32]),
    "pd_get_decode_tuning": (ctypes.c_int, [ctypes.POINTER(_c_i32)] * 4),
    "pd_set_decode_mode": (ctypes.c_int, [_c_i32, _c_i32, _c_i32]),
    "pd_get_decode_mode": (ctypes.c_int, [ctypes.POINTER(_c_i32)] * 3),
    "pd_set_prefill_mode": (ctypes.c_int, [_c_i32]),
    "pd_get_prefill_mode": (ctypes.c_int, []),
    "pd_set_wait_limit": (ctypes.c_int, [ctypes.c_uint64]),
    "pd_get_wait_limit": (ctypes.c_uint64, []),
}

#: Names exported by the library (the header's entry points); tests check all resolve.
EXPORTS = tuple(_SIGNATURES)


def _load():
    if not LIB_PATH.exists():
        return None, f"{LIB_PATH} is missing; run `python llm-serving_b200/build.py`"
    try:
        lib = ctypes.CDLL(str(LIB_PATH))
    except OSError as exc:  # pragma: no cover - depends on the host
        return None, f"could not load {LIB_PATH}: {exc}"
    for name, (restype, argtypes) in _SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    return lib, None


lib, LOAD_ERROR = _load()
#: True when the native library loaded (says nothing about a GPU being present).
AVAILABLE: bool = lib is not None


def require() -> ctypes.CDLL:
    if lib is None:
        raise RuntimeError(f"the sm_100a paged-decode library is not available: {LOAD_ERROR}")
    return lib


def dtype_code(dtype: torch.dtype) -> int:
    try:
        return _DTYPES[dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {dtype}") from None


def status_string(status: int) -> str:
    return require().pd_status_string(status).decode()


def check(status: int, what: str) -> None:
    """Raise on a non-zero status. Argument/shape problems are ValueError, CUDA failures
    RuntimeError -- the same split the reference wrapper uses."""
    if status == PD_OK:
        return
    message = f"{what} failed: {status_string(status)} (status {status})"
    if status in (PD_ERR_INVALID, PD_ERR_UNSUPPORTED, PD_ERR_WORKSPACE):
        raise ValueError(message)
    detail = require().pd_last_error_string().decode()
    raise RuntimeError(f"{message}: {detail}" if detail else message)


def stream_handle(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def strides3(t: torch.Tensor):
    """The (dim0, dim1, dim2) element strides of a 4-D pool or 3-D row tensor as int64[3]."""
    s = t.stride()
    return (_c_i64 * 3)(*(int(x) for x in s[:3]))


def launch_count() -> int:
    """Kernels this library launched in this process so far."""
    return int(require().pd_launch_count())


def log2e_scale(scale: float) -> float:
    return float(scale) * 1.4426950408889634


def workspace_bytes(batch: int, n_head: int, n_kv_head: int, head_dim: int, dtype: torch.dtype) -> int:
    return int(require().pd_decode_workspace_bytes(batch, n_head, n_kv_head, head_dim, dtype_code(dtype)))


def device_error(clear: bool = True) -> int:
    """Device error word of the current device (synchronises). 0 means no problem recorded."""
    bits = ctypes.c_uint(0)
    check(require().pd_device_error(ctypes.byref(bits), int(bool(clear))), "pd_device_error")
    return int(bits.value)


def set_decode_tuning(warps: int = 0, stages: int = 0, ctas_per_sm: int = 0, min_tiles: int = 0) -> None:
    check(require().pd_set_decode_tuning(warps, stages, ctas_per_sm, min_tiles), "pd_set_decode_tuning")


def get_decode_tuning() -> tuple[int, int, int, int]:
    vals = [_c_i32(0) for _ in range(4)]
    check(require().pd_get_decode_tuning(*[ctypes.byref(v) for v in vals]), "pd_get_decode_tuning")
    return tuple(int(v.value) for v in vals)


def set_decode_mode(mode: int, shared_stages: int = 0, row_cost: int = -1) -> None:
    """0: per-warp kernel, tensor-core tile math where it applies (default); 1: shared-stage
    kernel where it applies; 2: per-warp kernel with CUDA-core tile math everywhere.
    row_cost: extra columns charged per row start by the column split (-1 keeps it)."""
    check(require().pd_set_decode_mode(int(mode), int(shared_stages), int(row_cost)), "pd_set_decode_mode")


def get_decode_mode() -> tuple[int, int, int]:
    vals = [_c_i32(0) for _ in range(3)]
    check(require().pd_get_decode_mode(*[ctypes.byref(v) for v in vals]), "pd_get_decode_mode")
    return tuple(int(v.value) for v in vals)


def set_prefill_mode(mode: int) -> None:
    """0: tcgen05 / TMEM prefill kernel (default); 1: mma.sync prefill kernel."""
    check(require().pd_set_prefill_mode(int(mode)), "pd_set_prefill_mode")


def get_prefill_mode() -> int:
    return int(require().pd_get_prefill_mode())


def set_wait_limit(limit_ns: int) -> None:
    """Limit of the kernels' stage and arrival-counter waits for later launches (0: the 1 s
    default). A wait that runs out sets DEVERR_WAIT_TIMEOUT and the launch returns."""
    check(require().pd_set_wait_limit(int(limit_ns)), "pd_set_wait_limit")


def get_wait_limit() -> int:
    return int(require().pd_get_wait_limit())


def decode(q, k_cache, v_cache, block_table, seqlen, out, scale_log2, workspace) -> None:
    """One pd_decode launch on the current stream. Tensors are already validated."""
    B, H, D = q.shape
    _, bs, hkv, _ = k_cache.shape
    status = require().pd_decode(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0], bs,
        strides3(k_cache), strides3(v_cache),
        block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
        seqlen.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
        B, H, hkv, D, dtype_code(q.dtype), float(scale_log2),
        workspace.data_ptr(), workspace.numel(), stream_handle(q.device),
    )
    check(status, "pd_decode")


def prefill(q, k_cache, v_cache, block_table, cu_seqlens_q, seqlen_k, max_seqlen_q, out, n_head,
            scale_log2) -> None:
    """One pd_prefill launch on the current stream. Tensors are already validated: q/out are
    packed (total_q, H, D); cu_seqlens_q (B + 1) and seqlen_k (B) int32."""
    _, bs, hkv, D = k_cache.shape
    B = seqlen_k.shape[0]
    status = require().pd_prefill(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0], bs,
        strides3(k_cache), strides3(v_cache),
        block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
        cu_seqlens_q.data_ptr(), seqlen_k.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
        B, int(max_seqlen_q), int(n_head), hkv, D, dtype_code(q.dtype), float(scale_log2),
        stream_handle(q.device),
    )
    check(status, "pd_prefill")


def decode_noalloc(q, k_cache, v_cache, block_table, seqlen, out, scale_log2) -> None:
    """pd_decode without a workspace: the library's built-in scratch array is used, and the
    call allocates nothing (for hosts that cannot allocate device memory). Calls on one device
    share that array, so keep them ordered on one stream."""
    B, H, D = q.shape
    _, bs, hkv, _ = k_cache.shape
    status = require().pd_decode_noalloc(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0], bs,
        strides3(k_cache), strides3(v_cache),
        block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
        seqlen.data_ptr(), out.data_ptr(), out.stride(0), out.stride(1),
        B, H, hkv, D, dtype_code(q.dtype), float(scale_log2), stream_handle(q.device),
    )
    if status == PD_ERR_WORKSPACE:
        raise ValueError(f"pd_decode_noalloc failed: {require().pd_last_error_string().decode()}")
    check(status, "pd_decode_noalloc")


def decode_partials(q, k_cache, v_cache, block_table, seqlen, m_out, l_out, acc_out, scale_log2,
                    workspace) -> None:
    B, H, D = q.shape
    _, bs, hkv, _ = k_cache.shape
    status = require().pd_decode_partials(
        q.data_ptr(), q.stride(0), q.stride(1),
        k_cache.data_ptr(), v_cache.data_ptr(), k_cache.shape[0], bs,
        strides3(k_cache), strides3(v_cache),
        block_table.data_ptr(), block_table.stride(0), block_table.shape[1],
        seqlen.data_ptr(), m_out.data_ptr(), l_out.data_ptr(), acc_out.data_ptr(),
        B, H, hkv, D, dtype_code(q.dtype), float(scale_log2),
        workspace.data_ptr(), workspace.numel(), stream_handle(q.device),
    )
    check(status, "pd_decode_partials")


def lse_merge(m_parts, l_parts, acc_parts, out) -> None:
    """Merge parts: m/l ``(n_parts, B, H)`` and acc ``(n_parts, B, H, D)``, each part
    contiguous (the part axis may be strided, e.g. slices of one gathered buffer)."""
    n_parts, B, H, D = acc_parts.shape
    if m_parts.stride(0) != l_parts.stride(0):
        raise ValueError("m and l parts must share one part stride")
    status = require().pd_lse_merge(
        m_parts.data_ptr(), l_parts.data_ptr(), acc_parts.data_ptr(), m_parts.stride(0),
        acc_parts.stride(0), n_parts, B, H, D, out.data_ptr(), out.stride(0), out.stride(1),
        dtype_code(out.dtype), stream_handle(out.device),
    )
    check(status, "pd_lse_merge")


def append_slots(k_pool, v_pool, slot_ids, k, v) -> None:
    n_blocks, bs, hkv, D = k_pool.shape
    status = require().pd_kv_append_slots(
        k_pool.data_ptr(), v_pool.data_ptr(), n_blocks, bs, strides3(k_pool), strides3(v_pool),
        dtype_code(k_pool.dtype), slot_ids.data_ptr(),
        PD_SLOT_I64 if slot_ids.dtype == torch.int64 else PD_SLOT_I32,
        k.data_ptr(), strides3(k), v.data_ptr(), strides3(v), dtype_code(k.dtype),
        k.shape[0], hkv, D, stream_handle(k_pool.device),
    )
    check(status, "pd_kv_append_slots")


def append_table(k_pool, v_pool, block_table, pos, k, v, rope=None) -> None:
    """``rope`` = (cos, sin, rotary_dim): rotate the K rows first; cos/sin (B, rotary_dim / 2)
    with a unit last stride, in the pool dtype."""
    n_blocks, bs, hkv, D = k_pool.shape
    args = (
        k_pool.data_ptr(), v_pool.data_ptr(), n_blocks, bs, strides3(k_pool), strides3(v_pool),
        dtype_code(k_pool.dtype), block_table.data_ptr(), block_table.stride(0),
        block_table.shape[1], pos.data_ptr(), k.data_ptr(), strides3(k), v.data_ptr(), strides3(v),
        dtype_code(k.dtype), k.shape[0], hkv, D,
    )
    if rope is None:
        check(require().pd_kv_append_table(*args, stream_handle(k_pool.device)), "pd_kv_append_table")
        return
    cos, sin, rotary_dim = rope
    status = require().pd_kv_append_table_rope(*args, cos.data_ptr(), sin.data_ptr(), cos.stride(0),
                                               int(rotary_dim), stream_handle(k_pool.device))
    check(status, "pd_kv_append_table_rope")


class NativePlan:
    """Owner of one ``pd_plan`` handle (host memory); destroyed with the object."""

    __slots__ = ("_handle", "_lib", "_overlap", "__weakref__")

    def __init__(self, k_caches, v_caches, block_table, seqlen, batch, n_head, scale_log2,
                 workspace) -> None:
        lib_ = require()
        k0 = k_caches[0]
        n_blocks, bs, hkv, D = k0.shape
        n = len(k_caches)
        kptrs = (_c_ptr * n)(*[t.data_ptr() for t in k_caches])
        vptrs = (_c_ptr * n)(*[t.data_ptr() for t in v_caches])
        handle = _c_ptr(0)
        status = lib_.pd_plan_create(
            ctypes.byref(handle), n, kptrs, vptrs, n_blocks, bs, strides3(k0), strides3(v_caches[0]),
            block_table.data_ptr(), block_table.stride(0), block_table.shape[1], seqlen.data_ptr(),
            batch, n_head, hkv, D, dtype_code(k0.dtype), float(scale_log2),
            workspace.data_ptr(), workspace.numel(),
        )
        check(status, "pd_plan_create")
        self._handle = handle
        self._lib = lib_
        self._overlap = False

    def _set_overlap(self, overlap: bool) -> None:
        if bool(overlap) != self._overlap:
            check(self._lib.pd_plan_set_overlap(self._handle, int(bool(overlap))), "pd_plan_set_overlap")
            self._overlap = bool(overlap)

    def set_static_table(self, fixed: bool) -> None:
        """The block table keeps its contents for the plan's lifetime: the step cache may keep
        table windows too (pd_plan_set_static_table)."""
        check(self._lib.pd_plan_set_static_table(self._handle, int(bool(fixed))), "pd_plan_set_static_table")

    def run(self, layer: int, q, out, stream: int, overlap: bool = False) -> None:
        """``overlap``: the launch may start before the previous kernel of the stream ends
        (pd_plan_set_overlap's contract: that kernel writes no seqlen, table or pool)."""
        self._set_overlap(overlap)
        status = self._lib.pd_plan_run(self._handle, layer, q.data_ptr(), out.data_ptr(), stream)
        if status:
            check(status, "pd_plan_run")

    def run_append(self, layer: int, q, out, k_new, v_new, pos, stream: int, rope=None,
                   overlap: bool = False) -> None:
        """Append ``k_new``/``v_new`` ``(B, H_kv, D)`` at ``pos`` (int64) and decode, one launch;
        ``rope`` = (cos, sin, rotary_dim) rotates ``k_new`` first (see :func:`append_table`)."""
        self._set_overlap(overlap)
        args = (self._handle, layer, q.data_ptr(), out.data_ptr(), k_new.data_ptr(), k_new.stride(0),
                k_new.stride(1), v_new.data_ptr(), v_new.stride(0), v_new.stride(1), pos.data_ptr())
        if rope is None:
            status = self._lib.pd_plan_run_append(*args, stream)
            name = "pd_plan_run_append"
        else:
            cos, sin, rotary_dim = rope
            status = self._lib.pd_plan_run_append_rope(*args, cos.data_ptr(), sin.data_ptr(), cos.stride(0),
                                                       int(rotary_dim), stream)
            name = "pd_plan_run_append_rope"
        if status:
            check(status, name)

    def __del__(self) -> None:
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            self._lib.pd_plan_destroy(handle)
            self._handle = None


def default_scale(head_dim: int) -> float:
    return 1.0 / math.sqrt(head_dim)
