"""CPU oracle for the paged-decode path. TEST INFRASTRUCTURE -- never the product.

Only ``tests/``, ``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference``
legs of ``bench.py`` import this module; the shipped path (``llm-serving_b200/``) has no CPU
fallback and never calls it.

Two independent restatements of the reference (paths relative to the reference root):

* the C library ``pd_oracle.c`` (built by :func:`build` with gcc into ``oracle/_build``):
  ``reference_paged_decode`` (tests/reference/paged.py:225-274), ``write_slots`` /
  ``write_token_reference`` (model/paged.py:188-239, tests/reference/paged.py:93-124),
  ``gather_pool`` (tests/reference/paged.py:40-90), the seat decode
  (model/attention/hand_baddbmm.py:80-126) and the split-KV partial / LSE merge algebra of
  the decode kernel's online softmax (model/triton_decode.py:576-639);
* pure-Python per-token loops in float64 (:func:`dense_decode_py`, :func:`slot_of`),
  written like the reference's second oracle ``_dense_oracle``
  (tests/unit/test_triton_decode.py:75-105), for small cases only.

Both are pinned against golden vectors produced by the reference's own functions
(``tests/golden/make_golden.py``). Tensor arguments are CPU torch tensors; bf16/fp16 data is
passed as raw 16-bit patterns.
"""

from __future__ import annotations

import ctypes
import math
import subprocess
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
SOURCE = HERE / "pd_oracle.c"
LIB = HERE / "_build" / "libpd_oracle.so"

_DT = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def build(force: bool = False) -> Path:
    """Compile ``pd_oracle.c`` with gcc (OpenMP) if the .so is missing or stale."""
    LIB.parent.mkdir(exist_ok=True)
    if force or not LIB.exists() or LIB.stat().st_mtime < SOURCE.stat().st_mtime:
        cmd = ["gcc", "-O3", "-ffp-contract=off", "-fopenmp", "-fPIC", "-shared", "-std=c11", str(SOURCE),
               "-o", str(LIB), "-lm"]
        subprocess.run(cmd, check=True)
    return LIB


_lib = None


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        path = build()
        _lib = ctypes.CDLL(str(path))
        P, I, I64, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
        _lib.oracle_paged_decode.argtypes = [P, P, P, P, P, I64, I, P, I64, I, P, I, I, I, I, I, F, P, P, I]
        _lib.oracle_paged_decode.restype = I
        _lib.oracle_decode_partials.argtypes = [P, P, P, P, P, I64, I, P, I64, P, P, P, I, I, I, I, I, F, P, P, P, I]
        _lib.oracle_decode_partials.restype = I
        _lib.oracle_lse_merge.argtypes = [P, P, P, I, I, I, I, I, P, P]
        _lib.oracle_lse_merge.restype = None
        _lib.oracle_append_slots.argtypes = [P, P, P, P, I64, I, I, P, P, P, P, P, I, I64, I, I]
        _lib.oracle_append_slots.restype = I64
        _lib.oracle_append_table.argtypes = [P, P, P, P, I64, I, I, P, I64, I, P, P, P, P, P, I, I, I, I]
        _lib.oracle_append_table.restype = I64
        _lib.oracle_gather_pool.argtypes = [P, P, P, P, I64, I, P, I64, I, P, I, I, I, I, I, P, P, I]
        _lib.oracle_gather_pool.restype = I
        _lib.oracle_seat_decode.argtypes = [P, P, P, P, I, I, I, I, I, I, P, I]
        _lib.oracle_seat_decode.restype = None
        _lib.oracle_convert.argtypes = [P, I, P, I, I64]
        _lib.oracle_rope.restype = None
        _lib.oracle_rope.argtypes = [P, P, P, P, I64, I, I, I64, I64, I]
        _lib.oracle_convert.restype = None
        _lib.oracle_max_threads.argtypes = []
        _lib.oracle_max_threads.restype = I
    return _lib


def _cpu(t: torch.Tensor) -> torch.Tensor:
    return t.detach().cpu()


def _strides(t: torch.Tensor):
    return (ctypes.c_int64 * 3)(*[int(s) for s in t.stride()[:3]])


def max_threads() -> int:
    return int(lib().oracle_max_threads())


def paged_decode(q, k, v, table, seqlen, *, scale: float | None = None, threads: int = 0):
    """``reference_paged_decode`` on the CPU: returns ``(out_f32, out)`` (fp32 and q dtype)."""
    q, k, v = _cpu(q).contiguous(), _cpu(k), _cpu(v)
    table = _cpu(table).to(torch.int32).contiguous()
    seqlen = _cpu(seqlen).to(torch.int32).contiguous()
    if k.stride(-1) != 1:
        k = k.contiguous()
    if v.stride(-1) != 1:
        v = v.contiguous()
    B, H, D = q.shape
    n_blocks, bs, hkv, _ = k.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out_f32 = torch.empty(B, H, D, dtype=torch.float32)
    out = torch.empty(B, H, D, dtype=q.dtype)
    status = lib().oracle_paged_decode(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), _strides(k), _strides(v), n_blocks, bs,
        table.data_ptr(), table.stride(0), table.shape[1], seqlen.data_ptr(), B, H, hkv, D,
        _DT[q.dtype], float(scale), out_f32.data_ptr(), out.data_ptr(), threads,
    )
    if status != 0:
        raise ValueError("oracle_paged_decode: seqlen beyond the table or block id outside the pool")
    return out_f32, out


def decode_partials(q, k, v, table, seqlen, *, tok_begin=None, tok_end=None, scale: float | None = None,
                    threads: int = 0):
    """Split-KV triple ``(m, l, acc)`` over ``[tok_begin, tok_end)`` of each row (log2 domain)."""
    q, k, v = _cpu(q).contiguous(), _cpu(k), _cpu(v)
    table = _cpu(table).to(torch.int32).contiguous()
    seqlen = _cpu(seqlen).to(torch.int32).contiguous()
    B, H, D = q.shape
    n_blocks, bs, hkv, _ = k.shape
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    tb = None if tok_begin is None else _cpu(tok_begin).to(torch.int32).contiguous()
    te = None if tok_end is None else _cpu(tok_end).to(torch.int32).contiguous()
    m = torch.empty(B, H)
    l = torch.empty(B, H)
    acc = torch.empty(B, H, D)
    status = lib().oracle_decode_partials(
        q.data_ptr(), k.data_ptr(), v.data_ptr(), _strides(k), _strides(v), n_blocks, bs,
        table.data_ptr(), table.stride(0), seqlen.data_ptr(),
        None if tb is None else tb.data_ptr(), None if te is None else te.data_ptr(),
        B, H, hkv, D, _DT[q.dtype], float(scale) * 1.4426950408889634, m.data_ptr(), l.data_ptr(),
        acc.data_ptr(), threads,
    )
    if status != 0:
        raise ValueError("oracle_decode_partials: block id outside the pool")
    return m, l, acc


def lse_merge(m, l, acc, dtype=torch.float32):
    """Merge ``(n_parts, B, H[, D])`` triples; returns ``(out_f32, out)``."""
    m, l, acc = _cpu(m).float().contiguous(), _cpu(l).float().contiguous(), _cpu(acc).float().contiguous()
    n_parts, B, H, D = acc.shape
    out_f32 = torch.empty(B, H, D)
    out = torch.empty(B, H, D, dtype=dtype)
    lib().oracle_lse_merge(m.data_ptr(), l.data_ptr(), acc.data_ptr(), n_parts, B, H, D, _DT[dtype],
                           out_f32.data_ptr(), out.data_ptr())
    return out_f32, out


def append_slots(k_pool, v_pool, slots, k, v) -> int:
    """In place on CPU pools; returns the number of skipped (out-of-pool) tokens."""
    slots = _cpu(slots).to(torch.int64).contiguous()
    n_blocks, bs, hkv, D = k_pool.shape
    return int(lib().oracle_append_slots(
        k_pool.data_ptr(), v_pool.data_ptr(), _strides(k_pool), _strides(v_pool), n_blocks, bs,
        _DT[k_pool.dtype], slots.data_ptr(), k.data_ptr(), _strides(k), v.data_ptr(), _strides(v),
        _DT[k.dtype], k.shape[0], hkv, D,
    ))


def append_table(k_pool, v_pool, table, pos, k, v) -> int:
    table = _cpu(table).to(torch.int32).contiguous()
    pos = _cpu(pos).to(torch.int64).contiguous()
    n_blocks, bs, hkv, D = k_pool.shape
    return int(lib().oracle_append_table(
        k_pool.data_ptr(), v_pool.data_ptr(), _strides(k_pool), _strides(v_pool), n_blocks, bs,
        _DT[k_pool.dtype], table.data_ptr(), table.stride(0), table.shape[1], pos.data_ptr(),
        k.data_ptr(), _strides(k), v.data_ptr(), _strides(v), _DT[k.dtype], k.shape[0], hkv, D,
    ))


def gather_pool(k, v, table, lengths, lpad: int, *, threads: int = 0):
    """Dense zero-padded ``(B, H_kv, lpad, D)`` K/V of each row's first ``lengths`` tokens."""
    k, v = _cpu(k), _cpu(v)
    table = _cpu(table).to(torch.int32).contiguous()
    lengths = _cpu(lengths).to(torch.int32).contiguous()
    n_blocks, bs, hkv, D = k.shape
    B = lengths.shape[0]
    out_k = torch.empty(B, hkv, lpad, D, dtype=k.dtype)
    out_v = torch.empty_like(out_k)
    status = lib().oracle_gather_pool(
        k.data_ptr(), v.data_ptr(), _strides(k), _strides(v), n_blocks, bs, table.data_ptr(),
        table.stride(0), table.shape[1], lengths.data_ptr(), B, hkv, D, _DT[k.dtype], lpad,
        out_k.data_ptr(), out_v.data_ptr(), threads,
    )
    if status != 0:
        raise ValueError("oracle_gather_pool: length beyond lpad/table or block id outside the pool")
    return out_k, out_v


def seat_decode(q, slab_k, slab_v, lengths, *, threads: int = 0):
    """Seat (``hand_baddbmm``) decode over dense slabs; output in the q dtype."""
    q = _cpu(q).contiguous()
    slab_k, slab_v = _cpu(slab_k).contiguous(), _cpu(slab_v).contiguous()
    lengths = _cpu(lengths).to(torch.int32).contiguous()
    B, H, D = q.shape
    _, hkv, lpad, _ = slab_k.shape
    out = torch.empty(B, H, D, dtype=q.dtype)
    lib().oracle_seat_decode(q.data_ptr(), slab_k.data_ptr(), slab_v.data_ptr(), lengths.data_ptr(), B, H, hkv,
                             D, lpad, _DT[q.dtype], out.data_ptr(), threads)
    return out


def rope(x, cos, sin, rotary_dim: int) -> torch.Tensor:
    """GPT-NeoX rotary embedding (model/layers.py:59-117 ``apply_rotary_emb_partial``) of
    ``x`` (..., n_head, head_dim) with one cos/sin row per leading index: cos/sin shaped
    (..., rotary_dim / 2) matching ``x``'s leading dims without the head axis."""
    x = _cpu(x).contiguous()
    cos = _cpu(cos).contiguous().to(x.dtype)
    sin = _cpu(sin).contiguous().to(x.dtype)
    head_dim, n_head = x.shape[-1], x.shape[-2]
    n_rows = x.numel() // head_dim
    out = torch.empty_like(x)
    lib().oracle_rope(x.data_ptr(), cos.data_ptr(), sin.data_ptr(), out.data_ptr(), n_rows, head_dim,
                      int(rotary_dim), rotary_dim // 2, n_head, _DT[x.dtype])
    return out


def convert(x: torch.Tensor, dtype: torch.dtype) -> torch.Tensor:
    """The oracle's element conversion (round to nearest even), for pinning against torch."""
    x = _cpu(x).contiguous()
    out = torch.empty(x.shape, dtype=dtype)
    lib().oracle_convert(x.data_ptr(), _DT[x.dtype], out.data_ptr(), _DT[dtype], x.numel())
    return out


# ------------------------------------------------------------------ pure-Python restatements


def slot_of(block_table, position: int, block_size: int) -> int:
    """Flat pool slot of a logical position (model/paged.py:150-168): table[pos // bs] * bs + pos % bs."""
    return block_table[position // block_size] * block_size + position % block_size


def dense_decode_py(q, k, v, table, seqlen, scale: float | None = None):
    """Per-token float64 decode with plain indexing; small cases only.

    Every logical token is looked up through the block table one at a time, so a wrong
    page/offset mapping cannot agree with the C oracle or the kernel by accident.
    """
    q, k, v = _cpu(q), _cpu(k), _cpu(v)
    B, H, D = q.shape
    bs, hkv = k.shape[1], k.shape[2]
    group = H // hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = torch.zeros(B, H, D, dtype=torch.float64)
    for row in range(B):
        n = int(seqlen[row])
        if n <= 0:
            continue
        keys = torch.stack([k[int(table[row, t // bs]), t % bs] for t in range(n)]).double()
        vals = torch.stack([v[int(table[row, t // bs]), t % bs] for t in range(n)]).double()
        for head in range(H):
            hk = head // group
            scores = (q[row, head].double() @ keys[:, hk, :].T) * scale
            probs = torch.softmax(scores, dim=-1)
            out[row, head] = probs @ vals[:, hk, :]
    return out


def paged_prefill(q, k, v, table, cu_seqlens_q, seqlen_k, *, scale: float | None = None):
    """Chunked-prefill attention over the paged pool, float64 on the CPU: returns
    ``(out_f32, out)`` (fp32 and q dtype), ``q``/``out`` packed ``(total_q, H, D)``.

    Row ``b``'s query tokens ``q[cu[b]:cu[b+1]]`` (``Sq`` of them) sit at positions
    ``seqlen_k[b] - Sq + i`` and attend causally (bottom-right aligned, the varlen causal
    convention of the reference's prefill kernel, flash_attn 2.8.3 ``flash_attn_varlen_func``
    with ``causal=True``, model/varlen.py:20) to the row's keys, gathered token by token
    through the block table as :func:`dense_decode_py` does (tests/reference/paged.py:225-274
    for one query token). A query with no visible key gives zeros.
    """
    q, k, v = _cpu(q), _cpu(k), _cpu(v)
    table, cu, sk = _cpu(table), _cpu(cu_seqlens_q), _cpu(seqlen_k)
    T, H, D = q.shape
    bs, hkv = k.shape[1], k.shape[2]
    group = H // hkv
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    out = torch.zeros(T, H, D, dtype=torch.float64)
    for row in range(sk.shape[0]):
        q0, q1, n = int(cu[row]), int(cu[row + 1]), int(sk[row])
        sq = q1 - q0
        if sq <= 0 or n <= 0:
            continue
        idx = torch.tensor([int(table[row, t // bs]) for t in range(n)])
        off = torch.arange(n) % bs
        keys = k[idx, off].double()  # (n, hkv, D)
        vals = v[idx, off].double()
        pos = torch.arange(sq) + (n - sq)            # absolute query positions
        visible = torch.arange(n)[None, :] <= pos[:, None]  # (sq, n)
        for head in range(H):
            hk = head // group
            scores = (q[q0:q1, head].double() @ keys[:, hk, :].T) * scale
            scores = scores.masked_fill(~visible, float("-inf"))
            probs = torch.softmax(scores, dim=-1)
            probs = torch.nan_to_num(probs, nan=0.0)  # rows with no visible key
            out[q0:q1, head] = probs @ vals[:, hk, :]
    return out.float(), out.to(q.dtype)
