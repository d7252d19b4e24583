"""Block-table decode on B200: the drop-in for the reference's ``model/triton_decode.py``.

The module keeps the reference's public surface so ``PagedKV.attend``, the engines and the
tests call it unchanged (reference: ``model/triton_decode.py:250-538``):

* ``paged_decode(q, k_cache, v_cache, block_table, seqlen, *, scale=None)`` -- validating
  one-shot entry point;
* ``paged_decode_plan(...)`` / ``PagedDecodePlan.run(layer, q)`` -- validate a container's
  pools once, then one launch per layer;
* ``TRITON_AVAILABLE`` -- kept under the reference's name for its callers; here it means
  "the sm_100a paged-decode library is loaded".

Contract (identical to the reference): ``q`` is ``(B, H, D)`` (copied if non-contiguous);
``k_cache``/``v_cache`` are ``(n_blocks, block_size, H_kv, D)`` with the q dtype (fp16, bf16
or fp32); ``block_table`` is int32 ``(B, max_blocks)`` on the same CUDA device and only its
first ``ceil(seqlen[b] / block_size)`` entries of row ``b`` are read; ``seqlen`` is ``(B,)``
int32 (int64 is cast) with values in ``[0, max_blocks * block_size]``; the output is
``(B, H, D)`` in ``q.dtype``; ``scale=None`` means ``1 / sqrt(D)``. There is no CPU path and
no fallback: without the library or CUDA every entry point raises ``RuntimeError``.

What runs underneath is the C ABI of ``include/paged_decode.h`` (``pd_decode`` and
``pd_plan_*``): a TMA-fed, warp-pipelined sm_100a kernel that balances KV pages over every SM
and merges split rows in the same launch. Differences from the reference that a caller can
observe: ``head_dim`` must be in 8..256 (a power of two, as before); pool strides must be
16-byte multiples with a unit ``head_dim`` stride -- ``paged_decode`` copies a pool that is
not, ``paged_decode_plan`` refuses it; and a table entry outside the pool reads zeros
instead of faulting.
"""

from __future__ import annotations

import math

import torch

from model import _native

TRITON_AVAILABLE: bool = _native.AVAILABLE

__all__ = ["TRITON_AVAILABLE", "paged_decode", "paged_decode_plan", "PagedDecodePlan"]

_LOG2E = 1.4426950408889634
_MIN_HEAD_DIM = 8
_MAX_HEAD_DIM = 256

#: Last successful seqlen range check: ``(seqlen, version, capacity)``. Holding the tensor
#: keeps its storage alive, so the identity test cannot alias a freed tensor. The check is
#: the one host synchronisation of the wrapper; a persistent seqlen pays it once per version.
_SEQ_CHECK: tuple[torch.Tensor, int, int] | None = None

#: Per (device, stream) decode workspace for ``paged_decode``. Its contents never need
#: clearing (split rows are counted with per-launch epochs); one per stream, so two streams
#: never share one.
_WORKSPACES: dict[tuple[int, int], torch.Tensor] = {}


def _require_backend() -> None:
    """No library or no CUDA is an environment problem: RuntimeError, never a fallback."""
    if not TRITON_AVAILABLE:
        raise RuntimeError(
            "paged_decode requires the sm_100a CUDA library that replaces the Triton kernel, "
            f"but it could not be loaded ({_native.LOAD_ERROR}); the paged decode arm has no "
            "eager fallback. The dense oracle lives in oracle/ and tests/."
        )
    if not torch.cuda.is_available():
        raise RuntimeError(
            "paged_decode requires CUDA, but torch.cuda is unavailable; the paged decode arm "
            "has no CPU fallback. The dense oracle lives in oracle/ and tests/."
        )


def _require_cuda_tensors(tensors) -> None:
    for name, tensor in tensors:
        if not tensor.is_cuda:
            raise RuntimeError(
                f"paged_decode requires CUDA tensors, got {name} on device {tensor.device}; "
                "there is no silent fallback to a dense implementation."
            )


def _contract(q, k_cache, v_cache, block_table, seqlen):
    """The kernel's layout contract as (violated, message) rules, in the order they are checked.

    The messages are the reference's (model/triton_decode.py:120-231), which its callers and
    tests match on. A rule may rely on every rule before it holding (shapes are unpacked only
    after their ranks are checked), so the rules are produced lazily and the caller stops at
    the first violation.
    """
    yield q.dim() != 3, lambda: f"q must be (B, H, D), got shape {tuple(q.shape)}"
    pools = (k_cache, v_cache)
    yield any(t.dim() != 4 for t in pools), lambda: (
        "k_cache/v_cache must be (n_blocks, block_size, H_kv, D), got "
        f"{tuple(k_cache.shape)} / {tuple(v_cache.shape)}")
    yield k_cache.shape != v_cache.shape, lambda: (
        f"k_cache/v_cache shapes differ: {tuple(k_cache.shape)} vs {tuple(v_cache.shape)}")
    yield q.dtype not in _DTYPES, lambda: f"q dtype must be fp16, bf16 or fp32, got {q.dtype}"
    yield any(t.dtype != q.dtype for t in pools), lambda: (
        f"q/k_cache/v_cache must share one dtype, got {q.dtype}, {k_cache.dtype}, {v_cache.dtype}")

    n_head, head_dim = q.shape[1], q.shape[2]
    block_size, n_kv, cache_d = k_cache.shape[1], k_cache.shape[2], k_cache.shape[3]
    yield head_dim < 1, lambda: f"head_dim must be positive, got {head_dim}"
    yield head_dim != cache_d, lambda: f"q head_dim {head_dim} != cache head_dim {cache_d}"
    yield n_kv < 1 or n_head % n_kv != 0, lambda: f"n_head ({n_head}) must be a multiple of n_kv_head ({n_kv})"
    yield block_size < 1, lambda: f"block_size must be positive, got {block_size}"
    yield not _pow2(block_size), lambda: (
        f"block_size must be a power of two (16 and 32 are the supported sizes), got {block_size}")
    yield not _pow2(head_dim), lambda: f"head_dim must be a power of two for the kernel, got {head_dim}"
    yield not _MIN_HEAD_DIM <= head_dim <= _MAX_HEAD_DIM, lambda: (
        f"head_dim {head_dim} is outside the sm_100a kernel's range {_MIN_HEAD_DIM}..{_MAX_HEAD_DIM}")

    batch = q.shape[0]
    yield block_table.dim() != 2, lambda: (
        f"block_table must be (B, max_blocks), got shape {tuple(block_table.shape)}")
    yield block_table.shape[0] != batch, lambda: (
        f"block_table batch {block_table.shape[0]} does not match q batch {batch}")
    yield block_table.dtype != torch.int32, lambda: (
        "paged_decode requires an int32 block_table (the kernel's indexing contract); "
        f"got {block_table.dtype}. Cast at the allocator boundary, not per step.")
    yield seqlen.dim() != 1, lambda: f"seqlen must be (B,), got shape {tuple(seqlen.shape)}"
    yield seqlen.shape[0] != batch, lambda: f"seqlen has {seqlen.shape[0]} entries for a batch of {batch}"
    yield seqlen.dtype not in (torch.int32, torch.int64), lambda: f"seqlen must be int32 or int64, got {seqlen.dtype}"
    for name, tensor in (("q", q), ("k_cache", k_cache), ("v_cache", v_cache),
                         ("block_table", block_table), ("seqlen", seqlen)):
        yield tensor.device != q.device, lambda name=name, tensor=tensor: (
            f"{name} is on {tensor.device} but q is on {q.device}; all paged_decode tensors "
            "must share one device")


_DTYPES = (torch.float16, torch.bfloat16, torch.float32)


def _pow2(n: int) -> bool:
    return n > 0 and n & (n - 1) == 0


def _validate(q, k_cache, v_cache, block_table, seqlen) -> None:
    """Raise ValueError for the first violated rule of the layout contract, then range-check
    seqlen against the table's capacity.

    The range check needs the lengths on the host, so it is skipped while the same seqlen
    tensor, unmodified since it last passed (same version counter; an inference tensor has
    none and keeps its first pass), meets the same capacity: an engine that updates seqlen in
    place once per step pays one host read per step, not one per layer.
    """
    _raise_first(_contract(q, k_cache, v_cache, block_table, seqlen))
    if q.shape[0] == 0:
        return
    global _SEQ_CHECK
    capacity = block_table.shape[1] * k_cache.shape[1]
    version = -1 if seqlen.is_inference() else int(seqlen._version)
    last = _SEQ_CHECK
    if last is not None and last[0] is seqlen and last[1:] == (version, capacity):
        return
    low, high = int(seqlen.min()), int(seqlen.max())
    if low < 0:
        raise ValueError(f"seqlen values must be >= 0, got {low}")
    if high > capacity:
        raise ValueError(
            f"seqlen {high} exceeds the block table capacity {capacity} "
            f"({block_table.shape[1]} blocks x {k_cache.shape[1]} tokens)"
        )
    _SEQ_CHECK = (seqlen, version, capacity)


def _raise_first(rules) -> None:
    """ValueError for the first violated (violated, message) rule of a contract."""
    for violated, message in rules:
        if violated:
            raise ValueError(message())


def _plan_contract(q, block_table, seqlen, k_caches, v_caches):
    """What a plan needs beyond the per-call contract, as ordered (violated, message) rules
    (the reference's plan messages, model/triton_decode.py:380-440): a contiguous query, int32
    and unit-stride seqlen and block-table columns (both are held by reference, so in-place
    updates must stay visible), and one K and one V pool per layer."""
    yield q.dim() != 3, lambda: f"q must be (B, H, D), got shape {tuple(q.shape)}"
    yield not q.is_contiguous(), lambda: (
        f"paged_decode_plan needs a contiguous (B, H, D) query, got strides {q.stride()}; "
        "call .contiguous() once, not per layer")
    yield q.shape[0] == 0, lambda: "paged_decode_plan needs at least one row"
    yield seqlen.dtype != torch.int32, lambda: (
        "paged_decode_plan requires an int32 seqlen so in-place updates are visible; "
        f"got {seqlen.dtype}. Cast once at the container boundary.")
    yield seqlen.stride(0) != 1, lambda: (
        f"paged_decode_plan requires a contiguous 1-D seqlen; got strides {seqlen.stride()}")
    yield block_table.stride(1) != 1, lambda: (
        f"paged_decode_plan requires a column-contiguous block table; got strides {block_table.stride()}")
    yield len(k_caches) != len(v_caches) or not k_caches, lambda: (
        f"paged_decode_plan needs one k_cache/v_cache per layer, got {len(k_caches)} / {len(v_caches)}")


def _plan_layer_contract(k_cache, v_cache, k_first, v_first):
    """Every layer's pools share the first layer's shapes and strides (the plan encodes one
    launch geometry), and TMA can describe them as they are."""
    yield k_cache.shape != k_first.shape or v_cache.shape != v_first.shape, lambda: (
        "paged_decode_plan needs one pool shape for every layer")
    yield k_cache.stride() != k_first.stride(), lambda: "paged_decode_plan needs one pool layout for every layer"
    yield v_cache.stride() != v_first.stride(), lambda: "paged_decode_plan needs one v-pool layout for every layer"
    yield not (_tma_ready(k_cache) and _tma_ready(v_cache)), lambda: (
        "paged_decode_plan needs pools with a unit head_dim stride, 16-byte multiple strides and "
        "a 16-byte aligned base (any contiguous pool qualifies)")


def _tma_ready(pool: torch.Tensor) -> bool:
    """Whether the pool's layout can be described by a TMA descriptor as it is."""
    es = pool.element_size()
    s = pool.stride()
    return (
        s[3] == 1
        and all(x > 0 and (x * es) % 16 == 0 for x in s[:3])
        and pool.data_ptr() % 16 == 0
    )


def _kernel_pool(pool: torch.Tensor) -> torch.Tensor:
    if _tma_ready(pool):
        return pool
    copy = pool.contiguous() if not pool.is_contiguous() else pool.clone()
    if not _tma_ready(copy):  # pragma: no cover - a fresh contiguous tensor always is
        raise ValueError(f"cannot lay out a pool of shape {tuple(pool.shape)} for TMA")
    return copy


def _workspace(q: torch.Tensor, n_kv_head: int) -> torch.Tensor:
    B, H, D = q.shape
    need = _native.workspace_bytes(B, H, n_kv_head, D, q.dtype)
    key = (q.device.index if q.device.index is not None else torch.cuda.current_device(),
           _native.stream_handle(q.device))
    ws = _WORKSPACES.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.empty(max(need, 256), dtype=torch.uint8, device=q.device)
        _WORKSPACES[key] = ws
    return ws


def paged_prefill(q, k_cache, v_cache, block_table, cu_seqlens_q, seqlen_k, max_seqlen_q: int, *,
                  scale: float | None = None):
    """Chunked-prefill attention reading the paged pool (one kernel launch).

    ``q`` is the packed ``(total_q, H, D)`` query of every row's new tokens, row ``b`` owning
    ``q[cu_seqlens_q[b]:cu_seqlens_q[b + 1]]``; the chunk's K/V are already in the pools (written
    with ``PagedPool.write_slots`` / ``PagedKV``). Query token ``i`` of a chunk of ``Sq`` tokens sits
    at position ``seqlen_k[b] - Sq + i`` and attends causally to keys ``0 .. seqlen_k[b] - Sq + i``
    of its row (the bottom-right causal convention of varlen flash attention with a block
    table). ``max_seqlen_q`` must be at least the longest chunk (it sizes the launch without a
    host read of ``cu_seqlens_q``; tokens of a longer chunk past it are left unwritten), as in
    varlen flash attention. Returns ``out`` shaped like ``q``.

    bf16 / fp16 pools, head_dim 64, 128 or 256, 1/2/4/8 q heads per kv head, block_size >= 8. The
    reference has no counterpart to mirror: its packed varlen prefill (model/attention/varlen.py:
    317-357, docs/decisions.md D7) writes the paged pool but never reads it.
    """
    _require_backend()
    _require_cuda_tensors((("q", q), ("k_cache", k_cache), ("v_cache", v_cache), ("block_table", block_table),
                           ("cu_seqlens_q", cu_seqlens_q), ("seqlen_k", seqlen_k)))
    if q.dim() != 3 or k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("paged_prefill needs q (total_q, H, D) and k_cache/v_cache (n_blocks, bs, H_kv, D)")
    if q.dtype != k_cache.dtype or v_cache.dtype != k_cache.dtype:
        raise TypeError(f"dtype mismatch: q {q.dtype}, k_cache {k_cache.dtype}, v_cache {v_cache.dtype}")
    if q.shape[2] != k_cache.shape[3] or q.shape[1] % k_cache.shape[2] != 0:
        raise ValueError(f"q {tuple(q.shape)} does not match the pool {tuple(k_cache.shape)}")
    B = seqlen_k.shape[0]
    if cu_seqlens_q.shape != (B + 1,) or block_table.dim() != 2 or block_table.shape[0] != B:
        raise ValueError("paged_prefill needs cu_seqlens_q (B + 1,), seqlen_k (B,) and block_table (B, max_blocks)")
    q = q.contiguous()
    out = torch.empty_like(q)
    if B == 0 or q.shape[0] == 0 or max_seqlen_q <= 0:
        return out
    cu32 = cu_seqlens_q.contiguous().to(torch.int32)
    sk32 = seqlen_k.contiguous().to(torch.int32)
    if block_table.dtype != torch.int32 or block_table.stride(1) != 1:
        block_table = block_table.contiguous().to(torch.int32)
    if scale is None:
        scale = 1.0 / math.sqrt(q.shape[2])
    with torch.cuda.device(q.device):
        _native.prefill(q, _kernel_pool(k_cache), _kernel_pool(v_cache), block_table, cu32, sk32,
                        int(max_seqlen_q), out, q.shape[1], float(scale) * _LOG2E)
    return out


def paged_decode(q, k_cache, v_cache, block_table, seqlen, *, scale: float | None = None):
    """Decode one query token per row against a paged KV pool (one kernel launch)."""
    _require_backend()
    _require_cuda_tensors((("q", q), ("k_cache", k_cache), ("v_cache", v_cache),
                           ("block_table", block_table), ("seqlen", seqlen)))
    _validate(q, k_cache, v_cache, block_table, seqlen)
    B, H, D = q.shape
    if B == 0:
        return torch.empty_like(q)
    q = q.contiguous()
    if block_table.stride(1) != 1 or block_table.stride(0) < block_table.shape[1]:
        block_table = block_table.contiguous()
    seqlen = seqlen.contiguous()
    seqlen32 = seqlen if seqlen.dtype == torch.int32 else seqlen.to(torch.int32)
    k_cache = _kernel_pool(k_cache)
    v_cache = _kernel_pool(v_cache)
    out = torch.empty_like(q)
    if scale is None:
        scale = 1.0 / math.sqrt(D)
    with torch.cuda.device(q.device):
        _native.decode(q, k_cache, v_cache, block_table, seqlen32, out, float(scale) * _LOG2E,
                       _workspace(q, k_cache.shape[2]))
    return out


class PagedDecodePlan:
    """Per-container launch state for repeated decode calls (one launch per layer).

    Mirrors the reference's plan (``model/triton_decode.py:331-520``): every
    ``(k_cache, v_cache)`` pair is validated once with the full :func:`paged_decode` contract,
    the block table and int32 seqlen are held by reference (in-place updates are seen, an
    int64 seqlen is refused rather than snapshotted), and :meth:`run` checks only the query
    layout. On top of that the plan encodes each layer's two TMA descriptors once (in the
    native ``pd_plan``) and owns the decode workspace.
    """

    __slots__ = ("n_layer", "grid", "q_shape", "q_dtype", "q_device", "q_strides", "_k", "_v",
                 "_block_table", "_seqlen", "_native_plan", "_workspace", "_stream_cache")

    def __init__(self, q, k_caches, v_caches, block_table, seqlen, *, scale: float | None = None):
        _require_backend()
        _require_cuda_tensors((("q", q), ("block_table", block_table), ("seqlen", seqlen)))
        k_caches, v_caches = list(k_caches), list(v_caches)
        _raise_first(_plan_contract(q, block_table, seqlen, k_caches, v_caches))
        b, h, d = q.shape
        for layer, (k_cache, v_cache) in enumerate(zip(k_caches, v_caches)):
            # the whole paged_decode contract once per layer, then the layers must agree
            _require_cuda_tensors(((f"k_cache[{layer}]", k_cache), (f"v_cache[{layer}]", v_cache)))
            _validate(q, k_cache, v_cache, block_table, seqlen)
            _raise_first(_plan_layer_contract(k_cache, v_cache, k_caches[0], v_caches[0]))
        self.n_layer = len(k_caches)
        self._k = k_caches
        self._v = v_caches
        self._block_table = block_table
        self._seqlen = seqlen
        self.q_shape = (int(b), int(h), int(d))
        self.q_dtype = q.dtype
        self.q_device = q.device
        self.q_strides = (int(q.stride(0)), int(q.stride(1)), int(q.stride(2)))
        self.grid = (int(b), int(h))  # logical output grid; the launch is one CTA per SM
        if scale is None:
            scale = 1.0 / math.sqrt(d)
        with torch.cuda.device(q.device):
            need = _native.workspace_bytes(b, h, k_caches[0].shape[2], d, q.dtype)
            # two halves: consecutive launches alternate, which overlapped launches need
            half = -(-max(need, 256) // 256) * 256
            self._workspace = torch.empty(2 * half, dtype=torch.uint8, device=q.device)
            self._native_plan = _native.NativePlan(
                k_caches, v_caches, block_table, seqlen, b, h, float(scale) * _LOG2E, self._workspace
            )
        self._stream_cache = None

    def _check_query(self, layer: int, q) -> int:
        if not 0 <= int(layer) < self.n_layer:
            raise IndexError(f"layer {layer} outside the plan's {self.n_layer} layers")
        if (
            tuple(q.shape) != self.q_shape
            or q.dtype != self.q_dtype
            or q.device != self.q_device
            or q.stride() != self.q_strides
        ):
            raise ValueError(
                "paged_decode_plan.run got a query that does not match the validated layout "
                f"{(self.q_shape, self.q_dtype, self.q_strides)}; got "
                f"{(tuple(q.shape), q.dtype, q.stride())}. Rebuild the plan for a new layout."
            )
        return int(layer)

    def _output(self, out):
        if out is None:
            return torch.empty(self.q_shape, dtype=self.q_dtype, device=self.q_device)
        if (tuple(out.shape) != self.q_shape or out.dtype != self.q_dtype or out.device != self.q_device
                or out.stride() != self.q_strides):
            raise ValueError(f"out must be a contiguous {self.q_shape} {self.q_dtype} tensor on {self.q_device}")
        return out

    def run(self, layer: int, q, *, out=None, overlap: bool = False):
        """Launch the kernel for one layer; ``q`` must match the validated layout. ``out``
        (optional) is a preallocated contiguous ``(B, H, D)`` result buffer.

        ``overlap=True`` lets the launch start while the previous kernel of the stream
        finishes (programmatic dependent launch): it reads seqlen, the block table and the
        pools and issues its first K/V copies before it waits for that kernel, so that kernel
        must write none of them (the previous layer's decode of a step does not)."""
        layer = self._check_query(layer, q)
        out = self._output(out)
        self._native_plan.run(layer, q, out, torch.cuda.current_stream(self.q_device).cuda_stream, overlap)
        return out

    def can_fuse_append(self, k_new, v_new, pos, rope=None) -> bool:
        """Whether :meth:`run_append` takes these tensors: ``(B, H_kv, D)`` rows in the plan's
        dtype on its device with a unit last stride and 16-byte aligned rows, an int64
        ``(B,)`` contiguous ``pos``, and (with ``rope``) ``(B, rotary_dim / 2)`` cos/sin tables
        in the plan's dtype with a unit last stride."""
        if rope is not None:
            cos, sin, rotary_dim = rope
            half = int(rotary_dim) // 2
            for t in (cos, sin):
                if (t.dim() != 2 or tuple(t.shape) != (self.q_shape[0], half) or t.dtype != self.q_dtype
                        or t.device != self.q_device or t.stride(1) != 1 or t.stride(0) != cos.stride(0)):
                    return False
            if not (2 <= int(rotary_dim) <= self.q_shape[2] and int(rotary_dim) % 2 == 0):
                return False
        b, _, d = self.q_shape
        shape = (b, self._k[0].shape[2], d)
        es = self._k[0].element_size()
        for t in (k_new, v_new):
            if tuple(t.shape) != shape or t.dtype != self.q_dtype or t.device != self.q_device:
                return False
            if t.stride(2) != 1 or (t.stride(0) * es) % 16 or (t.stride(1) * es) % 16 or t.data_ptr() % 16:
                return False
        return (pos.dtype == torch.int64 and tuple(pos.shape) == (b,) and pos.device == self.q_device
                and pos.stride(0) == 1)

    def run_append(self, layer: int, q, k_new, v_new, pos, *, out=None, rope=None, overlap: bool = False):
        """Store row ``b``'s new K/V ``(B, H_kv, D)`` at logical position ``pos[b]`` of layer
        ``layer``'s pools and decode that layer, in one launch.

        Same result as ``PagedKV.write`` followed by :meth:`run` -- the pools and the output
        are bit-identical -- provided no row reads a slot another row appends (rows do not
        share blocks they write). ``rope`` = (cos, sin, rotary_dim) gives ``k_new`` before its
        rotary embedding, which the launch applies exactly as the model's torch ops would.
        Tensors must pass :meth:`can_fuse_append`. ``overlap`` as in :meth:`run` (``pos`` is
        read before the wait as well; ``k_new``/``v_new`` and ``q`` after it).
        """
        layer = self._check_query(layer, q)
        if not self.can_fuse_append(k_new, v_new, pos, rope):
            raise ValueError(
                "paged_decode_plan.run_append needs (B, H_kv, D) k/v rows in the plan's dtype with "
                "16-byte aligned rows and an int64 (B,) pos on the plan's device"
            )
        out = self._output(out)
        self._native_plan.run_append(layer, q, out, k_new, v_new, pos,
                                     torch.cuda.current_stream(self.q_device).cuda_stream, rope, overlap)
        return out


def paged_decode_plan(q, k_caches, v_caches, block_table, seqlen, *, scale: float | None = None):
    """Validate one container's paged-decode tensors and cache their launch state."""
    return PagedDecodePlan(q, k_caches, v_caches, block_table, seqlen, scale=scale)
