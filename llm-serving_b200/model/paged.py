"""Paged KV storage and the decode container, written over the sm_100a append/decode kernels.

Drop-in for the reference's ``model/paged.py`` (``PagedPool`` 82-306, ``PagedKV`` 309-586):
same constructor arguments, attributes, step protocol and error messages, so the engine,
scheduler and model layers call it unchanged. What changed is underneath:

* ``PagedPool.write_slots`` (prefill and decode writes) is one launch of the append kernel
  (``pd_kv_append_slots``) that moves K and V together, instead of two ``index_copy_``.
* ``PagedKV.write`` + ``PagedKV.attend`` of one layer are ONE launch
  (``pd_plan_run_append``): ``write`` validates and records the step's K/V, and the decode
  launch of ``attend`` first stores them at ``table[row, pos // bs] * bs + pos % bs`` and then
  attends over them. Anything else that touches the pool before that ``attend`` -- reading
  ``PagedPool.keys`` / ``values``, another write, ``build_mask``, ``advance``, ``flush`` --
  first performs the recorded append as its own launch (``pd_kv_append_table``), so every
  observer sees the same pool as with an immediate write. ``PagedKV(..., fuse_append=False)``
  always writes immediately.

Layout (unchanged): one ``(n_blocks, block_size, n_kv_head, head_dim)`` K and V tensor per
layer, allocated once and never replaced; token ``t`` of a request lives at block
``block_table[t // block_size]``, slot ``t % block_size``; every layer shares the block table.

Step order the model relies on (reference ``model/paged.py:37-46``)::

    paged.build_mask(next_token=True)   # seqlen := pos + 1 (int32, in place)
    for layer in layers:
        paged.write(layer, k, v)        # this step's token at pos[row]
        y = paged.attend(layer, q)      # block-table decode
    paged.advance()                     # pos += active

A pool may be created on the CPU (its host-side checks work there), but every write and the
decode container need CUDA: there is no CPU kernel path and no fallback. The CPU oracle used
by the tests lives in ``oracle/``.
"""

from __future__ import annotations

import torch

from model import _native
from model.triton_decode import TRITON_AVAILABLE

__all__ = ["PagedPool", "PagedKV"]


def _positive(name: str, value) -> int:
    if isinstance(value, bool) or not isinstance(value, int) or value < 1:
        raise ValueError(f"{name} must be a positive int, got {value!r}")
    return value


def _same_device(a: torch.device, b: torch.device) -> bool:
    """``cuda`` (current device) and ``cuda:N`` name the same device unless both are explicit."""
    return a.type == b.type and (a.index is None or b.index is None or a.index == b.index)


def _unit_last_stride(t: torch.Tensor) -> torch.Tensor:
    return t if t.stride(-1) == 1 else t.contiguous()


class PagedPool:
    """Physical KV blocks: one ``(n_blocks, block_size, n_kv_head, head_dim)`` K and V per layer."""

    def __init__(self, n_layer: int, n_blocks: int, block_size: int, n_kv_head: int, head_dim: int,
                 *, dtype: torch.dtype = torch.float32, device="cpu", n_head: int | None = None):
        self.n_layer = _positive("n_layer", n_layer)
        self.n_blocks = _positive("n_blocks", n_blocks)
        self.block_size = _positive("block_size", block_size)
        self.n_kv_head = _positive("n_kv_head", n_kv_head)
        self.head_dim = _positive("head_dim", head_dim)
        n_head = self.n_kv_head if n_head is None else int(n_head)
        if n_head % self.n_kv_head != 0:
            raise ValueError(f"n_head ({n_head}) must be a multiple of n_kv_head ({self.n_kv_head})")
        self.n_head = n_head
        self.n_group = n_head // self.n_kv_head
        self.dtype = dtype
        self.device = torch.device(device)
        shape = (self.n_blocks, self.block_size, self.n_kv_head, self.head_dim)
        self._keys = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(self.n_layer)]
        self._values = [torch.zeros(shape, dtype=dtype, device=self.device) for _ in range(self.n_layer)]
        # Flat (n_blocks * block_size, n_kv_head, head_dim) views: a slot id is a row of these.
        self._keys_flat = [t.view(-1, self.n_kv_head, self.head_dim) for t in self._keys]
        self._values_flat = [t.view(-1, self.n_kv_head, self.head_dim) for t in self._values]
        # A decode-step append recorded by PagedKV.write and not yet launched (see flush).
        self._pending = None
        # One-entry cache of the prefill slot map keyed by (table, start, length).
        self._prefill_key: tuple | None = None
        self._prefill_slots: torch.Tensor | None = None

    # ------------------------------------------------------------------ pool tensors
    @property
    def keys(self) -> list[torch.Tensor]:
        """Per-layer K pools. Reading them first performs a recorded append (:meth:`flush`)."""
        self.flush()
        return self._keys

    @property
    def values(self) -> list[torch.Tensor]:
        """Per-layer V pools. Reading them first performs a recorded append (:meth:`flush`)."""
        self.flush()
        return self._values

    def flush(self) -> None:
        """Launch the decode-step append that ``PagedKV.write`` recorded, if any, on the
        stream it was recorded on. Afterwards the pools hold every written token."""
        pending, self._pending = self._pending, None
        if pending is not None:
            pending.launch()

    def _record(self, pending) -> None:
        self.flush()
        self._pending = pending

    # ------------------------------------------------------------------ checks
    def _check_layer(self, layer: int) -> int:
        if not 0 <= int(layer) < self.n_layer:
            raise IndexError(f"layer {layer} outside the pool's {self.n_layer} layers")
        return int(layer)

    def _check_block_ids(self, block_ids, needed: int) -> None:
        for block_id in block_ids:
            if isinstance(block_id, bool) or not isinstance(block_id, int):
                raise ValueError(f"block ids must be ints, got {block_id!r}")
            if not 0 <= block_id < self.n_blocks:
                raise IndexError(f"block id {block_id} outside the pool's {self.n_blocks} blocks")
        if len(block_ids) < needed:
            raise IndexError(f"block table has {len(block_ids)} blocks, needs {needed} to address this write")

    def _check_rows(self, what: str, k: torch.Tensor, v: torch.Tensor) -> None:
        if k.dim() != 3 or v.dim() != 3:
            raise ValueError(f"{what} needs (length, n_kv_head, head_dim), got {tuple(k.shape)} / {tuple(v.shape)}")
        if tuple(k.shape) != tuple(v.shape):
            raise ValueError(f"k/v shapes differ: {tuple(k.shape)} vs {tuple(v.shape)}")
        if k.shape[1:] != (self.n_kv_head, self.head_dim):
            raise ValueError(
                f"{what} needs head shape {(self.n_kv_head, self.head_dim)}, got {tuple(k.shape[1:])}"
            )

    def _require_cuda(self, what: str) -> None:
        if self.device.type != "cuda":
            raise RuntimeError(
                f"PagedPool.{what} requires a CUDA pool (this one is on {self.device}): the paged "
                "append is the sm_100a kernel and has no CPU path"
            )
        if not TRITON_AVAILABLE:
            raise RuntimeError(f"PagedPool.{what} requires the sm_100a library: {_native.LOAD_ERROR}")

    # ------------------------------------------------------------------ slot maps
    def _slot_ids(self, block_table, start: int, length: int) -> torch.Tensor:
        """``(length,)`` flat slots of logical tokens ``[start, start + length)``, cached."""
        key = (tuple(block_table), start, length)
        if key == self._prefill_key and self._prefill_slots is not None:
            return self._prefill_slots
        bs = self.block_size
        slots = [block_table[t // bs] * bs + t % bs for t in range(start, start + length)]
        tensor = torch.tensor(slots, dtype=torch.long, device=self.device)
        self._prefill_key = key
        self._prefill_slots = tensor
        return tensor

    def slot_ids(self, block_table, start: int, length: int) -> torch.Tensor:
        """Public slot-map builder for a caller that writes the same map to every layer."""
        start, length = int(start), int(length)
        if start < 0:
            raise ValueError(f"start must be >= 0, got {start}")
        if length < 0:
            raise ValueError(f"length must be >= 0, got {length}")
        self._check_block_ids(block_table, (start + length + self.block_size - 1) // self.block_size)
        return self._slot_ids(block_table, start, length)

    # ------------------------------------------------------------------ writes
    def write_slots(self, layer: int, slot_ids: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        """Copy token ``i`` of k/v ``(n, n_kv_head, head_dim)`` into flat pool row ``slot_ids[i]``.

        One append-kernel launch for K and V together (the reference issues two
        ``index_copy_``). Slots must be distinct and inside the pool, as in the reference; the
        kernel skips one outside the pool and records it in the device error word instead of
        faulting. No host-side scan of the slots (that would be a sync per layer).
        """
        layer = self._check_layer(layer)
        self._check_rows("write_slots", k, v)
        if slot_ids.dim() != 1 or slot_ids.numel() != k.shape[0]:
            raise ValueError(
                f"slot_ids must be 1-D with one entry per token ({k.shape[0]}), got {tuple(slot_ids.shape)}"
            )
        if slot_ids.dtype not in (torch.int32, torch.int64):
            raise ValueError(f"slot_ids must be an integer tensor, got {slot_ids.dtype}")
        if not _same_device(slot_ids.device, self.device):
            raise ValueError(f"slot_ids on {slot_ids.device} but the pool is on {self.device}")
        self._require_cuda("write_slots")
        for name, t in (("k", k), ("v", v)):
            if not _same_device(t.device, self.device):
                raise ValueError(f"{name} on {t.device} but the pool is on {self.device}")
            if t.dtype not in (torch.float32, torch.float16, torch.bfloat16):
                raise ValueError(f"{name} dtype must be fp32, fp16 or bf16, got {t.dtype}")
        if k.shape[0] == 0:
            return
        self.flush()
        with torch.cuda.device(self._keys[layer].device):
            _native.append_slots(self._keys[layer], self._values[layer], slot_ids.contiguous(),
                                 _unit_last_stride(k), _unit_last_stride(v.to(k.dtype)))

    def write_prefill_slots(self, layer: int, slot_ids: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> None:
        """Named prefill entry point (``PagedWriteSink``): :meth:`write_slots` with a prebuilt map."""
        self.write_slots(layer, slot_ids, k, v)

    def write_prefill(self, layer: int, block_table, start: int, k: torch.Tensor, v: torch.Tensor) -> None:
        """Write logical tokens ``[start, start + len(k))`` of one request through its table."""
        layer = self._check_layer(layer)
        self._check_rows("write_prefill", k, v)
        start = int(start)
        if start < 0:
            raise ValueError(f"start must be >= 0, got {start}")
        length = k.shape[0]
        if length == 0:
            return
        self._check_block_ids(block_table, (start + length + self.block_size - 1) // self.block_size)
        self.write_prefill_slots(layer, self._slot_ids(block_table, start, length), k, v)

    # ------------------------------------------------------------------ accounting
    def bytes(self) -> int:
        """Physical KV bytes of the pool (K + V, all layers)."""
        return 2 * self.n_layer * self.n_blocks * self.block_size * self.n_kv_head * self.head_dim * self.dtype.itemsize

    def mb(self) -> float:
        return self.bytes() / 2**20


class _PendingAppend:
    """One decode-step append recorded by :meth:`PagedKV.write`: consumed by the fused launch
    of the same layer's ``attend``, or launched alone by :meth:`PagedPool.flush`."""

    __slots__ = ("owner", "layer", "k", "v", "rope", "stream")

    def __init__(self, owner: "PagedKV", layer: int, k: torch.Tensor, v: torch.Tensor, rope, stream) -> None:
        self.owner, self.layer, self.k, self.v, self.rope, self.stream = owner, layer, k, v, rope, stream

    def launch(self) -> None:
        with torch.cuda.stream(self.stream):
            self.owner._append_now(self.layer, self.k, self.v, self.rope)


def _fusable_rows(t: torch.Tensor, dtype: torch.dtype) -> bool:
    """(B, H_kv, D) rows the fused append reads directly: pool dtype, 16-byte aligned rows."""
    es = t.element_size()
    return (t.dtype == dtype and t.stride(2) == 1 and (t.stride(0) * es) % 16 == 0
            and (t.stride(1) * es) % 16 == 0 and t.data_ptr() % 16 == 0)


def _container_rules(pool, block_tables, lengths, rope_len: int, n_head, seats):
    """The arguments' contract for a decode container as (violated, exception, message) rules,
    in the order they are checked (the reference's ``PagedKV.__init__`` contract and messages,
    model/paged.py:334-451; its callers match on them). Later rules rely on earlier ones
    holding, so the rules are produced lazily and the caller stops at the first violation."""
    yield not isinstance(pool, PagedPool), TypeError, lambda: f"PagedKV needs a PagedPool, got {type(pool).__name__}"
    yield pool.device.type != "cuda", ValueError, lambda: (
        "paged decode is the sm_100a CUDA block-table kernel; the gather control arm was "
        f"deleted. The pool is on {pool.device}. Run the paged arm on CUDA, or use the seat "
        "arm on CPU. The dense numeric oracle lives in oracle/.")
    yield not TRITON_AVAILABLE, RuntimeError, lambda: (
        "paged decode requires the sm_100a library that replaces the Triton kernel, but it "
        f"could not be loaded ({_native.LOAD_ERROR}); there is no eager fallback.")
    n_rows = len(block_tables)
    yield n_rows < 1, ValueError, lambda: "PagedKV needs at least one row"
    yield len(lengths) != n_rows, ValueError, lambda: (
        f"PagedKV needs one length per block table, got {len(lengths)} for {n_rows}")
    yield rope_len < 1, ValueError, lambda: f"rope_len (the run's position bound) must be >= 1, got {rope_len}"
    n_head = pool.n_kv_head if n_head is None else int(n_head)
    yield n_head % pool.n_kv_head != 0, ValueError, lambda: (
        f"n_head ({n_head}) must be a multiple of n_kv_head ({pool.n_kv_head})")
    yield len(seats) != n_rows, ValueError, lambda: f"PagedKV needs one seat per row, got {len(seats)} for {n_rows}"
    for row, length in enumerate(lengths):
        blocks = len(block_tables[row])
        yield length < 0, ValueError, lambda row=row, length=length: f"row {row}: length must be >= 0, got {length}"
        yield length > blocks * pool.block_size, IndexError, lambda row=row, length=length, blocks=blocks: (
            f"row {row}: length {length} exceeds its block table's capacity ({blocks} blocks x {pool.block_size})")
        yield length > rope_len, IndexError, lambda row=row, length=length: (
            f"row {row}: length {length} exceeds the run's position bound {rope_len}")


class PagedKV:
    """Decode-time container over a :class:`PagedPool` (the ``KvSlab`` step protocol).

    Rows are the active requests; ``seats[row]`` is the engine seat. ``pos``/``valid``/
    ``active`` are device tensors updated in place with Python mirrors; ``max_len`` is the
    run's position bound (the RoPE table length). The padded int32 block table is built once
    per container and never mutated; the int32 ``seqlen`` is refreshed in place by
    :meth:`build_mask` and read by the decode plan by reference.
    """

    decode_container = True
    block_table_decode = True

    def __init__(self, pool: PagedPool, block_tables, lengths, *, rope_len: int, seats=None,
                 n_head: int | None = None, check_bounds: bool = True, fuse_append: bool = True,
                 overlap_layers: bool = True) -> None:
        lengths = [int(n) for n in lengths]
        rope_len = int(rope_len)
        seats = list(range(len(block_tables))) if seats is None else list(seats)
        for violated, error, message in _container_rules(pool, block_tables, lengths, rope_len, n_head, seats):
            if violated:
                raise error(message())
        n_head = pool.n_kv_head if n_head is None else int(n_head)

        self.pool = pool
        self.n_layer = pool.n_layer
        self.n_kv_head = pool.n_kv_head
        self.head_dim = pool.head_dim
        self.n_head = n_head
        self.n_group = n_head // pool.n_kv_head
        self.dtype = pool.dtype
        self.device = pool.device
        self.check_bounds = bool(check_bounds)
        self.block_tables = [list(bt) for bt in block_tables]
        self.seats = seats
        self.row_of_seat = {seat: row for row, seat in enumerate(seats)}
        self.batch = n_rows = len(block_tables)
        self.max_len = rope_len

        self.pos = torch.tensor(lengths, dtype=torch.long, device=self.device)
        self.valid = torch.tensor(lengths, dtype=torch.long, device=self.device)
        self.active = torch.ones(n_rows, dtype=torch.bool, device=self.device)
        self._host_pos = list(lengths)
        self._host_valid = list(lengths)
        self._host_active = [True] * n_rows

        width = max((len(t) for t in self.block_tables), default=1) or 1
        host_table = torch.zeros((n_rows, width), dtype=torch.int32)
        for row, table in enumerate(self.block_tables):
            if not table:
                continue
            pool._check_block_ids(table, (max(lengths[row], 1) + pool.block_size - 1) // pool.block_size)
            host_table[row, : len(table)] = torch.tensor(table, dtype=torch.int32)
        self._block_table_tensor = host_table.to(self.device)
        self._seqlen = torch.zeros(n_rows, dtype=torch.int32, device=self.device)
        self._slot_error: tuple[int, int, int, int] | None = None
        self._slot_cache: torch.Tensor | None = None
        self._refresh_slots()
        self._decode_plan = None
        self._step_written = False
        self._seqlen_ready = False
        # The fused append + decode launch needs rows that never share a block (a row must not
        # read a slot another row appends); tables from BlockManager never do.
        owned = [b for table in self.block_tables for b in table]
        self.fuse_append = bool(fuse_append) and len(owned) == len(set(owned))
        # A fused write + attend right after this container's previous fused attend may start
        # while that launch finishes (programmatic dependent launch): nothing it reads before
        # waiting (seqlen, positions, block table, pools) is written in between. Any other
        # launch of the container (the seqlen update, an append on its own, advance) clears
        # the flag, so the next attend waits for it as usual.
        self.overlap_layers = bool(overlap_layers)
        self._after_attend = False

    # ---------------------------------------------------------------- step hooks
    def build_mask(self, *, next_token: bool = False) -> None:
        """Step boundary: ``seqlen := pos + next_token`` as int32, in place (no mask/bias)."""
        self.pool.flush()
        longest = max(n + int(next_token) for n in self._host_valid)
        if self.check_bounds and longest > self.max_len:
            raise IndexError(f"PagedKV overflow: needs {longest} positions, run position bound is {self.max_len}")
        self._seqlen.copy_((self.pos + int(next_token)).to(torch.int32))
        self._step_written = False
        self._seqlen_ready = True
        self._after_attend = False
        return None

    def _refresh_slots(self) -> None:
        """Host bound check of the next write position of every row (no device work).

        A row whose position needs a block beyond its table parks the container in an error
        state that :meth:`write` reports; the fused append computes the slots on device.
        """
        bs = self.pool.block_size
        self._slot_error = None
        self._slot_cache = None
        for row, position in enumerate(self._host_pos):
            block_index = position // bs
            if block_index >= len(self.block_tables[row]):
                self._slot_error = (row, position, block_index, len(self.block_tables[row]))
                break

    @property
    def _slot_ids(self) -> torch.Tensor | None:
        """Flat slot each row writes next (``None`` past a row's table); built on demand."""
        if self._slot_error is not None:
            return None
        if self._slot_cache is None:
            bs = self.pool.block_size
            blocks = self._block_table_tensor.to(torch.int64).gather(1, (self.pos // bs).view(-1, 1)).squeeze(1)
            self._slot_cache = blocks * bs + self.pos % bs
        return self._slot_cache

    def _rope_tables(self, rope):
        """``rope`` = (cos, sin): per-row tables of the step's positions, (B, 1, R/2) as the model
        hands them to the layer or (B, R/2); returns (cos, sin, R) as (B, R/2) views."""
        cos, sin = rope
        if cos.dim() == 3 and cos.shape[1] == 1:
            cos, sin = cos[:, 0], sin[:, 0]
        half = cos.shape[-1]
        if cos.dim() != 2 or tuple(cos.shape) != (self.batch, half) or tuple(sin.shape) != tuple(cos.shape):
            raise ValueError(f"rope needs cos/sin of shape (B, 1, rotary_dim/2) or (B, rotary_dim/2) with "
                             f"B={self.batch}, got {tuple(rope[0].shape)} / {tuple(rope[1].shape)}")
        if not 1 <= half <= self.head_dim // 2:
            raise ValueError(f"rotary_dim {2 * half} must be in [2, head_dim={self.head_dim}]")
        for name, t in (("cos", cos), ("sin", sin)):
            if t.dtype != self.dtype or not _same_device(t.device, self.device):
                raise ValueError(f"rope {name} must be {self.dtype} on {self.device}, got {t.dtype} on {t.device}")
        cos, sin = _unit_last_stride(cos), _unit_last_stride(sin)
        if sin.stride(0) != cos.stride(0):
            sin = sin.contiguous()
            cos = cos.contiguous()
        return cos, sin, 2 * half

    def write(self, layer: int, k: torch.Tensor, v: torch.Tensor, *, rope=None) -> None:
        """Append this step's token of every row at its own position (one fused launch).

        ``rope`` = (cos, sin) passes K *before* its rotary embedding: the rows are rotated on
        the way into the pool (GPT-NeoX pairs over the first ``2 * cos.shape[-1]`` dims),
        bit-identical to the model rotating with torch and then writing
        (model/layers.py:210-211 followed by this call)."""
        expected = (self.batch, self.n_kv_head, 1, self.head_dim)
        if tuple(k.shape) != expected or tuple(v.shape) != expected:
            raise ValueError(f"write needs {expected}, got {tuple(k.shape)} / {tuple(v.shape)}")
        layer = self.pool._check_layer(layer)
        if self.check_bounds and max(self._host_pos) >= self.max_len:
            raise IndexError(f"PagedKV overflow: write position {max(self._host_pos)} >= max_len {self.max_len}")
        if self._slot_error is not None:
            row, position, block_index, have = self._slot_error
            raise IndexError(
                f"row {row}: position {position} needs block {block_index}, but its block table has {have} blocks"
            )
        for name, t in (("k", k), ("v", v)):
            if t.dtype not in (torch.float32, torch.float16, torch.bfloat16):
                raise ValueError(f"{name} dtype must be fp32, fp16 or bf16, got {t.dtype}")
            if not _same_device(t.device, self.device):
                raise ValueError(f"{name} on {t.device} but the pool is on {self.device}")
        tables = None if rope is None else self._rope_tables(rope)
        if tables is not None and k.dtype != self.dtype:
            raise ValueError(f"a rotated write needs K in the pool dtype {self.dtype}, got {k.dtype}")
        k3, v3 = k[:, :, 0, :], v[:, :, 0, :]
        if self.fuse_append and _fusable_rows(k3, self.dtype) and _fusable_rows(v3, self.dtype):
            self.pool._record(_PendingAppend(self, layer, k3, v3, tables, torch.cuda.current_stream(self.device)))
        else:
            self.pool.flush()
            self._append_now(layer, k3, v3, tables)
        self._step_written = True

    def _append_now(self, layer: int, k3: torch.Tensor, v3: torch.Tensor, rope=None) -> None:
        """The append alone: one ``pd_kv_append_table`` launch on the current stream."""
        self._after_attend = False
        with torch.cuda.device(self.pool._keys[layer].device):
            _native.append_table(self.pool._keys[layer], self.pool._values[layer], self._block_table_tensor,
                                 self.pos, _unit_last_stride(k3), _unit_last_stride(v3.to(k3.dtype)), rope)

    def flush(self) -> None:
        """Perform a recorded append now (see :meth:`PagedPool.flush`)."""
        self.pool.flush()

    def _plan_for(self, q3: torch.Tensor):
        from model.triton_decode import paged_decode_plan

        if self._decode_plan is None:
            self._decode_plan = paged_decode_plan(
                q3, self.pool._keys, self.pool._values, self._block_table_tensor, self._seqlen,
                scale=1.0 / (self.head_dim ** 0.5),
            )
            # The container's padded table is built once and never edited, so the plan's step
            # cache may keep the table windows of each step's first copies too.
            self._decode_plan._native_plan.set_static_table(True)
        return self._decode_plan

    def attend(self, layer: int, q: torch.Tensor, *, dropout_p: float = 0.0,
               out: torch.Tensor | None = None) -> torch.Tensor:
        """Block-table decode for one layer; ``q`` is ``(B, H, 1, D)``, output the same.
        ``out`` (optional) is a preallocated contiguous ``(B, H, 1, D)`` result buffer."""
        # The step protocol first (the reference's order and messages, model/paged.py:530-538).
        expected = (self.batch, self.n_head, 1, self.head_dim)
        for violated, error, message in (
                (not self._seqlen_ready, RuntimeError, "PagedKV.attend() before build_mask(): seqlen is stale"),
                (not self._step_written, RuntimeError, "PagedKV.attend() before write(): this step has no token yet"),
                (bool(dropout_p), ValueError, "paged decode is inference-only; dropout_p must be 0"),
                (tuple(q.shape) != expected, ValueError, f"attend needs q {expected}, got {tuple(q.shape)}")):
            if violated:
                raise error(message)
        q3 = q[:, :, 0, :].contiguous()
        plan = self._plan_for(q3)
        out3 = None if out is None else out[:, :, 0, :]
        pending = self.pool._pending
        if (pending is not None and pending.owner is self and pending.layer == int(layer)
                and pending.stream == torch.cuda.current_stream(self.device)
                and plan.can_fuse_append(pending.k, pending.v, self.pos, pending.rope)):
            self.pool._pending = None
            out3 = plan.run_append(layer, q3, pending.k, pending.v, self.pos, out=out3, rope=pending.rope,
                                   overlap=self.overlap_layers and self._after_attend)
            self._after_attend = True
            return out3.unsqueeze(2)
        self.pool.flush()
        self._after_attend = False
        return plan.run(layer, q3, out=out3).unsqueeze(2)

    def advance(self) -> None:
        """Move every active row's cursor one token (device in place, then host mirrors)."""
        self.pool.flush()
        self._after_attend = False
        self.pos.add_(self.active)
        self.valid.copy_(torch.maximum(self.valid, self.pos))
        for row in range(self.batch):
            if self._host_active[row]:
                self._host_pos[row] += 1
                self._host_valid[row] = max(self._host_valid[row], self._host_pos[row])
        self._step_written = False
        self._seqlen_ready = False
        if self.check_bounds and max(self._host_pos) > self.max_len:
            raise IndexError(f"PagedKV overflow: max_len={self.max_len}; a request decoded past its budget")
        self._refresh_slots()

    # ---------------------------------------------------------------- CUDA-graph support
    def prepare(self, q: torch.Tensor) -> None:
        """Build the decode plan for queries shaped like ``q`` ``(B, H, 1, D)`` and load its
        kernel (one decode into a scratch output), touching neither the pool nor the step
        state -- what a captured step needs to exist before capture."""
        expected = (self.batch, self.n_head, 1, self.head_dim)
        if tuple(q.shape) != expected:
            raise ValueError(f"prepare needs q {expected}, got {tuple(q.shape)}")
        q3 = q[:, :, 0, :].contiguous()
        self._plan_for(q3).run(0, q3)

    def _host_snapshot(self):
        return (list(self._host_pos), list(self._host_valid), self._slot_error, self._step_written,
                self._seqlen_ready)

    def _host_restore(self, snap) -> None:
        (self._host_pos, self._host_valid, self._slot_error, self._step_written, self._seqlen_ready) = (
            list(snap[0]), list(snap[1]), snap[2], snap[3], snap[4])
        self._slot_cache = None

    def _replayed_step(self, next_token: bool) -> None:
        """Host side of one step whose device work was replayed from a graph: the checks that
        build_mask and write make, then the position mirrors advance makes."""
        longest = max(n + int(next_token) for n in self._host_valid)
        if self.check_bounds and longest > self.max_len:
            raise IndexError(f"PagedKV overflow: needs {longest} positions, run position bound is {self.max_len}")
        if self.check_bounds and max(self._host_pos) >= self.max_len:
            raise IndexError(f"PagedKV overflow: write position {max(self._host_pos)} >= max_len {self.max_len}")
        if self._slot_error is not None:
            row, position, block_index, have = self._slot_error
            raise IndexError(
                f"row {row}: position {position} needs block {block_index}, but its block table has {have} blocks"
            )

    def _replayed_advance(self) -> None:
        for row in range(self.batch):
            if self._host_active[row]:
                self._host_pos[row] += 1
                self._host_valid[row] = max(self._host_valid[row], self._host_pos[row])
        self._step_written = False
        self._seqlen_ready = False
        self._refresh_slots()

    # ---------------------------------------------------------------- helpers
    def past_len(self) -> int:
        return max(self._host_valid) if self._host_valid else 0

    def bytes(self) -> int:
        return self.pool.bytes()

    def mb(self) -> float:
        return self.bytes() / 2**20
