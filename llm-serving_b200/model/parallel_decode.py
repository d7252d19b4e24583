"""Multi-GPU paged decode: sequence sharding and context-parallel split-KV.

The reference is single-GPU and has no distributed code. On one 8-GPU box the decode path
parallelises in two ways, one process per GPU (``torch.distributed``, NCCL over NVLink):

* **Row sharding** (long batches): decode rows are independent -- row ``b``'s output depends
  only on its own table and length -- so each rank owns the rows
  ``[rank * B / world, (rank + 1) * B / world)`` with its own pool, block table and seqlen.
  There is no collective on the data path. :func:`shard_rows` is the split.
* **Context parallel** (long contexts): every rank owns a contiguous token range of every
  row (its slice of the block table, its own pool). Each rank computes the split-KV triple
  ``(m, l, acc)`` of its range with one ``pd_decode_partials`` launch, the triples are
  exchanged with ONE ``all_gather_into_tensor`` of a packed fp32 buffer
  ``[acc (B*H*D) | m (B*H) | l (B*H)]`` per rank, and each rank merges all parts with
  ``pd_lse_merge`` (the log-sum-exp rule, acc / max(l, 1) over the union), so every rank
  ends with the full output. Remote partials only ever reach a kernel through NCCL into a
  local buffer; no kernel reads peer memory.

The gathered tensor lives in this rank's memory and the merge reads it with strided part
offsets, so nothing is copied after the collective.
"""

from __future__ import annotations

import math
from typing import Callable

import torch

from model import _native

__all__ = ["shard_rows", "shard_tokens", "ContextParallelDecode"]

_LOG2E = 1.4426950408889634


def shard_rows(n_rows: int, rank: int, world: int) -> tuple[int, int]:
    """Contiguous row range ``[lo, hi)`` of ``rank``; the ranges tile ``[0, n_rows)``."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return rank * n_rows // world, (rank + 1) * n_rows // world


def shard_tokens(context: int, rank: int, world: int, block_size: int) -> tuple[int, int]:
    """Contiguous token range of ``rank`` for context parallelism, cut at block boundaries."""
    lo_blk, hi_blk = shard_rows(-(-context // block_size), rank, world)
    return min(context, lo_blk * block_size), min(context, hi_blk * block_size)


class ContextParallelDecode:
    """One decode step for rows whose tokens are spread over the ranks of ``group``.

    ``partials`` and ``merge`` default to the sm_100a kernels; a test on CPU ranks may pass
    callables with the same signatures (this is how the gloo tests drive the exchange logic).
    Without an initialised process group the object stands for a world of one: the step is the
    partials launch and the merge of that single part, with no collective.

    Every buffer (the send and gathered partials, the workspace and, unless the caller passes
    ``out``, the result) is allocated on the first call and reused while the shape stays, so a
    steady decode loop allocates nothing and its step can be captured in a CUDA graph (the
    NCCL all-gather included, as torch supports).
    """

    def __init__(self, group=None, *, partials: Callable | None = None, merge: Callable | None = None):
        import torch.distributed as dist

        self.dist = dist if dist.is_available() and dist.is_initialized() else None
        self.group = group
        self.world = self.dist.get_world_size(group) if self.dist is not None else 1
        self.rank = self.dist.get_rank(group) if self.dist is not None else 0
        self._partials = partials or self._native_partials
        self._merge = merge or self._native_merge
        self._workspace: torch.Tensor | None = None
        self._send: torch.Tensor | None = None
        self._recv: torch.Tensor | None = None
        self._out: torch.Tensor | None = None

    # ---------------------------------------------------------------- default kernels
    def _native_partials(self, q, k_cache, v_cache, block_table, seqlen, m, l, acc, scale):
        B, H, D = q.shape
        need = _native.workspace_bytes(B, H, k_cache.shape[2], D, q.dtype)
        if self._workspace is None or self._workspace.numel() < need or self._workspace.device != q.device:
            self._workspace = torch.empty(max(need, 256), dtype=torch.uint8, device=q.device)
        _native.decode_partials(q, k_cache, v_cache, block_table, seqlen, m, l, acc, scale * _LOG2E,
                                self._workspace)

    @staticmethod
    def _native_merge(m_parts, l_parts, acc_parts, out):
        _native.lse_merge(m_parts, l_parts, acc_parts, out)

    # ---------------------------------------------------------------- step
    def buffers(self, B: int, H: int, D: int, device) -> tuple[torch.Tensor, torch.Tensor]:
        """The packed send buffer of this rank and the gathered buffer of all ranks (the same
        tensor in a world of one)."""
        n = B * H * (D + 2)
        if self._send is None or self._send.numel() != n or self._send.device != torch.device(device):
            self._send = torch.empty(n, dtype=torch.float32, device=device)
            self._recv = (self._send if self.world == 1
                          else torch.empty(self.world * n, dtype=torch.float32, device=device))
        return self._send, self._recv

    @staticmethod
    def views(buf: torch.Tensor, B: int, H: int, D: int, parts: int | None = None):
        """(acc, m, l) views of a packed buffer (one part) or a gathered one (``parts`` parts)."""
        bhd, bh = B * H * D, B * H
        if parts is None:
            return buf[:bhd].view(B, H, D), buf[bhd:bhd + bh].view(B, H), buf[bhd + bh:].view(B, H)
        stride = bhd + 2 * bh
        acc = torch.as_strided(buf, (parts, B, H, D), (stride, H * D, D, 1))
        m = torch.as_strided(buf, (parts, B, H), (stride, H, 1), storage_offset=bhd)
        l = torch.as_strided(buf, (parts, B, H), (stride, H, 1), storage_offset=bhd + bh)
        return acc, m, l

    def __call__(self, q, k_cache, v_cache, block_table, local_seqlen, *, scale: float | None = None,
                 out: torch.Tensor | None = None, events=None) -> torch.Tensor:
        """``q`` (B, H, D) is the same on every rank; ``local_seqlen`` counts this rank's tokens.

        ``events`` (optional): four CUDA events recorded on the current stream before the
        partials launch, after it, after the all-gather and after the merge, so a caller can
        time the compute and the collective apart."""
        B, H, D = q.shape
        if scale is None:
            scale = 1.0 / math.sqrt(D)
        send, recv = self.buffers(B, H, D, q.device)
        acc, m, l = self.views(send, B, H, D)
        if events is not None:
            events[0].record()
        self._partials(q, k_cache, v_cache, block_table, local_seqlen, m, l, acc, scale)
        if events is not None:
            events[1].record()
        if self.world > 1:
            self.dist.all_gather_into_tensor(recv, send, group=self.group)
        if events is not None:
            events[2].record()
        acc_p, m_p, l_p = self.views(recv, B, H, D, parts=self.world)
        if out is None:
            if (self._out is None or self._out.shape != q.shape or self._out.dtype != q.dtype
                    or self._out.device != q.device):
                self._out = torch.empty_like(q)
            out = self._out
        self._merge(m_p, l_p, acc_p, out)
        if events is not None:
            events[3].record()
        return out
