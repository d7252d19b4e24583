"""CUDA-graph capture of a paged decode step: its attention alone, or the whole model's step.

One decode step of the engine's paged arm issues, per step, ``build_mask`` (``seqlen :=
pos + 1``), then for every layer ``PagedKV.write`` + ``PagedKV.attend`` (one fused append +
decode launch each), then ``advance``. The Python work around those launches costs about as
much host time per layer as the kernel takes on the GPU, so an eager step can leave the GPU
waiting. :class:`PagedStepGraph` captures the step once and replays it: one graph launch per
step, the GPU never waits on Python. :class:`DecodeStepGraph` does the same for a whole
model's step (projections, norms, MLP, sampling) around the same container calls.

Capture is possible because everything the step touches has a stable address: the pools,
the int32 block table and seqlen, the int64 ``pos``/``valid``/``active`` tensors (all updated
in place), the decode plan's workspace, and the caller's input buffers. The decode kernel keeps
its split-row epoch in the workspace and advances it itself, so every replay is a fresh launch
as far as its arrival counters are concerned. What a graph cannot replay is the container's
host-side bookkeeping (the Python mirrors of ``pos``/``valid`` and the bound checks); the
helper performs it on the host around each replay.

The reference engine has no paged graph path (its ``serve/graph.py`` design is seat-only and
parked); this module is that missing piece for the paged arm.
"""

from __future__ import annotations

import torch

from model import _native
from model.paged import PagedKV

__all__ = ["PagedStepGraph", "DecodeStepGraph"]


class DecodeStepGraph:
    """One captured decode step of a whole model that drives a :class:`PagedKV` container.

    ``body()`` issues the step's device work between ``build_mask`` and ``advance``: every
    layer's projections, ``kv.write`` / ``kv.attend`` and the rest of the model, reading and
    writing only tensors with stable addresses (inputs the caller refills before each
    :meth:`replay`, outputs it reads after). ``prepare`` is a query-shaped tensor for the
    container's decode plan (``(B, H, 1, D)``, any contents). The container's host-side
    bookkeeping runs around each replay, as in :class:`PagedStepGraph`.
    """

    def __init__(self, kv: PagedKV, body, prepare: torch.Tensor, *, next_token: bool = True) -> None:
        if not isinstance(kv, PagedKV):
            raise TypeError(f"DecodeStepGraph needs a PagedKV, got {type(kv).__name__}")
        self.kv = kv
        self.next_token = bool(next_token)
        kv.pool.flush()
        kv.prepare(prepare)
        torch.cuda.synchronize(prepare.device)
        snapshot = kv._host_snapshot()
        self.graph = torch.cuda.CUDAGraph()
        before = _native.launch_count()
        try:
            with torch.cuda.graph(self.graph):
                kv.build_mask(next_token=self.next_token)
                body()
                kv.advance()
        finally:
            kv._host_restore(snapshot)
        #: Library kernels launched by one replay.
        self.launches_per_step = _native.launch_count() - before

    def replay(self) -> None:
        kv = self.kv
        kv._replayed_step(self.next_token)
        self.graph.replay()
        kv._replayed_advance()


class PagedStepGraph:
    """One captured decode step (attention part) of a :class:`PagedKV` container.

    ``q`` ``(n_layer, B, H, 1, D)`` and ``k``/``v`` ``(n_layer, B, H_kv, 1, D)`` are device
    buffers the caller refills before each :meth:`replay` (their addresses are baked into the
    graph). :attr:`out` ``(n_layer, B, H, 1, D)`` receives every layer's attention output.
    ``rope`` = (cos, sin) device buffers of the step's per-row rotary tables, (B, 1, R/2):
    then ``k`` holds K before its rotary embedding, which the fused append applies.
    """

    def __init__(self, kv: PagedKV, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, *,
                 next_token: bool = True, rope=None) -> None:
        if not isinstance(kv, PagedKV):
            raise TypeError(f"PagedStepGraph needs a PagedKV, got {type(kv).__name__}")
        n = kv.n_layer
        q_shape = (n, kv.batch, kv.n_head, 1, kv.head_dim)
        kv_shape = (n, kv.batch, kv.n_kv_head, 1, kv.head_dim)
        if tuple(q.shape) != q_shape or tuple(k.shape) != kv_shape or tuple(v.shape) != kv_shape:
            raise ValueError(
                f"PagedStepGraph needs q {q_shape} and k/v {kv_shape}; got "
                f"{tuple(q.shape)} / {tuple(k.shape)} / {tuple(v.shape)}"
            )
        for name, t in (("q", q), ("k", k), ("v", v)):
            if t.device.type != "cuda" or t.dtype != kv.dtype:
                raise ValueError(f"{name} must be a {kv.dtype} CUDA tensor, got {t.dtype} on {t.device}")
        self.kv = kv
        self.q, self.k, self.v = q, k, v
        self.rope = rope
        self.next_token = bool(next_token)
        self.out = torch.empty(q_shape, dtype=kv.dtype, device=q.device)

        kv.pool.flush()
        kv.prepare(q[0])
        torch.cuda.synchronize(q.device)
        snapshot = kv._host_snapshot()
        self.graph = torch.cuda.CUDAGraph()
        before = _native.launch_count()
        try:
            with torch.cuda.graph(self.graph):
                kv.build_mask(next_token=self.next_token)
                for layer in range(n):
                    kv.write(layer, k[layer], v[layer], rope=rope)
                    kv.attend(layer, q[layer], out=self.out[layer])
                kv.advance()
        finally:
            kv._host_restore(snapshot)  # capture ran the host side once without the device side
        #: Library kernels launched by one replay.
        self.launches_per_step = _native.launch_count() - before

    def replay(self) -> torch.Tensor:
        """Run one step: host-side checks, one graph launch, host-side position update.
        Returns :attr:`out` (overwritten by the next replay)."""
        kv = self.kv
        kv._replayed_step(self.next_token)
        self.graph.replay()
        kv._replayed_advance()
        return self.out
