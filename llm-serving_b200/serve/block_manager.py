"""Paged-KV block allocator and fragmentation accounting (host side, stdlib only).

Drop-in for the reference's ``serve/block_manager.py`` (``BlockManager`` 32-143,
``FragStats`` 146-239): the same API, ids and accounting, so the block tables it produces are
identical to the reference's for the same sequence of calls. That matters for the length-skew
workload, whose fragmented tables come from a seeded reserve/free history.

Allocation contract (reference D6): a request reserves ``ceil((prompt + budget) / block_size)``
blocks up front, all or nothing, and frees them all at once; ids come out smallest first.
The free set is kept as an ascending list: ``reserve(n)`` takes its first ``n`` entries and
``free`` merges the returned ids back in order.
"""

from __future__ import annotations

from typing import Sequence

__all__ = ["BlockManager", "FragStats"]


def _count(name: str, value, *, allow_zero: bool) -> int:
    low = 0 if allow_zero else 1
    if isinstance(value, bool) or not isinstance(value, int) or value < low:
        kind = "non-negative" if allow_zero else "positive"
        raise ValueError(f"{name} must be a {kind} int, got {value!r}")
    return value


class BlockManager:
    """Deterministic free list of ``n_blocks`` physical blocks of ``block_size`` tokens."""

    def __init__(self, n_blocks: int, block_size: int) -> None:
        self.n_blocks = _count("n_blocks", n_blocks, allow_zero=False)
        self.block_size = _count("block_size", block_size, allow_zero=False)
        self._free: list[int] = list(range(n_blocks))  # ascending
        self._allocated: set[int] = set()
        self._peak = 0
        self._alloc_calls = 0
        self._free_calls = 0

    def reserve(self, n: int) -> list[int] | None:
        """The ``n`` smallest free ids, or ``None`` (pool untouched) if fewer are free."""
        n = _count("n", n, allow_zero=True)
        if n > len(self._free):
            return None
        if n == 0:
            return []
        ids = self._free[:n]
        del self._free[:n]
        self._allocated.update(ids)
        self._alloc_calls += 1
        self._peak = max(self._peak, len(self._allocated))
        return ids

    def free(self, ids: Sequence[int]) -> None:
        """Return every id; the whole call is validated before anything changes."""
        returned: list[int] = []
        seen: set[int] = set()
        for block_id in ids:
            if isinstance(block_id, bool) or not isinstance(block_id, int):
                raise ValueError(f"block ids must be ints, got {block_id!r}")
            if block_id in seen:
                raise ValueError(f"duplicate block id {block_id} in one free call")
            seen.add(block_id)
            if block_id not in self._allocated:
                raise ValueError(f"block {block_id} is not allocated")
            returned.append(block_id)
        if not returned:
            return
        self._allocated.difference_update(seen)
        self._free = sorted(self._free + returned)
        self._free_calls += 1

    @property
    def in_use(self) -> int:
        return len(self._allocated)

    @property
    def peak(self) -> int:
        return self._peak

    def stats(self) -> dict:
        in_use = len(self._allocated)
        return {
            "n_blocks": self.n_blocks,
            "block_size": self.block_size,
            "in_use": in_use,
            "free": len(self._free),
            "reserved": in_use,
            "peak": self._peak,
            "alloc_calls": self._alloc_calls,
            "free_calls": self._free_calls,
        }

    def blocks_for(self, prompt_len: int, budget: int) -> int:
        """``max(1, ceil((prompt_len + budget) / block_size))`` blocks for one request."""
        prompt_len = _count("prompt_len", prompt_len, allow_zero=True)
        budget = _count("budget", budget, allow_zero=True)
        return max(1, -(-(prompt_len + budget) // self.block_size))

    def __repr__(self) -> str:  # pragma: no cover - debugging aid
        return (f"BlockManager(n_blocks={self.n_blocks}, block_size={self.block_size}, "
                f"in_use={len(self._allocated)}, peak={self._peak})")


class FragStats:
    """Time-weighted internal fragmentation and reservation slack (reference D6 definitions).

    ``internal_frag = 1 - sum(written * dt) / sum(allocated_blocks * block_size * dt)``;
    ``reservation_slack = 1 - actual / reserved``; ``seat_row_slack`` is the seat arm's
    ``1 - live / row_width`` with the same time weighting. Samples with ``dt <= 0`` carry no
    time and are ignored.
    """

    def __init__(self, block_size: int) -> None:
        self.block_size = _count("block_size", block_size, allow_zero=False)
        self._written_dt = 0.0
        self._capacity_dt = 0.0
        self._seat_live_dt = 0.0
        self._seat_width_dt = 0.0

    def observe(self, dt_s: float, written_tokens: int, allocated_blocks: int) -> None:
        _count("written_tokens", written_tokens, allow_zero=True)
        _count("allocated_blocks", allocated_blocks, allow_zero=True)
        if dt_s <= 0 or allocated_blocks == 0:
            return
        self._written_dt += written_tokens * dt_s
        self._capacity_dt += allocated_blocks * self.block_size * dt_s

    def internal_frag(self) -> float | None:
        if self._capacity_dt <= 0:
            return None
        return 1.0 - self._written_dt / self._capacity_dt

    def reservation_slack(self, reserved_tokens: int, actual_tokens: int) -> float | None:
        if reserved_tokens <= 0:
            return None
        return 1.0 - actual_tokens / reserved_tokens

    def seat_row_slack(self, live_tokens: int, row_width: int, dt_s: float) -> float | None:
        _count("live_tokens", live_tokens, allow_zero=True)
        _count("row_width", row_width, allow_zero=True)
        if dt_s > 0 and row_width > 0:
            self._seat_live_dt += live_tokens * dt_s
            self._seat_width_dt += row_width * dt_s
        if self._seat_width_dt <= 0:
            return None
        return 1.0 - self._seat_live_dt / self._seat_width_dt
