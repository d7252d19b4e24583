"""Seeded synthetic paged-decode workloads with the shapes of the five benchmark configs.

There is no dataset on this path: every config is synthetic by definition (random K/V and
queries, seeded lengths and block tables). Block tables come from :class:`BlockManager`,
the same allocator the engine uses, so fragmentation is what the serving stack produces.

* ``config1``: B=8, Qwen3-0.6B heads (16 q / 8 kv, D=128), L ~ U[128, 1024], block size 16,
  a 1024-block pool whose blocks are handed out by a seeded random permutation.
* ``config2``: the decode step of the 28-layer model through the paged pool: B=32, every
  row at context 2048 (+ the step index), 28 distinct per-layer pools of
  ``32 * ceil((2048 + 64) / 16) = 4224`` blocks, tables reserved smallest-id first.
* ``config3``: B=64, L = clip(round(exp(ln 512 + N(0, 1))), 16, 8192); the free list is
  fragmented by a seeded history of reserve/free calls before the rows are reserved.
* ``config4``: B=32, every row at 8192 tokens (long-context split-KV). ``shard(rank,
  world)`` keeps rank's contiguous 8192/world token range of every row.
* ``config5``: 1024 rows, L ~ U[256, 4096], sharded by row index over the ranks.
* ``qwen35``: the hybrid Qwen3.5-0.8B engine's full-attention layers (H=8, H_kv=2, D=256,
  four q heads per kv head; 6 layers), B=32 rows at context 2048, block size 16.

K/V/q are N(0, 1) in bf16 (scale 1/sqrt(D)). Large pools are drawn with a CUDA generator.

This is benchmark and test input generation, not part of the library: ``bench.py`` and
``tests/`` import it (with ``llm-serving_b200/`` on the import path for the block manager).
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from serve.block_manager import BlockManager

QWEN3_H, QWEN3_HKV, QWEN3_D = 16, 8, 128


@dataclass
class PagedWorkload:
    """One paged-decode problem: per-layer pools, shared table/seqlen, one query per layer."""

    name: str
    q: list[torch.Tensor]          # per layer (B, H, D)
    k_pools: list[torch.Tensor]    # per layer (n_blocks, bs, H_kv, D)
    v_pools: list[torch.Tensor]
    block_table: torch.Tensor      # (B, max_blocks) int32
    seqlen: torch.Tensor           # (B,) int32
    tables: list[list[int]] = field(default_factory=list)
    meta: dict = field(default_factory=dict)

    @property
    def n_layer(self) -> int:
        return len(self.k_pools)

    def kv_bytes_per_layer(self) -> int:
        """Algorithmic K+V bytes one layer reads: sum(seqlen) * 2 * H_kv * D * itemsize."""
        _, _, hkv, d = self.k_pools[0].shape
        es = self.k_pools[0].element_size()
        return int(self.seqlen.to(torch.int64).sum().item()) * 2 * hkv * d * es


def _randn(shape, gen, device, dtype):
    return torch.randn(shape, generator=gen, device=gen.device, dtype=torch.float32).to(device=device, dtype=dtype)


def _generator(seed: int, device) -> torch.Generator:
    device = torch.device(device)
    return torch.Generator(device=device if device.type == "cuda" else "cpu").manual_seed(seed)


def _table_tensor(tables: list[list[int]], device) -> torch.Tensor:
    width = max(1, max(len(t) for t in tables))
    out = torch.zeros(len(tables), width, dtype=torch.int32)
    for row, t in enumerate(tables):
        if t:
            out[row, : len(t)] = torch.tensor(t, dtype=torch.int32)
    return out.to(device)


def _build(name, lengths, tables, n_blocks, *, n_layer=1, H=QWEN3_H, H_kv=QWEN3_HKV, D=QWEN3_D,
           block_size=16, device="cuda", dtype=torch.bfloat16, seed=0, meta=None) -> PagedWorkload:
    gen = _generator(seed, device)
    B = len(lengths)
    k_pools, v_pools, qs = [], [], []
    for _ in range(n_layer):
        k_pools.append(_randn((n_blocks, block_size, H_kv, D), gen, device, dtype))
        v_pools.append(_randn((n_blocks, block_size, H_kv, D), gen, device, dtype))
        qs.append(_randn((B, H, D), gen, device, dtype))
    seqlen = torch.tensor(lengths, dtype=torch.int32, device=device)
    return PagedWorkload(name, qs, k_pools, v_pools, _table_tensor(tables, device), seqlen,
                         tables=tables, meta=dict(meta or {}))


def config1(device="cuda", seed=0, dtype=torch.bfloat16, n_layer=1) -> PagedWorkload:
    gen = torch.Generator().manual_seed(seed)
    B, bs, n_blocks = 8, 16, 1024
    lengths = torch.randint(128, 1025, (B,), generator=gen).tolist()
    perm = torch.randperm(n_blocks, generator=gen).tolist()
    tables, cursor = [], 0
    for n in lengths:
        pages = -(-n // bs)
        tables.append(perm[cursor: cursor + pages])
        cursor += pages
    return _build("config1", lengths, tables, n_blocks, n_layer=n_layer, device=device, dtype=dtype,
                  seed=seed + 1, meta={"B": B, "block_size": bs, "n_blocks": n_blocks})


def config2(device="cuda", seed=0, dtype=torch.bfloat16, n_layer=28, context=2048, new_tokens=64,
            batch=32) -> PagedWorkload:
    bs = 16
    manager = BlockManager(batch * -(-(context + new_tokens) // bs), bs)
    tables = [manager.reserve(manager.blocks_for(context, new_tokens)) for _ in range(batch)]
    lengths = [context] * batch
    return _build("config2", lengths, tables, manager.n_blocks, n_layer=n_layer, device=device,
                  dtype=dtype, seed=seed + 2,
                  meta={"B": batch, "context": context, "new_tokens": new_tokens, "block_size": bs,
                        "n_blocks": manager.n_blocks})


def fragmented_tables(lengths: list[int], n_blocks: int, block_size: int, seed: int,
                      churn: int = 256) -> list[list[int]]:
    """Tables for ``lengths`` from a BlockManager whose free list a seeded history fragmented.

    History: ``churn`` rounds; each reserves a dummy request of 1..64 blocks (if it fits) and,
    with probability 1/2, frees a random live dummy. Smallest-first reservations refill the
    holes during the churn, so a random half of the dummies still live is then freed (finished
    requests), leaving holes of many sizes. Every row then reserves its blocks -- its table
    threads through those holes -- and the remaining dummies stay allocated (other requests'
    KV).
    """
    import random

    rng = random.Random(seed)
    manager = BlockManager(n_blocks, block_size)
    live: list[list[int]] = []
    for _ in range(churn):
        ids = manager.reserve(rng.randint(1, 64))
        if ids is not None:
            live.append(ids)
        if live and rng.random() < 0.5:
            manager.free(live.pop(rng.randrange(len(live))))
    for _ in range(len(live) // 2):
        manager.free(live.pop(rng.randrange(len(live))))
    while live and manager.stats()["free"] < sum(-(-n // block_size) for n in lengths):
        manager.free(live.pop(rng.randrange(len(live))))
    tables = []
    for n in lengths:
        ids = manager.reserve(manager.blocks_for(n, 0))
        if ids is None:
            raise RuntimeError("pool too small for the config-3 rows")
        tables.append(ids)
    return tables


def lognormal_lengths(batch: int, seed: int, median: int = 512, sigma: float = 1.0,
                      low: int = 16, high: int = 8192) -> list[int]:
    gen = torch.Generator().manual_seed(seed)
    z = torch.randn(batch, generator=gen, dtype=torch.float64)
    raw = torch.exp(math.log(median) + sigma * z).round().to(torch.int64)
    return raw.clamp(low, high).tolist()


def config3(device="cuda", seed=0, dtype=torch.bfloat16, n_layer=1, batch=64) -> PagedWorkload:
    bs = 16
    lengths = lognormal_lengths(batch, seed)
    n_blocks = 2 * sum(-(-n // bs) for n in lengths) + 4096
    tables = fragmented_tables(lengths, n_blocks, bs, seed)
    return _build("config3", lengths, tables, n_blocks, n_layer=n_layer, device=device, dtype=dtype,
                  seed=seed + 3, meta={"B": batch, "block_size": bs, "n_blocks": n_blocks})


def config4(device="cuda", seed=0, dtype=torch.bfloat16, n_layer=1, batch=32, context=8192,
            rank=0, world=1) -> PagedWorkload:
    """Rank's contiguous ``context / world`` token slice of every row (its own pool and table)."""
    bs = 16
    span = context // world
    pages = -(-span // bs)
    manager = BlockManager(batch * pages, bs)
    tables = [manager.reserve(pages) for _ in range(batch)]
    return _build("config4", [span] * batch, tables, manager.n_blocks, n_layer=n_layer, device=device,
                  dtype=dtype, seed=seed + 4 + 1000 * rank,
                  meta={"B": batch, "context": context, "rank": rank, "world": world,
                        "token_begin": rank * span, "block_size": bs})


def config5_lengths(seed: int = 0, rows: int = 1024) -> list[int]:
    gen = torch.Generator().manual_seed(seed)
    return torch.randint(256, 4097, (rows,), generator=gen).tolist()


def config5(device="cuda", seed=0, dtype=torch.bfloat16, n_layer=1, rank=0, world=1, rows=1024) -> PagedWorkload:
    """Rows ``[rank * rows / world, (rank + 1) * rows / world)`` of the 1024-row sweep."""
    bs = 16
    all_lengths = config5_lengths(seed, rows)
    lo, hi = rank * rows // world, (rank + 1) * rows // world
    lengths = all_lengths[lo:hi]
    manager = BlockManager(sum(-(-n // bs) for n in lengths), bs)
    tables = [manager.reserve(manager.blocks_for(n, 0)) for n in lengths]
    return _build("config5", lengths, tables, manager.n_blocks, n_layer=n_layer, device=device, dtype=dtype,
                  seed=seed + 5 + 1000 * rank,
                  meta={"rows": rows, "row_begin": lo, "row_end": hi, "rank": rank, "world": world,
                        "block_size": bs})


QWEN35_H, QWEN35_HKV, QWEN35_D = 8, 2, 256


def qwen35(device="cuda", seed=0, dtype=torch.bfloat16, n_layer=6, context=2048, batch=32) -> PagedWorkload:
    """Full-attention decode of the hybrid Qwen3.5 engine at config-2 batch and context."""
    bs = 16
    manager = BlockManager(batch * -(-(context + 64) // bs), bs)
    tables = [manager.reserve(manager.blocks_for(context, 64)) for _ in range(batch)]
    return _build("qwen35", [context] * batch, tables, manager.n_blocks, n_layer=n_layer, H=QWEN35_H,
                  H_kv=QWEN35_HKV, D=QWEN35_D, device=device, dtype=dtype, seed=seed + 35,
                  meta={"B": batch, "context": context, "block_size": bs, "n_blocks": manager.n_blocks})
