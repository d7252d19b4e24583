"""Multi-rank logic on CPU ranks (gloo, world size 2): the same exchange code the NCCL path
runs, with the CPU oracle standing in for the two kernels (test-only injection).

* context parallel: each rank decodes its token slice of every row, the packed
  (acc | m | l) buffers are all-gathered, the LSE merge of all parts equals the oracle on the
  whole rows;
* row sharding: the shards tile the batch and each rank's rows decode like the same rows
  of the full batch;
* failure: a rank that leaves between steps (before the exchange) makes the surviving rank's
  next exchange end with an error inside the process-group timeout instead of waiting forever.
"""

from __future__ import annotations

import os
import socket
import sys
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank: int, world: int, port: int, results):
    for path in (ROOT / "llm-serving_b200", ROOT, ROOT / "tests"):
        sys.path.insert(0, str(path))
    import torch.distributed as dist

    from helpers import build_case
    from model.parallel_decode import ContextParallelDecode, shard_rows, shard_tokens
    from oracle import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        bs = 16
        lengths = [300, 45, 512, 1, 0, 200]
        q, k, v, table, seqlen = build_case(len(lengths), 8, 2, 32, bs, lengths, seed=21)
        whole, _ = oracle.paged_decode(q, k, v, table, seqlen)

        # ---- context parallel: this rank's token range of every row (table columns)
        lo, hi = shard_tokens(max(lengths), rank, world, bs)
        local_table = table[:, lo // bs: -(-hi // bs)].contiguous()
        local_len = (seqlen - lo).clamp(0, hi - lo).to(torch.int32)

        def partials(q_, k_, v_, table_, seqlen_, m, l, acc, scale):
            mm, ll, aa = oracle.decode_partials(q_, k_, v_, table_, seqlen_, scale=scale)
            m.copy_(mm), l.copy_(ll), acc.copy_(aa)

        def merge(m_p, l_p, acc_p, out):
            merged, _ = oracle.lse_merge(m_p.contiguous(), l_p.contiguous(), acc_p.contiguous())
            out.copy_(merged)

        cp = ContextParallelDecode(partials=partials, merge=merge)
        got = cp(q, k, v, local_table, local_len)
        cp_err = (got - whole).abs().max().item()

        # ---- row sharding: no collective, each rank decodes its rows only
        r0, r1 = shard_rows(len(lengths), rank, world)
        part, _ = oracle.paged_decode(q[r0:r1], k, v, table[r0:r1], seqlen[r0:r1])
        row_err = (part - whole[r0:r1]).abs().max().item() if r1 > r0 else 0.0
        results[rank] = (cp_err, row_err, (r0, r1))
    finally:
        dist.destroy_process_group()


def test_context_parallel_and_row_sharding_on_two_cpu_ranks():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0, f"rank exited with {p.exitcode}"
    ranges = []
    for rank in range(world):
        cp_err, row_err, rows = results[rank]
        assert cp_err < 2e-6, f"rank {rank}: context-parallel merge differs by {cp_err}"
        assert row_err == 0.0
        ranges.append(rows)
    assert ranges[0][0] == 0 and ranges[-1][1] == 6 and ranges[0][1] == ranges[1][0]


def _leaving_worker(rank: int, world: int, port: int, results):
    for path in (ROOT / "llm-serving_b200", ROOT, ROOT / "tests"):
        sys.path.insert(0, str(path))
    from datetime import timedelta

    import torch.distributed as dist

    from model.parallel_decode import ContextParallelDecode

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    dist.barrier()
    if rank == 1:
        os._exit(3)  # leaves between steps: nothing of it is in flight

    def partials(q_, k_, v_, table_, seqlen_, m, l, acc, scale):
        m.zero_(), l.zero_(), acc.zero_()

    cp = ContextParallelDecode(partials=partials, merge=lambda *a: None)
    q = torch.zeros(2, 4, 8)
    try:
        cp(q, None, None, None, None)
        results[rank] = "no error"
    except Exception as exc:  # noqa: BLE001 - the test inspects the type name
        results[rank] = type(exc).__name__
    os._exit(0)


def test_a_rank_that_leaves_ends_the_next_exchange_with_an_error():
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_leaving_worker, args=(r, world, port, results)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    codes = [p.exitcode for p in procs]
    for p in procs:
        if p.exitcode is None:
            p.kill()
    assert codes == [0, 3], codes
    assert results[0] != "no error", "the exchange with a departed rank returned normally"


def test_shard_helpers_tile_their_ranges():
    sys.path.insert(0, str(ROOT / "llm-serving_b200"))
    from model.parallel_decode import shard_rows, shard_tokens

    for n, world in ((1024, 8), (7, 3), (1, 4), (0, 2)):
        spans = [shard_rows(n, r, world) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    for ctx_len, world in ((8192, 8), (8192, 3), (100, 4)):
        spans = [shard_tokens(ctx_len, r, world, 16) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == ctx_len
        assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
        assert all(lo % 16 == 0 for lo, _ in spans)
    with pytest.raises(ValueError):
        shard_rows(8, 3, 2)


def test_a_world_of_one_merges_its_single_part_without_a_process_group():
    """Without an initialised process group the context-parallel step is the partials of the
    whole rows and the merge of that one part (no collective), and it reuses its buffers."""
    sys.path.insert(0, str(ROOT / "llm-serving_b200"))
    sys.path.insert(0, str(ROOT / "tests"))
    from helpers import build_case
    from model.parallel_decode import ContextParallelDecode
    from oracle import oracle

    q, k, v, table, seqlen = build_case(4, 8, 2, 32, 16, [100, 0, 33, 64], seed=3)
    whole, _ = oracle.paged_decode(q, k, v, table, seqlen)

    def partials(q_, k_, v_, table_, seqlen_, m, l, acc, scale):
        mm, ll, aa = oracle.decode_partials(q_, k_, v_, table_, seqlen_, scale=scale)
        m.copy_(mm), l.copy_(ll), acc.copy_(aa)

    def merge(m_p, l_p, acc_p, out):
        merged, _ = oracle.lse_merge(m_p.contiguous(), l_p.contiguous(), acc_p.contiguous())
        out.copy_(merged)

    cp = ContextParallelDecode(partials=partials, merge=merge)
    assert cp.world == 1 and cp.dist is None
    first = cp(q, k, v, table, seqlen)
    send, recv = cp.buffers(*q.shape, q.device)
    assert recv is send
    again = cp(q, k, v, table, seqlen)
    assert again is first  # the result buffer is reused
    assert (again - whole).abs().max().item() < 2e-6
