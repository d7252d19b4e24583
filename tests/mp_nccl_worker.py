"""One rank of the multi-GPU parity check (launched by ``test_multigpu_gpu.py`` under torchrun).

Each rank owns one B200 and talks to the others over NCCL:

* context parallel (B=32 x 8192 tokens): every rank decodes its
  block-aligned token slice of every row with ``pd_decode_partials``; ``ContextParallelDecode``
  all-gathers the packed (acc | m | l) buffers and merges them with ``pd_lse_merge``. The
  merged output must be within the suite's tolerance of the fp32 oracle on a row subset
  (checked on every rank, which builds the same seeded pool) and bitwise identical on all
  ranks; its distance to the single-GPU decode is reported;
* row sharding: each rank decodes only its rows, with its own pool and
  table and no collective on the data path; a seeded subset of its rows is checked against
  the CPU oracle.

Rank 0 writes a JSON summary to the path given as the first argument.
"""

from __future__ import annotations

import json
import math
import os
import sys
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for path in (ROOT / "llm-serving_b200", ROOT, ROOT / "tests"):
    sys.path.insert(0, str(path))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402


def main(out_path: str) -> int:
    from helpers import assert_output_close, oracle_rows
    from model import _native
    from model.parallel_decode import ContextParallelDecode, shard_tokens
    from model.triton_decode import paged_decode
    from oracle import oracle
    import workloads

    local = int(os.environ["LOCAL_RANK"])
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=device)
    rank, world = dist.get_rank(), dist.get_world_size()
    summary = {"world": world}
    failures: list[str] = []

    def check(name, fn):
        """Host-side checks record their failure instead of raising, so that every rank
        still takes the same collective steps in the same order."""
        try:
            fn()
        except Exception as exc:  # noqa: BLE001 - reported below
            failures.append(f"rank {rank} {name}: {type(exc).__name__}: {exc}")

    # ---- context parallel over NCCL (config 4)
    wl = workloads.config4(device)
    q, k, v = wl.q[0], wl.k_pools[0], wl.v_pools[0]
    whole = paged_decode(q, k, v, wl.block_table, wl.seqlen)
    bs = 16
    lo, hi = shard_tokens(8192, rank, world, bs)
    local_table = wl.block_table[:, lo // bs: hi // bs].contiguous()
    local_len = (wl.seqlen - lo).clamp(0, hi - lo).to(torch.int32)
    cp = ContextParallelDecode()
    got = cp(q, k, v, local_table, local_len, scale=1.0 / math.sqrt(q.shape[2]))   # all-gather 1
    torch.cuda.synchronize()
    cp_err = (got.float() - whole.float()).abs().max().item()
    rows = torch.arange(0, q.shape[0], 8)
    ref = oracle_rows(oracle, q, k, v, wl.block_table, wl.seqlen, rows)
    check("config4 vs oracle", lambda: assert_output_close(got[rows].cpu(), ref, torch.bfloat16))
    gathered = torch.empty((world,) + tuple(got.shape), dtype=got.dtype, device=device)
    dist.all_gather_into_tensor(gathered, got)                                        # all-gather 2
    same = all(torch.equal(gathered[0], gathered[r]) for r in range(world))
    summary.update(cp_max_abs_vs_single_gpu=cp_err, cp_identical_on_all_ranks=same)
    check("single-GPU config4 vs oracle", lambda: assert_output_close(whole[rows].cpu(), ref, torch.bfloat16))
    if not same:
        failures.append(f"rank {rank}: ranks disagree on the merged output")

    # ---- row sharding, no collective on the data path (config 5)
    shard = workloads.config5(device, rank=rank, world=world)
    out = paged_decode(shard.q[0], shard.k_pools[0], shard.v_pools[0], shard.block_table, shard.seqlen)
    n = shard.q[0].shape[0]
    sub = torch.arange(0, n, max(1, n // 16))
    ref = oracle_rows(oracle, shard.q[0], shard.k_pools[0], shard.v_pools[0], shard.block_table,
                       shard.seqlen, sub)
    check("config5 rows vs oracle", lambda: assert_output_close(out[sub].cpu(), ref, torch.bfloat16))
    rows_done = torch.tensor([n], device=device)
    dist.all_reduce(rows_done)                                                         # all-reduce 3
    summary.update(rows_total=int(rows_done.item()))
    if int(rows_done.item()) != 1024:
        failures.append(f"rank {rank}: shards cover {int(rows_done.item())} rows, not 1024")
    if _native.device_error() != 0:
        failures.append(f"rank {rank}: device error word set")
    for line in failures:
        print(line, file=sys.stderr, flush=True)
    ok = torch.tensor([0.0 if failures else 1.0], device=device)
    dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    passed = bool(ok.item() == 1)
    if rank == 0:
        summary["passed"] = passed
        Path(out_path).write_text(json.dumps(summary))
    dist.destroy_process_group()
    return 0 if passed else 1


if __name__ == "__main__":
    raise SystemExit(main(sys.argv[1]))
