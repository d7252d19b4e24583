"""Benchmark of the B200 paged-decode path (one JSON line on rank 0).

Workload (the 28-layer Qwen3-0.6B decode step through the paged pool):
B=32 rows, every context at 2048 tokens, block size 16, 16 q / 8 kv heads, head_dim 128,
bf16, 28 per-layer pools of 4224 blocks (7.75 GB of K/V, far larger than the 126 MB L2, so
every step reads cold HBM). One *step* = one decode step's attention for all 28 layers,
exactly as ``MiniLLM.forward`` drives ``PagedKV``: ``build_mask`` (seqlen := pos + 1), then
per layer ``write`` (records the new token) and ``attend`` (ONE launch that appends the
token to the paged pool and runs the block-table decode over it), then ``advance``. The
context grows by one token per step (2048 -> 2048 + steps). After ``--warmup`` eager steps
the step is captured once as a CUDA graph (``serve.graph.PagedStepGraph``) and every timed
step is one replay, so Python never sits between two kernels. ``gpu_launches`` = the
library launches one replay contains (counted at capture) x timed steps.

Reported (``metric`` is BASELINE.json's): ``value`` = KV HBM GB/s of the decode kernels over
the timed steps (sum of seqlen * 2 * H_kv * D * 2 B per layer-step, every rank, / max-over-
ranks device time); ``us_per_layer_step``; ``roofline`` of the decode kernel with its launch
duration bounded by the timed region / decode launches (a replay runs the decode launches back
to back plus six tiny bookkeeping kernels per step);
``e2e`` = the same metric through the public API with every step's q/k/v copied from pinned
host memory into a step graph's input buffers and all outputs copied back, the copies on a
second stream overlapping the neighbouring steps (two step graphs alternate);
``cpu_baseline`` = the reference's CPU gather + seat-decode path (ported, oracle/) on a
bounded sample of the same workload using every host core.

The same line carries the rest of the metric, each measured after the headline's timed region:
``decode_step`` / ``decode_tok_s`` = config 2's whole decode step (a random-init Qwen3-0.6B
around the same ``PagedKV`` calls, 64 greedy steps, CUDA graph per step) and the attention
share of it; ``seat`` / ``paged_over_seat`` = the attention part of the config-2 step against
the reference's seat (dense slab) step restated in torch, both as CUDA graphs; ``config5`` =
1024 rows sharded by index over the ranks (strong scaling, no collective); ``config4_cp`` =
32 x 8192 rows split by context over the ranks with one NCCL all-gather per layer-step,
compute and collective timed apart. Both sharded blocks carry an fp32 parity field.
``prefill`` = the block-table-aware chunked prefill on tcgen05 (4 rows x 512 new tokens after
2,048 cached, 28 layers, rank 0) with its fraction of the measured sustained bf16 peak.

``--impl reference`` times that CPU port alone (the reference's own CPU implementation of this
path; rank 0 only) and prints the same line with ``"impl": "reference"``.

Multi-GPU (``torchrun --nproc-per-node N``): for the headline, rows shard by sequence with no
collective, so every rank decodes its own B=32 batch (weak scaling); time is the max over ranks.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from datetime import timedelta
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "llm-serving_b200"))
sys.path.insert(0, str(ROOT))

import torch  # noqa: E402

METRIC = "paged-decode attn µs/layer-step & KV HBM GB/s vs 8 TB/s peak; decode tok/s"
N_LAYER, BATCH, CONTEXT, NEW_TOKENS = 28, 32, 2048, 64
H, H_KV, D, BS = 16, 8, 128, 16


def _peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": float(data["hbm_gbs"]), "bf16_tflops": float(data.get("bf16_tflops", 1590.0)),
                "bf16_tflops_sustained": float(data.get("bf16_tflops_sustained", 1400.0)), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi clock / throttle samples during the timed region (background process that
    writes to a temporary file; stopped with SIGINT so it flushes)."""

    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        import tempfile

        self.index = index
        self.proc = None
        self.path = Path(tempfile.mkstemp(prefix="clocks_", suffix=".csv")[1])

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits", "-i",
                 str(self.index), "-lms", "20", "-f", str(self.path)],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
            time.sleep(0.3)  # first sample before the timed region starts
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            import signal

            time.sleep(0.05)
            self.proc.send_signal(signal.SIGINT)
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        sm, max_sm, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        try:
            lines = self.path.read_text().splitlines()
            self.path.unlink()
        except OSError:
            lines = []
        for line in lines:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                max_sm = float(parts[2])
            except ValueError:
                continue
            for name, flag in zip(names, parts[5:9]):
                if flag.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": max_sm, "reasons": sorted(reasons), "samples": 0}
        loaded = [x for x in sm if max_sm is None or x >= 0.3 * max_sm] or sm
        return {"sm_mhz": statistics.median(loaded), "sm_max_mhz": max_sm, "reasons": sorted(reasons),
                "samples": len(sm)}


def _dist_setup(gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import torch.distributed as dist

        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
        return dist, dist.get_rank(), world, local
    return None, 0, 1, 0


def _max_over_ranks(dist, value: float, device) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _sum_over_ranks(dist, value: float, device) -> float:
    if dist is None:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.SUM)
    return float(t.item())


def _barrier(dist, device):
    torch.cuda.synchronize(device)
    if dist is not None:
        dist.barrier()
    torch.cuda.synchronize(device)


# ------------------------------------------------------------------------------ GPU arm


def _container(device, budget: int, seed: int):
    """The engine's paged arm at config-2 shape: BlockManager tables, a PagedPool of 28
    per-layer K/V pools filled with N(0, 1) bf16, and the PagedKV decode container."""
    from model.paged import PagedKV, PagedPool
    from serve.block_manager import BlockManager

    manager = BlockManager(BATCH * -(-(CONTEXT + budget) // BS), BS)
    tables = [manager.reserve(manager.blocks_for(CONTEXT, budget)) for _ in range(BATCH)]
    pool = PagedPool(N_LAYER, manager.n_blocks, BS, H_KV, D, dtype=torch.bfloat16, device=device, n_head=H)
    gen = torch.Generator(device=device).manual_seed(seed)
    for t in pool.keys + pool.values:
        t.copy_(torch.randn(t.shape, generator=gen, device=device))
    return PagedKV(pool, tables, [CONTEXT] * BATCH, rope_len=CONTEXT + budget, n_head=H)


def run_gpu(args) -> dict | None:
    from model import _native
    from serve.graph import PagedStepGraph

    dist, rank, world, local = _dist_setup(args.gpus)
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    steps, warmup = args.steps, args.warmup
    # tokens each row may still append: eager warm-up, graph warm-up, timed steps, e2e steps
    budget = max(NEW_TOKENS, warmup + 2 + 2 * steps + 1)
    kv = _container(device, budget, seed=rank)
    gen = torch.Generator(device=device).manual_seed(1234 + rank)
    # The step's per-layer inputs live in fixed device buffers (the captured graph reads them).
    q_buf = torch.randn(N_LAYER, BATCH, H, 1, D, generator=gen, device=device).to(torch.bfloat16)
    k_buf = torch.randn(N_LAYER, BATCH, H_KV, 1, D, generator=gen, device=device).to(torch.bfloat16)
    v_buf = torch.randn(N_LAYER, BATCH, H_KV, 1, D, generator=gen, device=device).to(torch.bfloat16)
    stream = torch.cuda.current_stream(device)

    def kv_bytes_of_step() -> int:
        # seqlen after build_mask(next_token=True) is pos + 1 for every row.
        return sum(p + 1 for p in kv._host_pos) * 2 * H_KV * D * 2 * N_LAYER

    def eager_step():
        kv.build_mask(next_token=True)
        for layer in range(N_LAYER):
            kv.write(layer, k_buf[layer], v_buf[layer])
            kv.attend(layer, q_buf[layer])
        kv.advance()

    for _ in range(warmup):  # eager steps: decode plan, kernels and allocator warmed up
        eager_step()
    graph = PagedStepGraph(kv, q_buf, k_buf, v_buf)
    for _ in range(2):
        graph.replay()
    assert _native.device_error() == 0, "device error word set during warm-up"

    # ---- device-resident timed region: one graph replay per step ----------------------
    kv_bytes = 0
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    _barrier(dist, device)
    with ClockSampler(local) as clocks:
        start.record(stream)
        for _ in range(steps):
            kv_bytes += kv_bytes_of_step()
            graph.replay()
        stop.record(stream)
        _barrier(dist, device)
    launches = graph.launches_per_step * steps
    ms_local = start.elapsed_time(stop)
    assert _native.device_error() == 0, "device error word set in the timed region"
    ms = _max_over_ranks(dist, ms_local, device)
    total_bytes = _sum_over_ranks(dist, float(kv_bytes), device)

    # ---- roofline of the decode kernel: inside a replay the decode launches run back to back
    # (one per layer, queued by the graph) and the only other work is the step's six tiny
    # bookkeeping kernels, so timed region / decode launches bounds one launch's duration from
    # above (achieved is a lower bound).
    per_launch_bytes = kv_bytes / (steps * N_LAYER)
    per_launch_ms = ms_local / (steps * N_LAYER)
    kernel_timing = ("CUDA events around the timed graph replays / decode launches (the amortised time per "
                     "launch; layers 1-27 overlap the previous layer's tail, so it is not one launch's span)")

    # ---- end to end through the public API with host buffers ---------------------------
    e2e = _run_e2e(kv, graph, device, stream, rank, steps, dist)
    del graph, kv, q_buf, k_buf, v_buf
    torch.cuda.empty_cache()

    # ---- the rest of the metric: config 2's whole decode step, the paged/seat step ratio,
    # and the two sharded configs (every rank takes the same collective steps in order)
    decode_step = run_decode_step(device, rank, dist)
    decode_step["attention_share"] = round((ms / steps) / decode_step["ms_per_step"], 3)
    sharded_reps = max(5, min(steps, 20))
    config5 = run_config5(device, rank, world, dist, reps=sharded_reps)
    config4_cp = run_config4_cp(device, rank, world, dist, steps=sharded_reps)
    seat = seat_case(device, "config2_b32_ctx2048", [CONTEXT] * BATCH) if rank == 0 else None
    # the block-table-aware chunked prefill on tcgen05 (one GPU, rank 0): 4 rows x 512 new tokens
    # after 2,048 cached ones, 28 layers
    prefill = prefill_case(device, _peaks(), 5, "tcgen05", *PREFILL_CASES[0]) if rank == 0 else None

    if rank != 0:
        _finish(dist)
        return None
    peaks = _peaks()
    achieved = per_launch_bytes / (per_launch_ms * 1e-3) / 1e9
    gbs = total_bytes / (ms * 1e-3) / 1e9
    traffic = _profiled_traffic(per_launch_bytes)
    line = {
        "metric": METRIC,
        "value": round(gbs, 1),
        "unit": "GB/s (KV bytes read by decode, all ranks)",
        "n_gpus": world,
        "steps": steps,
        "warmup": warmup,
        "ms_per_step": round(ms / steps, 4),
        "us_per_layer_step": round(ms * 1e3 / (steps * N_LAYER), 2),
        "decode_kernel_us_per_layer": round(per_launch_ms * 1e3, 2),
        "decode_tok_s_attention_only": round(world * BATCH * steps / (ms * 1e-3), 1),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V/q, random-init; no dataset on this path)",
        "config": {
            "workload": "BASELINE configs[1] attention path: 28-layer Qwen3-0.6B decode step through "
                        "PagedKV (append + block-table decode fused into one launch per layer), the "
                        "step captured once as a CUDA graph (serve.graph.PagedStepGraph) and replayed",
            "launch_overlap": "layers 1-27 are programmatic dependent launches: each one's prologue and "
                              "first K/V copies run while the previous layer's launch finishes; it waits "
                              "for that launch before reading q or the new K/V rows (layer 0 waits for "
                              "the step's seqlen update as usual)",
            "batch_per_gpu": BATCH, "context": f"{CONTEXT}+step", "layers": N_LAYER, "block_size": BS,
            "heads": f"{H}q/{H_KV}kv", "head_dim": D, "parallelism": f"rows sharded by sequence x{world}",
            "l2": "inputs larger than L2 (7.75 GB of per-layer pools per GPU; each layer reads 268 MB)",
        },
        "roofline": {
            "bound": "hbm", "achieved": round(achieved, 1), "peak": peaks["hbm_gbs"], "unit": "GB/s",
            "frac": round(achieved / peaks["hbm_gbs"], 4), "peak_source": peaks["source"],
            "traffic": traffic, "kernel": "pd_decode_kernel<bf16,128,2>",
            "algorithmic_bytes_per_launch": int(per_launch_bytes), "timing": kernel_timing,
        },
        "e2e": e2e,
        "gpu_launches": launches,
        "clocks": clocks.summary(),
        "decode_tok_s": decode_step["decode_tok_s"],
        "decode_step": decode_step,
        "paged_over_seat": seat["paged_over_seat"],
        "seat": seat,
        "config5": config5,
        "config4_cp": config4_cp,
        "prefill": prefill,
    }
    line["cpu_baseline"] = cpu_baseline(sample_layers=args.cpu_sample_layers)
    _finish(dist)
    return line


def _run_e2e(kv, graph, device, stream, rank, steps, dist) -> dict:
    """The same steps through the public API with host buffers. Every step copies its
    per-layer q/k/v from pinned host memory into a step graph's input buffers, replays the
    step and copies all layers' attention outputs back to pinned host memory, all inside the
    timed region. As a serving loop would, the copies run on a second stream and overlap the
    neighbouring steps' compute: two captured step graphs alternate, so step i+1's inputs
    land while step i computes and step i's outputs leave while step i+1 computes (events
    order every buffer reuse)."""
    from serve.graph import PagedStepGraph

    gen = torch.Generator().manual_seed(99 + rank)
    hq = torch.randn(tuple(graph.q.shape), generator=gen).to(torch.bfloat16).pin_memory()
    hk = torch.randn(tuple(graph.k.shape), generator=gen).to(torch.bfloat16).pin_memory()
    hv = torch.randn(tuple(graph.v.shape), generator=gen).to(torch.bfloat16).pin_memory()
    hout = torch.empty((2,) + tuple(graph.out.shape), dtype=torch.bfloat16).pin_memory()
    graphs = [graph, PagedStepGraph(kv, torch.empty_like(graph.q), torch.empty_like(graph.k),
                                    torch.empty_like(graph.v))]
    copy = torch.cuda.Stream(device)
    ready = [torch.cuda.Event() for _ in range(2)]  # inputs of the buffer set are in place
    done = [torch.cuda.Event() for _ in range(2)]   # the step that used the buffer set finished
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def upload(g, i):
        g.q.copy_(hq, non_blocking=True)
        g.k.copy_(hk, non_blocking=True)
        g.v.copy_(hv, non_blocking=True)
        ready[i % 2].record(copy)

    kv_bytes = 0
    _barrier(dist, device)
    start.record(stream)
    copy.wait_stream(stream)
    with torch.cuda.stream(copy):
        upload(graphs[0], 0)
    for i in range(steps):
        g = graphs[i % 2]
        kv_bytes += sum(p + 1 for p in kv._host_pos) * 2 * H_KV * D * 2 * N_LAYER
        stream.wait_event(ready[i % 2])
        g.replay()
        done[i % 2].record(stream)
        with torch.cuda.stream(copy):
            if i + 1 < steps:  # the other set was last used by step i - 1
                if i >= 1:
                    copy.wait_event(done[(i + 1) % 2])
                upload(graphs[(i + 1) % 2], i + 1)
            copy.wait_event(done[i % 2])
            hout[i % 2].copy_(g.out, non_blocking=True)
    stream.wait_stream(copy)
    stop.record(stream)
    _barrier(dist, device)
    ms = _max_over_ranks(dist, start.elapsed_time(stop), device)
    total = _sum_over_ranks(dist, float(kv_bytes), device)
    h2d = (hq.numel() + hk.numel() + hv.numel()) * 2
    d2h = graph.out.numel() * 2
    return {"value": round(total / (ms * 1e-3) / 1e9, 1), "unit": "GB/s (KV bytes read by decode, all ranks)",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "steps": steps,
            "us_per_layer_step": round(ms * 1e3 / (steps * N_LAYER), 2),
            "copies": "overlapped with neighbouring steps on a second stream (two step graphs alternate)"}


def _profiled_traffic(algorithmic_bytes: float):
    """DRAM bytes of one decode launch: the ncu-measured ratio of DRAM bytes (read + write) to
    algorithmic KV bytes on the config-2 profile case (profiles/decode_traffic.json), scaled
    to this launch's algorithmic bytes (traffic grows with the KV bytes read)."""
    path = ROOT / "profiles" / "decode_traffic.json"
    try:
        ratio = json.loads(path.read_text())["dram_over_algorithmic"]
    except (OSError, ValueError, KeyError):
        return None
    return int(ratio * algorithmic_bytes)


def _finish(dist):
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


# ------------------------------------------------------------------------------ sharded configs


def _fp32_attention(q, keys, values) -> torch.Tensor:
    """softmax(q K^T / sqrt(D)) V in fp32 for one row: q (H, D), keys/values (L, H_kv, D) -- the
    arithmetic of the reference's reference_paged_decode (tests/reference/paged.py:225-274) in
    torch on the device, as the bench line's own parity field."""
    h, d = q.shape
    hkv = keys.shape[1]
    qg = q.float().view(hkv, h // hkv, d)
    scores = torch.einsum("kgd,tkd->kgt", qg, keys.float()) / math.sqrt(d)
    probs = torch.softmax(scores, dim=-1)
    return torch.einsum("kgt,tkd->kgd", probs, values.float()).reshape(h, d)


def _max_abs_vs_fp32_rows(q, k_pool, v_pool, table, seqlen, rows, out) -> float:
    """Largest |out - fp32 reference| over ``rows`` of a paged decode (rows gathered through the
    block table)."""
    bs, hkv, d = k_pool.shape[1], k_pool.shape[2], k_pool.shape[3]
    worst = 0.0
    for r in rows.tolist():
        n = int(seqlen[r])
        blocks = table[r, :-(-n // bs)].long()
        keys = k_pool[blocks].reshape(-1, hkv, d)[:n]
        values = v_pool[blocks].reshape(-1, hkv, d)[:n]
        ref = _fp32_attention(q[r], keys, values)
        worst = max(worst, (out[r].float() - ref).abs().max().item())
    return worst


def _time_replays(fn, reps: int, stream) -> float:
    """Device time in ms of ``reps`` back-to-back calls of ``fn`` (CUDA events on ``stream``)."""
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for _ in range(reps):
        fn()
    stop.record(stream)
    stop.synchronize()
    return start.elapsed_time(stop)


def run_config5(device, rank: int, world: int, dist, reps: int) -> dict:
    """1024 rows, L ~ U[256, 4096], sharded by row index over the ranks (each
    its own pool, table and seqlen; no collective on the data path), strong scaling. Two layers
    with distinct pools (each layer's K/V larger than L2 at every world size) are launched back
    to back in a CUDA graph, the second overlapping the first; ``reps`` replays are timed."""
    from model import _native
    from model.triton_decode import paged_decode_plan
    import workloads

    n_layer = 2
    wl = workloads.config5(device, rank=rank, world=world, n_layer=n_layer)
    plan = paged_decode_plan(wl.q[0], wl.k_pools, wl.v_pools, wl.block_table, wl.seqlen)
    outs = [torch.empty_like(q) for q in wl.q]
    graph = torch.cuda.CUDAGraph()
    for layer in range(n_layer):
        plan.run(layer, wl.q[layer], out=outs[layer])
    torch.cuda.synchronize(device)
    with torch.cuda.graph(graph):
        for layer in range(n_layer):
            plan.run(layer, wl.q[layer], out=outs[layer], overlap=layer > 0)
    stream = torch.cuda.current_stream(device)
    graph.replay()
    _barrier(dist, device)
    ms_local = _time_replays(graph.replay, reps, stream)
    _barrier(dist, device)
    assert _native.device_error() == 0, "device error word set in config 5"
    kv_local = wl.kv_bytes_per_layer() * n_layer * reps
    ms = _max_over_ranks(dist, ms_local, device)
    total = _sum_over_ranks(dist, float(kv_local), device)
    gbs_local = kv_local / (ms_local * 1e-3) / 1e9
    gbs_min = -_max_over_ranks(dist, -gbs_local, device)
    # parity of the device's output: a subset of this rank's rows against an fp32 reference
    rows = torch.arange(0, wl.q[0].shape[0], max(1, wl.q[0].shape[0] // 8))
    err = _max_abs_vs_fp32_rows(wl.q[0], wl.k_pools[0], wl.v_pools[0], wl.block_table, wl.seqlen, rows, outs[0])
    err = _max_over_ranks(dist, err, device)
    peak = _peaks()["hbm_gbs"]
    line = {
        "workload": "BASELINE configs[4]: 1024 rows, L~U[256,4096], Qwen3-0.6B heads, bf16, rows sharded by "
                    "index over the ranks (own pool/table per rank, no collective); strong scaling",
        "rows_per_gpu": int(wl.q[0].shape[0]), "layers_per_replay": n_layer, "replays": reps,
        "us_per_layer_step": round(ms * 1e3 / (reps * n_layer), 2),
        "aggregate_kv_gbs": round(total / (ms * 1e-3) / 1e9, 1),
        "kv_gbs_per_gpu_min": round(gbs_min, 1),
        "roofline_frac_per_gpu_min": round(gbs_min / peak, 4),
        "max_abs_vs_fp32_reference": err, "checked_rows_per_gpu": int(rows.numel()),
        "timing": "CUDA events around the replays, max over ranks; per-GPU GB/s = that rank's KV bytes / its time",
    }
    del graph, plan, wl, outs
    torch.cuda.empty_cache()
    return line


def run_config4_cp(device, rank: int, world: int, dist, steps: int) -> dict:
    """BASELINE config 4, context parallel: B=32 rows of 8192 tokens; rank r owns the contiguous
    8192 / world token slice of every row (its own pool and table). Per layer and step, inside
    the timed region: one ``pd_decode_partials`` launch over the slice, ONE NCCL
    ``all_gather_into_tensor`` of the packed fp32 (acc | m | l) buffer, one ``pd_lse_merge``
    (every rank ends with the full output). Four layers with distinct pools per step. CUDA
    events separate compute (partials + merge) from the collective; each is the max over
    ranks. The merged output of a row subset is checked against an fp32 reference over the
    whole 8192-token rows in fp32 (their slices all-gathered to every rank, outside the timed
    region)."""
    from model import _native
    from model.parallel_decode import ContextParallelDecode
    import workloads

    n_layer, B, ctx = 4, BATCH, 8192
    wl = workloads.config4(device, n_layer=n_layer, rank=rank, world=world)
    gen = torch.Generator(device=device).manual_seed(4444)  # q is the same on every rank
    qs = [torch.randn(B, H, D, generator=gen, device=device).to(torch.bfloat16) for _ in range(n_layer)]
    outs = [torch.empty_like(q) for q in qs]
    cp = ContextParallelDecode()
    scale = 1.0 / math.sqrt(D)
    events = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(n_layer * steps)]

    def step(ev=None):
        for layer in range(n_layer):
            cp(qs[layer], wl.k_pools[layer], wl.v_pools[layer], wl.block_table, wl.seqlen, scale=scale,
               out=outs[layer], events=None if ev is None else ev[layer])

    for _ in range(3):
        step()
    stream = torch.cuda.current_stream(device)
    _barrier(dist, device)
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(stream)
    for i in range(steps):
        step(events[i * n_layer:(i + 1) * n_layer])
    stop.record(stream)
    _barrier(dist, device)
    assert _native.device_error() == 0, "device error word set in config 4"
    ms_local = start.elapsed_time(stop)
    compute = sum(e[0].elapsed_time(e[1]) + e[2].elapsed_time(e[3]) for e in events)
    collective = sum(e[1].elapsed_time(e[2]) for e in events)
    ms = _max_over_ranks(dist, ms_local, device)
    compute_max = _max_over_ranks(dist, compute, device)
    collective_max = _max_over_ranks(dist, collective, device)
    kv_local = wl.kv_bytes_per_layer() * n_layer * steps
    total = _sum_over_ranks(dist, float(kv_local), device)
    layer_steps = n_layer * steps

    # parity: rows 0, 8, 16, 24 of layer 0, whole 8192-token rows gathered from every rank's slice
    rows = list(range(0, B, 8))
    span = ctx // world
    pages = span // BS
    kk = torch.stack([wl.k_pools[0][wl.block_table[r, :pages].long()] for r in rows])  # (R, pages, bs, Hkv, D)
    vv = torch.stack([wl.v_pools[0][wl.block_table[r, :pages].long()] for r in rows])
    if dist is not None:
        kk_all = torch.empty((world,) + tuple(kk.shape), dtype=kk.dtype, device=device)
        vv_all = torch.empty_like(kk_all)
        dist.all_gather_into_tensor(kk_all, kk.contiguous())
        dist.all_gather_into_tensor(vv_all, vv.contiguous())
        kk = kk_all.permute(1, 0, 2, 3, 4, 5).reshape(len(rows), world * pages, BS, H_KV, D)
        vv = vv_all.permute(1, 0, 2, 3, 4, 5).reshape(len(rows), world * pages, BS, H_KV, D)
    err = 0.0
    for i, r in enumerate(rows):
        ref = _fp32_attention(qs[0][r], kk[i].reshape(-1, H_KV, D), vv[i].reshape(-1, H_KV, D))
        err = max(err, (outs[0][r].float() - ref).abs().max().item())
    err = _max_over_ranks(dist, err, device)
    identical = True
    if dist is not None:
        mine = outs[0].contiguous()
        everyone = torch.empty((world,) + tuple(mine.shape), dtype=mine.dtype, device=device)
        dist.all_gather_into_tensor(everyone, mine)
        identical = all(torch.equal(everyone[0], everyone[r]) for r in range(world))
    peak = _peaks()["hbm_gbs"]
    compute_us = compute_max * 1e3 / layer_steps
    line = {
        "workload": "BASELINE configs[3] context-parallel: B=32 x 8192 tokens, Qwen3-0.6B heads, bf16; each rank "
                    "owns 8192/N tokens of every row; pd_decode_partials + one NCCL all_gather_into_tensor of "
                    "(acc|m|l) + pd_lse_merge per layer-step",
        "tokens_per_gpu_per_row": span, "layers_per_step": n_layer, "steps": steps,
        "us_per_layer_step": round(ms * 1e3 / layer_steps, 2),
        "compute_us_per_layer_step": round(compute_us, 2),
        "allgather_us_per_layer_step": round(collective_max * 1e3 / layer_steps, 2),
        "allgather_bytes_per_rank": B * H * (D + 2) * 4,
        "aggregate_kv_gbs": round(total / (ms * 1e-3) / 1e9, 1),
        "compute_kv_gbs_per_gpu": round(kv_local / layer_steps / (compute_us * 1e-6) / 1e9, 1),
        "compute_roofline_frac_per_gpu": round(kv_local / layer_steps / (compute_us * 1e-6) / 1e9 / peak, 4),
        "limiter": "allgather" if collective_max > compute_max else "compute",
        "max_abs_vs_fp32_reference": err, "checked_rows": rows, "identical_on_all_ranks": identical,
        "timing": "CUDA events on the launching stream around each stage, summed, max over ranks",
    }
    del wl, qs, outs, cp, kk, vv
    torch.cuda.empty_cache()
    return line


def run_decode_step(device, rank: int, dist, steps: int = NEW_TOKENS) -> dict:
    """BASELINE config 2's whole decode step: a random-init Qwen3-0.6B-shaped model
    (``decode_model.PagedDecoder``: 28 layers of norms, projections, RoPE, SwiGLU; tied lm_head
    and greedy argmax) whose attention is ``PagedKV.write`` + ``attend`` (the fused sm_100a
    append + decode, K rotated in the append, layers overlapped). B=32 rows at context 2048
    (K/V of the prompts drawn N(0, 1)), greedy for ``steps`` steps; the step is captured once
    as a CUDA graph and every timed step is one replay (next token = this step's argmax on
    the device)."""
    from decode_model import PagedDecoder
    from model import _native
    from serve.graph import DecodeStepGraph

    warm = 3
    budget = steps + warm + 2 + 1
    kv = _container(device, budget, seed=100 + rank)
    model = PagedDecoder(kv, n_layer=N_LAYER, n_head=H, n_kv_head=H_KV, head_dim=D, rotary=D,
                         max_pos=CONTEXT + budget + 1, seed=7, device=device)
    gen = torch.Generator(device=device).manual_seed(8 + rank)
    model.tok.copy_(torch.randint(0, 151936, (BATCH,), generator=gen, device=device))
    with torch.no_grad():
        for _ in range(warm):
            kv.build_mask(next_token=True)
            model.step()
            kv.advance()
        graph = DecodeStepGraph(kv, model.step, model.prepare_q)
        for _ in range(2):
            graph.replay()
        stream = torch.cuda.current_stream(device)
        _barrier(dist, device)
        ms_local = _time_replays(graph.replay, steps, stream)
        _barrier(dist, device)
    assert _native.device_error() == 0, "device error word set in the decode step"
    ms = _max_over_ranks(dist, ms_local, device)
    world = 1 if dist is None else dist.get_world_size()
    line = {
        "workload": "BASELINE configs[1] whole decode step: random-init Qwen3-0.6B (28 layers, hidden 1024, "
                    "16q/8kv, D=128, SwiGLU 3072, vocab 151936, tied lm_head), B=32 at context 2048, "
                    f"{steps} greedy steps, attention through PagedKV; CUDA graph per step",
        "decode_tok_s": round(world * BATCH * steps / (ms * 1e-3), 1),
        "ms_per_step": round(ms / steps, 4),
        "steps": steps, "context": f"{CONTEXT + warm + 2}..{CONTEXT + warm + 2 + steps}",
        "library_launches_per_step": graph.launches_per_step,
        "reference_decode_only_tok_s_rtx4090": 1230.5,
    }
    del graph, model, kv
    torch.cuda.empty_cache()
    return line


# ------------------------------------------------------------------------------ CPU arm


def _cpu_sample(sample_layers: int, seed: int = 0):
    """Config-2 shapes for ``sample_layers`` layers on the CPU (bf16 K/V, same generator)."""
    import workloads

    wl = workloads.config2("cpu", seed=seed, n_layer=sample_layers)
    return wl


def cpu_baseline(sample_layers: int = 2, threads: int = 0) -> dict:
    """The reference's CPU path (gather_pool + hand_baddbmm seat decode, ported in oracle/)
    on a bounded sample: ``sample_layers`` layer-steps of the config-2 workload."""
    from oracle import oracle

    threads = threads or os.cpu_count() or 1
    wl = _cpu_sample(sample_layers)
    lpad = -(-CONTEXT // 64) * 64
    oracle.seat_decode(wl.q[0][:1], torch.zeros(1, H_KV, 64, D, dtype=torch.bfloat16),
                       torch.zeros(1, H_KV, 64, D, dtype=torch.bfloat16), torch.tensor([1]), threads=threads)
    t0 = time.perf_counter()
    for layer in range(sample_layers):
        gk, gv = oracle.gather_pool(wl.k_pools[layer], wl.v_pools[layer], wl.block_table, wl.seqlen, lpad,
                                    threads=threads)
        oracle.seat_decode(wl.q[layer], gk, gv, wl.seqlen, threads=threads)
    dt = time.perf_counter() - t0
    kv = wl.kv_bytes_per_layer() * sample_layers
    return {"value": round(kv / dt / 1e9, 3), "unit": "GB/s (KV bytes read by decode)", "cores": threads,
            "kind": "port",
            "sample": f"{sample_layers} layer-steps of config 2 (B=32, L=2048, 16q/8kv, D=128, bf16): "
                      f"gather_pool + hand_baddbmm seat decode, {dt * 1e3 / sample_layers:.1f} ms/layer-step",
            "us_per_layer_step": round(dt * 1e6 / sample_layers, 1)}


def run_reference(args) -> dict | None:
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return None
    threads = os.cpu_count() or 1
    base = cpu_baseline(sample_layers=1, threads=threads)  # warm-up + first sample
    per_step = []
    for _ in range(args.steps):
        per_step.append(cpu_baseline(sample_layers=1, threads=threads)["us_per_layer_step"])
    us = statistics.median(per_step)
    gbs = CONTEXT * BATCH * 2 * H_KV * D * 2 / (us * 1e-6) / 1e9
    return {
        "metric": METRIC, "impl": "reference", "value": round(gbs, 3),
        "unit": "GB/s (KV bytes read by decode, all ranks)", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(us * N_LAYER / 1e3, 2), "us_per_layer_step": round(us, 1),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (seeded N(0,1) K/V/q)",
        "config": {"workload": "BASELINE configs[1] attention path on the CPU: reference gather_pool + "
                               "hand_baddbmm seat decode (ported, oracle/), one layer-step per sample",
                   "batch": BATCH, "context": CONTEXT, "layers": N_LAYER, "block_size": BS},
        "cpu_baseline": {**base, "value": round(gbs, 3)},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s (KV bytes read by decode, all ranks)",
                "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def profile_case(name: str, launches: int = 4) -> None:
    """A short, deterministic run for profilers: one layer of a benchmark config, one
    stand-alone append and ``launches`` fused append + decode launches (the bench step's
    kernel; each appends the same token again), nothing else on the GPU afterwards."""
    from model import _native
    from model.triton_decode import paged_decode_plan
    import workloads

    device = torch.device("cuda", 0)
    if name == "prefill":  # chunked prefill: 4 rows x (2048 cached + 512 new tokens), one layer
        from model.triton_decode import paged_prefill

        gen = torch.Generator(device=device).manual_seed(11)
        rows, ctx, chunk = 4, 2048, 512
        pages = -(-(ctx + chunk) // BS)
        k = torch.randn(rows * pages + 1, BS, H_KV, D, generator=gen, device=device, dtype=torch.bfloat16)
        v = torch.randn(rows * pages + 1, BS, H_KV, D, generator=gen, device=device, dtype=torch.bfloat16)
        table = torch.randperm(rows * pages + 1, generator=gen, device=device)[: rows * pages]
        table = table.view(rows, pages).to(torch.int32)
        q = torch.randn(rows * chunk, H, D, generator=gen, device=device, dtype=torch.bfloat16)
        cu = torch.arange(rows + 1, device=device, dtype=torch.int32) * chunk
        sk = torch.full((rows,), ctx + chunk, device=device, dtype=torch.int32)
        for _ in range(launches):
            paged_prefill(q, k, v, table, cu, sk, chunk)
        torch.cuda.synchronize()
        if _native.device_error() != 0:
            raise SystemExit("device error word set")
        print(json.dumps({"profile_case": name, "launches": launches, "rows": rows, "context": ctx, "chunk": chunk}))
        return
    wl = getattr(workloads, name)(device, n_layer=1)
    plan = paged_decode_plan(wl.q[0], wl.k_pools, wl.v_pools, wl.block_table, wl.seqlen)
    B = wl.q[0].shape[0]
    hkv, d = wl.k_pools[0].shape[2], wl.k_pools[0].shape[3]
    gen = torch.Generator(device=device).manual_seed(5)
    k_new = torch.randn(B, hkv, d, generator=gen, device=device).to(wl.k_pools[0].dtype)
    pos = (wl.seqlen.to(torch.int64) - 1).clamp_min(0)
    _native.append_table(wl.k_pools[0], wl.v_pools[0], wl.block_table, pos, k_new, k_new)
    for _ in range(launches):
        plan.run_append(0, wl.q[0], k_new, k_new, pos)
    torch.cuda.synchronize()
    if _native.device_error() != 0:
        raise SystemExit("device error word set")
    print(json.dumps({"profile_case": name, "launches": launches, "kv_bytes": wl.kv_bytes_per_layer()}))


def config_sweep(reps: int = 5) -> None:
    """The decode kernel alone on every BASELINE config (and the hybrid Qwen3.5 engine's
    full-attention shape): each layer's plan launched once, the
    layers back to back in a CUDA graph (distinct per-layer pools, so every launch reads cold
    HBM), best and median of ``reps`` replays, once with plain launches and once with layers
    1.. overlapping their predecessor (programmatic dependent launch, as in a decode step).
    One JSON line per config (not the bench line)."""
    from model import _native
    from model.triton_decode import paged_decode_plan
    import workloads

    device = torch.device("cuda", 0)
    peak = _peaks()["hbm_gbs"]
    for name, n_layer in (("config1", 28), ("config2", 28), ("config3", 28), ("config4", 4), ("config5", 2),
                          ("qwen35", 6)):
        wl = getattr(workloads, name)(device, n_layer=n_layer)
        plan = paged_decode_plan(wl.q[0], wl.k_pools, wl.v_pools, wl.block_table, wl.seqlen)
        plan._native_plan.set_static_table(True)  # the workloads' tables are fixed, as PagedKV's are
        for layer in range(n_layer):
            plan.run(layer, wl.q[layer])
        torch.cuda.synchronize(device)
        line = {"config": name, "rows": int(wl.q[0].shape[0]), "layers": n_layer}
        kv = wl.kv_bytes_per_layer()
        line["kv_bytes_per_launch"] = kv
        for overlap in (False, True):
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for layer in range(n_layer):
                    plan.run(layer, wl.q[layer], overlap=overlap and layer > 0)
            graph.replay()
            times = []
            for _ in range(reps):
                start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                start.record()
                graph.replay()
                stop.record()
                torch.cuda.synchronize(device)
                times.append(start.elapsed_time(stop) * 1e3 / n_layer)
            if _native.device_error() != 0:
                raise SystemExit(f"{name}: device error word set")
            best, med = min(times), statistics.median(times)
            tag = "overlapped_" if overlap else ""
            line.update({f"{tag}us_per_launch_best": round(best, 2), f"{tag}us_per_launch_median": round(med, 2),
                         f"{tag}kv_gbs_best": round(kv / best / 1e3, 1),
                         f"{tag}roofline_frac_best": round(kv / best / 1e3 / peak, 4)})
            del graph
        line["peak_gbs"] = peak
        print(json.dumps(line), flush=True)
        del plan, wl
        torch.cuda.empty_cache()


def prefill_sweep(reps: int = 5) -> None:
    """Chunked prefill over the paged pool (``paged_prefill``) at Qwen3-0.6B head shapes (and
    the Qwen3.5 full-attention heads, 8q/2kv, head_dim 256): each
    layer's launch once per replay of a CUDA graph, distinct per-layer pools (larger than L2),
    best of ``reps`` replays. FLOPs are the causal ones: 4 * D per visible (query, key) pair per
    q head. Each case runs on both prefill kernels (tcgen05 / TMEM, the default, and the
    mma.sync kernel). One JSON line per case and kernel (not the bench line)."""
    from model import _native

    device = torch.device("cuda", 0)
    peaks = _peaks()
    for mode, kernel in ((0, "tcgen05"), (1, "mma_sync")):
        _native.set_prefill_mode(mode)
        try:
            _prefill_cases(device, peaks, reps, kernel)
        finally:
            _native.set_prefill_mode(0)


PREFILL_CASES = (
    # name, rows, cached context, chunk, layers, (q heads, kv heads, head_dim)
    ("chunk512_ctx2048", 4, 2048, 512, 28, (16, 8, 128)),
    ("chunk2048_ctx0", 4, 0, 2048, 28, (16, 8, 128)),
    ("chunk128_ctx4096", 16, 4096, 128, 8, (16, 8, 128)),
    ("qwen35_chunk512_ctx2048", 4, 2048, 512, 6, (8, 2, 256)),
)


def _prefill_cases(device, peaks, reps, kernel) -> None:
    for case in PREFILL_CASES:
        print(json.dumps(prefill_case(device, peaks, reps, kernel, *case)), flush=True)


def prefill_case(device, peaks, reps, kernel, name, rows, ctx, chunk, n_layer, heads) -> dict:
    """One chunked-prefill case: every layer's ``paged_prefill`` launch once per replay of a
    CUDA graph over distinct per-layer pools, best of ``reps`` replays."""
    from model import _native
    from model.triton_decode import paged_prefill

    H, H_KV, D = heads
    gen = torch.Generator(device=device).manual_seed(11)
    total = ctx + chunk
    pages = -(-total // BS)
    n_blocks = rows * pages + 1
    pools_k = [torch.randn(n_blocks, BS, H_KV, D, generator=gen, device=device, dtype=torch.bfloat16)
               for _ in range(n_layer)]
    pools_v = [torch.randn(n_blocks, BS, H_KV, D, generator=gen, device=device, dtype=torch.bfloat16)
               for _ in range(n_layer)]
    perm = torch.randperm(n_blocks, generator=gen, device=device)[: rows * pages]
    table = perm.view(rows, pages).to(torch.int32)
    q = [torch.randn(rows * chunk, H, D, generator=gen, device=device, dtype=torch.bfloat16)
         for _ in range(n_layer)]
    cu = torch.arange(rows + 1, device=device, dtype=torch.int32) * chunk
    sk = torch.full((rows,), total, device=device, dtype=torch.int32)
    outs = [paged_prefill(q[i], pools_k[i], pools_v[i], table, cu, sk, chunk) for i in range(n_layer)]
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        outs = [paged_prefill(q[i], pools_k[i], pools_v[i], table, cu, sk, chunk) for i in range(n_layer)]
    graph.replay()
    times = []
    for _ in range(reps):
        start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        graph.replay()
        stop.record()
        torch.cuda.synchronize(device)
        times.append(start.elapsed_time(stop) * 1e3 / n_layer)
    if _native.device_error() != 0:
        raise SystemExit(f"{name}: device error word set")
    best = min(times)
    pairs = rows * (chunk * ctx + chunk * (chunk + 1) // 2)  # visible (query, key) pairs
    flops = 4.0 * D * H * pairs
    kv_bytes = rows * total * H_KV * D * 2 * 2
    tflops = flops / (best * 1e-6) / 1e12
    result = {
        "prefill_case": name, "kernel": kernel, "rows": rows, "context": ctx, "chunk": chunk, "layers": n_layer,
        "heads": f"{H}q/{H_KV}kv", "head_dim": D, "dtype": "bf16",
        "us_per_launch_best": round(best, 2), "us_per_launch_median": round(statistics.median(times), 2),
        "causal_tflops": round(tflops, 1),
        "tensor_roofline_frac": round(tflops / peaks["bf16_tflops_sustained"], 4),
        "tensor_peak_tflops": peaks["bf16_tflops_sustained"], "kv_gbs": round(kv_bytes / best / 1e3, 1),
        "hbm_roofline_frac": round(kv_bytes / best / 1e3 / peaks["hbm_gbs"], 4),
        "peak_source": peaks["source"],
        "note": "P as hi+lo 16-bit operands: 3 tensor products per (query, key, d) where a "
                "16-bit-P kernel needs 2; tcgen05: S and O in TMEM, mma_sync: warp-level tiles"}
    del graph, outs, pools_k, pools_v, q
    torch.cuda.empty_cache()
    return result


class _SeatStep:
    """The reference's seat decode step, restated in torch as the cost comparator (it is not
    the product and not the numeric oracle). Per step: the additive bias of the dense slab is
    built once (``KvSlab.build_mask(next_token=True)``, model/slab.py:302-328, with
    ``additive_bias``, model/attention/hand_baddbmm.py:129-149). Per layer: the token's K/V are
    scattered into column ``pos`` of the layer's ``(B, H_kv, width, D)`` slab (slab.py:251-266),
    then ``HandBaddbmmBackend.decode`` (hand_baddbmm.py:80-126) runs: q scaled by 1/sqrt(D),
    ``baddbmm(bias, q, K^T)`` over the whole slab width, a bf16 softmax and ``bmm`` with V, with
    the GQA group as the GEMM's row dimension. The slab width is a 64-column bucket."""

    def __init__(self, device, lengths, budget: int, gen):
        self.B = len(lengths)
        self.G = H // H_KV
        self.width = -(-(max(lengths) + budget) // 64) * 64
        shape = (self.B, H_KV, self.width, D)
        self.keys = [torch.randn(shape, generator=gen, device=device).to(torch.bfloat16) for _ in range(N_LAYER)]
        self.values = [torch.randn(shape, generator=gen, device=device).to(torch.bfloat16) for _ in range(N_LAYER)]
        self.pos = torch.tensor(lengths, device=device, dtype=torch.int64)
        self.columns = torch.arange(self.width, device=device)
        self.bias = torch.empty(self.B * H_KV, self.G, self.width, device=device, dtype=torch.bfloat16)
        self.out = torch.empty(N_LAYER, self.B * H_KV, self.G, D, device=device, dtype=torch.bfloat16)

    def step(self, q_buf, k_buf, v_buf) -> None:
        B, G, W = self.B, self.G, self.width
        allowed = self.columns.view(1, W) < (self.pos + 1).view(B, 1)
        bias = torch.where(allowed, 0.0, float("-inf")).to(torch.bfloat16)
        self.bias.copy_(bias.view(B, 1, 1, W).expand(B, H_KV, G, W).reshape(B * H_KV, G, W))
        index = self.pos.view(B, 1, 1, 1).expand(B, H_KV, 1, D)
        for layer in range(N_LAYER):
            self.keys[layer].scatter_(2, index, k_buf[layer])
            self.values[layer].scatter_(2, index, v_buf[layer])
            qg = (q_buf[layer] * (1.0 / math.sqrt(D))).reshape(B * H_KV, G, D)
            k_t = self.keys[layer].transpose(-2, -1).reshape(B * H_KV, D, W)
            probs = torch.softmax(torch.baddbmm(self.bias, qg, k_t), dim=-1)
            torch.bmm(probs, self.values[layer].reshape(B * H_KV, W, D), out=self.out[layer])
        self.pos += 1


def seat_case(device, name: str, lengths: list[int], reps: int = 10) -> dict:
    """Decode-step cost of the paged arm against the seat arm at Qwen3-0.6B head shapes, both
    steps (28 layers of K/V append + attention, with the step's bookkeeping) captured once as
    CUDA graphs and replayed, best of ``reps`` replays, for rows of the given lengths."""
    from model import _native
    from model.paged import PagedKV, PagedPool
    from serve.block_manager import BlockManager
    from serve.graph import PagedStepGraph

    eager, budget = 3, 3 + 2 + reps + 2
    B = len(lengths)
    gen = torch.Generator(device=device).manual_seed(21)
    q_buf = torch.randn(N_LAYER, B, H, 1, D, generator=gen, device=device).to(torch.bfloat16)
    k_buf = torch.randn(N_LAYER, B, H_KV, 1, D, generator=gen, device=device).to(torch.bfloat16)
    v_buf = torch.randn(N_LAYER, B, H_KV, 1, D, generator=gen, device=device).to(torch.bfloat16)

    def timed(replay) -> list[float]:
        times = []
        for _ in range(reps):
            start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            replay()
            stop.record()
            torch.cuda.synchronize(device)
            times.append(start.elapsed_time(stop) * 1e3 / N_LAYER)
        return times

    manager = BlockManager(sum(-(-(n + budget) // BS) for n in lengths), BS)
    tables = [manager.reserve(manager.blocks_for(n, budget)) for n in lengths]
    pool = PagedPool(N_LAYER, manager.n_blocks, BS, H_KV, D, dtype=torch.bfloat16, device=device, n_head=H)
    for t in pool.keys + pool.values:
        t.copy_(torch.randn(t.shape, generator=gen, device=device))
    kv = PagedKV(pool, tables, lengths, rope_len=max(lengths) + budget, n_head=H)
    for _ in range(eager):
        kv.build_mask(next_token=True)
        for layer in range(N_LAYER):
            kv.write(layer, k_buf[layer], v_buf[layer])
            kv.attend(layer, q_buf[layer])
        kv.advance()
    graph = PagedStepGraph(kv, q_buf, k_buf, v_buf)
    for _ in range(2):
        graph.replay()
    paged = timed(graph.replay)
    if _native.device_error() != 0:
        raise SystemExit(f"{name}: device error word set")
    del graph, kv, pool
    torch.cuda.empty_cache()

    seat = _SeatStep(device, lengths, budget, gen)
    for _ in range(eager):
        seat.step(q_buf, k_buf, v_buf)
    torch.cuda.synchronize(device)
    seat_graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(seat_graph):
        seat.step(q_buf, k_buf, v_buf)
    for _ in range(2):
        seat_graph.replay()
    seat_times = timed(seat_graph.replay)
    line = {
        "seat_case": name, "rows": B, "contexts": f"{min(lengths)}..{max(lengths)} (+step)",
        "layers": N_LAYER, "heads": f"{H}q/{H_KV}kv", "head_dim": D, "dtype": "bf16",
        "paged_us_per_layer_step": round(min(paged), 2), "seat_us_per_layer_step": round(min(seat_times), 2),
        "paged_over_seat": round(min(paged) / min(seat_times), 3),
        "paged_median": round(statistics.median(paged), 2), "seat_median": round(statistics.median(seat_times), 2),
        "seat_slab_width": seat.width,
        "note": "attention part of the decode step (append + attention + step bookkeeping), both arms as "
                "CUDA graphs; the reference's own paged/seat figure is a whole-model step"}
    del seat_graph, seat
    torch.cuda.empty_cache()
    return line


def seat_sweep(reps: int = 10) -> None:
    """:func:`seat_case` for config 2 (B=32 at 2048 tokens) and the reference's own paged/seat
    comparison size (B=8, contexts up to 1645 tokens; seeded uniform in [1024, 1645] here). One
    JSON line per case (not the bench line)."""
    device = torch.device("cuda", 0)
    cases = (("config2_b32_ctx2048", [CONTEXT] * BATCH),
             ("b8_ctx1024_1645", torch.randint(1024, 1646, (8,), generator=torch.Generator().manual_seed(5)).tolist()))
    for name, lengths in cases:
        print(json.dumps(seat_case(device, name, lengths, reps)), flush=True)


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--profile-case", default=None,
                        help="run a short profiler case (config1..config5, qwen35, prefill) instead of the benchmark")
    parser.add_argument("--decode-mode", type=int, default=None, choices=(0, 1, 2),
                        help="with --profile-case / --configs: pd_set_decode_mode first (0 tensor-core "
                             "tile math where it applies, 1 shared stages, 2 CUDA-core tile math)")
    parser.add_argument("--configs", action="store_true",
                        help="time the decode kernel alone on every BASELINE config instead of the benchmark")
    parser.add_argument("--prefill", action="store_true",
                        help="time the chunked-prefill kernel (paged_prefill) instead of the benchmark")
    parser.add_argument("--seat", action="store_true",
                        help="time the paged decode step against the seat (dense slab) step instead of the benchmark")
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=100)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=("b200", "reference"), default="b200")
    parser.add_argument("--cpu-sample-layers", type=int, default=2)
    args = parser.parse_args(argv)
    if args.decode_mode is not None:
        if not (args.profile_case or args.configs):
            raise SystemExit("--decode-mode applies to --profile-case and --configs only")
        from model import _native
        _native.set_decode_mode(args.decode_mode)
    if args.profile_case:
        profile_case(args.profile_case)
        return 0
    if args.configs:
        config_sweep()
        return 0
    if args.prefill:
        prefill_sweep()
        return 0
    if args.seat:
        seat_sweep()
        return 0
    if args.warmup < 3:
        raise SystemExit("--warmup must be >= 3")
    line = run_reference(args) if args.impl == "reference" else run_gpu(args)
    if line is not None:
        print(json.dumps(line), flush=True)
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
