"""Host-side checks of ``bench.py``: the seat comparator computes the seat decode it stands
for, and the timing rules are enforced before any GPU work."""

from __future__ import annotations

import math
import sys
from pathlib import Path

import pytest
import torch

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
import bench  # noqa: E402


def test_seat_step_appends_at_pos_and_attends_over_the_allowed_columns():
    B, lengths = 3, [5, 9, 1]
    gen = torch.Generator().manual_seed(0)
    seat = bench._SeatStep(torch.device("cpu"), lengths, 3, gen)
    assert seat.width == 64
    shape_q, shape_kv = (bench.N_LAYER, B, bench.H, 1, bench.D), (bench.N_LAYER, B, bench.H_KV, 1, bench.D)
    q = torch.randn(shape_q, generator=gen).to(torch.bfloat16)
    k = torch.randn(shape_kv, generator=gen).to(torch.bfloat16)
    v = torch.randn(shape_kv, generator=gen).to(torch.bfloat16)
    seat.step(q, k, v)
    assert seat.pos.tolist() == [n + 1 for n in lengths]
    G = bench.H // bench.H_KV
    for layer in (0, bench.N_LAYER - 1):
        for b, n in enumerate(lengths):
            assert torch.equal(seat.keys[layer][b, :, n], k[layer, b, :, 0])
            assert torch.equal(seat.values[layer][b, :, n], v[layer, b, :, 0])
            keys = seat.keys[layer][b, :, :n + 1].float()
            vals = seat.values[layer][b, :, :n + 1].float()
            qg = q[layer, b, :, 0].float().view(bench.H_KV, G, bench.D)
            p = torch.softmax(torch.einsum("kgd,ktd->kgt", qg, keys) / math.sqrt(bench.D), dim=-1)
            ref = torch.einsum("kgt,ktd->kgd", p, vals)
            got = seat.out[layer].view(B, bench.H_KV, G, bench.D)[b].float()
            # the seat path's softmax is bf16: a few bf16 ulps of the probabilities
            assert (got - ref).abs().max().item() < 0.05


def test_fewer_than_three_warmup_steps_are_refused():
    with pytest.raises(SystemExit, match="warmup"):
        bench.main(["--warmup", "2"])


def test_bench_parity_reference_equals_the_oracle():
    """The bench line's own parity field (an fp32 torch restatement of the reference's
    reference_paged_decode) agrees with the pinned oracle on a paged case."""
    from helpers import build_case
    from oracle import oracle

    q, k, v, table, seqlen = build_case(3, 16, 8, 128, 16, [40, 300, 17], dtype=torch.bfloat16, seed=4)
    ref, _ = oracle.paged_decode(q, k, v, table, seqlen)
    got = torch.stack([
        bench._fp32_attention(q[r], k[table[r, :-(-int(seqlen[r]) // 16)].long()].reshape(-1, 8, 128)[:int(seqlen[r])],
                              v[table[r, :-(-int(seqlen[r]) // 16)].long()].reshape(-1, 8, 128)[:int(seqlen[r])])
        for r in range(3)])
    assert (got - ref).abs().max().item() < 1e-5
    assert bench._max_abs_vs_fp32_rows(q, k, v, table, seqlen, torch.arange(3), ref) < 1e-5
