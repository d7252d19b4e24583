"""CUDA-graph replay of the paged decode step (``serve.graph.PagedStepGraph``) on a B200.

* N replays of a captured step equal N eager steps bit for bit: every layer's output, the
  pools, the device positions and the host mirrors. Rows are long enough that items are split
  across workers, so every replay depends on the kernel's own per-launch epoch (a graph
  replays identical launch parameters).
* A replay that would write past the run's position bound is refused on the host before
  anything is launched.
"""

from __future__ import annotations

import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

N_LAYER, B, H, HKV, D, BS = 3, 6, 16, 8, 128, 16
LENGTHS = [2048, 1500, 17, 3000, 1, 700]


def _container(device, budget):
    from model.paged import PagedKV, PagedPool
    from serve.block_manager import BlockManager

    manager = BlockManager(sum(-(-(n + budget) // BS) for n in LENGTHS) + 8, BS)
    tables = [manager.reserve(manager.blocks_for(n, budget)) for n in LENGTHS]
    pool = PagedPool(N_LAYER, manager.n_blocks, BS, HKV, D, dtype=torch.bfloat16, device=device, n_head=H)
    gen = torch.Generator(device=device).manual_seed(11)
    for t in pool.keys + pool.values:
        t.copy_(torch.randn(t.shape, generator=gen, device=device))
    return PagedKV(pool, tables, LENGTHS, rope_len=max(LENGTHS) + budget, n_head=H)


def _inputs(device, steps):
    gen = torch.Generator(device=device).manual_seed(12)
    q = torch.randn(steps, N_LAYER, B, H, 1, D, generator=gen, device=device).to(torch.bfloat16)
    k = torch.randn(steps, N_LAYER, B, HKV, 1, D, generator=gen, device=device).to(torch.bfloat16)
    v = torch.randn(steps, N_LAYER, B, HKV, 1, D, generator=gen, device=device).to(torch.bfloat16)
    return q, k, v


def test_graph_replays_equal_eager_steps(cuda_device):
    from serve.graph import PagedStepGraph

    steps = 12
    q, k, v = _inputs(cuda_device, steps + 1)

    eager = _container(cuda_device, steps + 4)
    eager_out = []
    for i in range(steps + 1):
        eager.build_mask(next_token=True)
        outs = []
        for layer in range(N_LAYER):
            eager.write(layer, k[i, layer], v[i, layer])
            outs.append(eager.attend(layer, q[i, layer]).clone())
        eager.advance()
        eager_out.append(torch.stack(outs))

    graphed = _container(cuda_device, steps + 4)
    # first step eager (what an engine does before capturing), then replays
    graphed.build_mask(next_token=True)
    first = []
    for layer in range(N_LAYER):
        graphed.write(layer, k[0, layer], v[0, layer])
        first.append(graphed.attend(layer, q[0, layer]).clone())
    graphed.advance()
    assert torch.equal(torch.stack(first), eager_out[0])

    qb, kb, vb = q[0].clone(), k[0].clone(), v[0].clone()
    graph = PagedStepGraph(graphed, qb, kb, vb)
    assert graph.launches_per_step == N_LAYER  # one fused append + decode launch per layer
    for i in range(1, steps + 1):
        qb.copy_(q[i]), kb.copy_(k[i]), vb.copy_(v[i])
        out = graph.replay()
        assert torch.equal(out, eager_out[i]), f"step {i}: max diff {(out.float() - eager_out[i].float()).abs().max()}"

    assert graphed._host_pos == eager._host_pos and graphed._host_valid == eager._host_valid
    assert torch.equal(graphed.pos, eager.pos) and torch.equal(graphed.valid, eager.valid)
    for a, b in zip(graphed.pool.keys + graphed.pool.values, eager.pool.keys + eager.pool.values):
        assert torch.equal(a, b)

    # and the last step against the oracle (fp32 reference over the same pools)
    seqlen = (graphed.pos).to(torch.int32).cpu()
    ref, _ = oracle.paged_decode(q[steps, 0, :, :, 0, :].cpu(), graphed.pool.keys[0].cpu(),
                                 graphed.pool.values[0].cpu(), graphed._block_table_tensor.cpu(), seqlen)
    got = eager_out[steps][0, :, :, 0, :].float().cpu()
    assert (got - ref).abs().max().item() < 4e-3


def test_replay_past_the_position_bound_is_refused(cuda_device):
    from serve.graph import PagedStepGraph

    kv = _container(cuda_device, 2)
    q, k, v = _inputs(cuda_device, 1)
    graph = PagedStepGraph(kv, q[0].clone(), k[0].clone(), v[0].clone())
    graph.replay()
    graph.replay()
    pos_before = kv.pos.clone()
    with pytest.raises(IndexError):
        graph.replay()
    torch.cuda.synchronize()
    assert torch.equal(kv.pos, pos_before)

