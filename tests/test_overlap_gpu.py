"""Overlapped launches (programmatic dependent launch) on a B200.

A launch made with ``overlap=True`` may start while the previous kernel of the stream runs:
it computes its work split and issues its first K/V copies, then waits for that kernel before
it reads q or the appended rows. The tests chain layers so that layer l+1 READS what layer l
WRITES (q_{l+1} = out_l, and for the fused append k_new/v_new taken from out_l): a read placed
before the wait would see a partly written buffer. The overlapped sequence must equal the
plain one bit for bit, eagerly and replayed from a CUDA graph.
"""

from __future__ import annotations

import pytest
import torch

from helpers import assert_output_close
from oracle import oracle

pytestmark = pytest.mark.gpu


def _chain_case(device, n_layer=6, B=32, H=16, Hkv=8, D=128, bs=16, ctx=1500, seed=3):
    gen = torch.Generator().manual_seed(seed)
    pages = -(-(ctx + 1) // bs)
    n_blocks = B * pages + 2
    perm = torch.randperm(n_blocks, generator=gen)
    table = perm[: B * pages].view(B, pages).to(torch.int32)
    ks = [torch.randn(n_blocks, bs, Hkv, D, generator=gen).to(torch.bfloat16).to(device) for _ in range(n_layer)]
    vs = [torch.randn(n_blocks, bs, Hkv, D, generator=gen).to(torch.bfloat16).to(device) for _ in range(n_layer)]
    q0 = torch.randn(B, H, D, generator=gen).to(torch.bfloat16).to(device)
    lengths = torch.randint(ctx // 2, ctx + 1, (B,), generator=gen)
    seqlen = lengths.to(torch.int32).to(device)
    return q0, ks, vs, table.to(device), seqlen


def _run_chain(plan, q0, n_layer, overlap):
    q, outs = q0, []
    for layer in range(n_layer):
        q = plan.run(layer, q, overlap=overlap and layer > 0)
        outs.append(q)
    return outs


def test_overlapped_layers_read_the_previous_layers_output(cuda_device):
    from model import _native
    from model.triton_decode import paged_decode_plan

    q0, ks, vs, table, seqlen = _chain_case(cuda_device)
    plan = paged_decode_plan(q0, ks, vs, table, seqlen)
    plain = [o.clone() for o in _run_chain(plan, q0, len(ks), overlap=False)]
    over = _run_chain(plan, q0, len(ks), overlap=True)
    torch.cuda.synchronize()
    for a, b in zip(plain, over):
        assert torch.equal(a, b)
    # the chain itself is the decode: check its first layer against the oracle
    ref, _ = oracle.paged_decode(q0.cpu(), ks[0].cpu(), vs[0].cpu(), table.cpu(), seqlen.cpu())
    assert_output_close(plain[0], ref, torch.bfloat16)

    # the same chain captured once and replayed
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        captured = _run_chain(plan, q0, len(ks), overlap=True)
    for _ in range(3):
        g.replay()
        torch.cuda.synchronize()
        for a, b in zip(plain, captured):
            assert torch.equal(a, b)
    assert _native.device_error() == 0


def test_overlapped_fused_append_reads_rows_the_previous_layer_wrote(cuda_device):
    from model import _native
    from model.triton_decode import paged_decode_plan

    q0, ks, vs, table, seqlen = _chain_case(cuda_device, n_layer=4, seed=9)
    Hkv = ks[0].shape[2]
    pos = (seqlen.to(torch.int64) - 1).clamp_min(0)
    pools = ([k.clone() for k in ks], [v.clone() for v in vs])

    def chain(k_pools, v_pools, overlap):
        plan = paged_decode_plan(q0, k_pools, v_pools, table, seqlen)
        q, outs = q0, []
        for layer in range(len(k_pools)):
            # the new K/V rows of layer l+1 are slices of layer l's output
            k_new, v_new = q[:, :Hkv, :], q[:, Hkv:2 * Hkv, :]
            q = plan.run_append(layer, q, k_new, v_new, pos, overlap=overlap and layer > 0)
            outs.append(q)
        return outs

    plain = [o.clone() for o in chain(ks, vs, overlap=False)]
    over = chain(*pools, overlap=True)
    torch.cuda.synchronize()
    for a, b in zip(plain, over):
        assert torch.equal(a, b)
    for a, b in zip(ks + vs, pools[0] + pools[1]):
        assert torch.equal(a, b)
    assert _native.device_error() == 0


def test_overlap_switch_is_per_launch(cuda_device):
    """A plan used with and without overlap keeps producing the same result."""
    from model.triton_decode import paged_decode_plan

    q0, ks, vs, table, seqlen = _chain_case(cuda_device, n_layer=2, B=4, ctx=300, seed=4)
    plan = paged_decode_plan(q0, ks, vs, table, seqlen)
    a = plan.run(1, q0)
    b = plan.run(1, q0, overlap=True)
    c = plan.run(1, q0)
    torch.cuda.synchronize()
    assert torch.equal(a, b) and torch.equal(a, c)


def test_paged_kv_overlaps_only_fused_layers_after_its_own_attend(cuda_device, monkeypatch):
    """In a decode step, layer 0 follows the seqlen update and must wait for it; layers 1.. of
    the fused path follow the previous layer's decode and may overlap it. The unfused path
    (a separate append just before each decode) never overlaps."""
    from model import _native
    from test_fused_append_gpu import _container_steps

    seen = []
    original = _native.NativePlan._set_overlap

    def spy(self, overlap):
        seen.append(bool(overlap))
        return original(self, overlap)

    monkeypatch.setattr(_native.NativePlan, "_set_overlap", spy)
    _container_steps(cuda_device, fuse=True, steps=2, n_layer=3)
    assert seen[-6:] == [False, True, True] * 2
    seen.clear()
    _container_steps(cuda_device, fuse=False, steps=2, n_layer=3)
    assert seen and not any(seen)
