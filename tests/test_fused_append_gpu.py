"""Fused append + decode (``pd_plan_run_append``) against the two-launch path on a B200.

The contract: one launch that stores every row's new K/V at ``pos[row]`` and decodes equals
``pd_kv_append_table`` followed by ``pd_plan_run`` -- output AND pools bit-identical -- when
rows do not share blocks. ``PagedKV`` uses it by default; every other observer of the pool
(reading ``PagedPool.keys``, another write, the step hooks) sees the append first.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from helpers import assert_output_close, decode_mode
from oracle import oracle

pytestmark = pytest.mark.gpu


def _disjoint_case(B, H, Hkv, D, bs, lengths, *, dtype, seed, device):
    """Pool, q and per-row tables that never share a block (one permutation split by row)."""
    gen = torch.Generator().manual_seed(seed)
    pages = [max(1, -(-(n + 1) // bs)) for n in lengths]  # room for the appended token
    n_blocks = sum(pages) + 3
    k = torch.randn(n_blocks, bs, Hkv, D, generator=gen).to(dtype)
    v = torch.randn(n_blocks, bs, Hkv, D, generator=gen).to(dtype)
    q = torch.randn(B, H, D, generator=gen).to(dtype)
    perm = torch.randperm(n_blocks, generator=gen)
    table = torch.zeros(B, max(pages), dtype=torch.int32)
    at = 0
    for row, n in enumerate(pages):
        table[row, :n] = perm[at:at + n].to(torch.int32)
        at += n
    k_new = torch.randn(B, Hkv, D, generator=gen).to(dtype)
    v_new = torch.randn(B, Hkv, D, generator=gen).to(dtype)
    return [t.to(device) for t in (q, k, v, table, k_new, v_new)]


CASES = [
    pytest.param(32, 16, 8, 128, 16, [2048] * 32, torch.bfloat16, id="qwen3-b32-l2048"),
    pytest.param(5, 16, 8, 128, 16, [1, 16, 17, 700, 3000], torch.bfloat16, id="qwen3-ragged"),
    pytest.param(3, 8, 2, 64, 32, [31, 32, 100], torch.float16, id="gqa4-d64-bs32"),
    pytest.param(2, 32, 2, 64, 16, [90, 300], torch.bfloat16, id="gqa16-chunks"),
    pytest.param(2, 8, 2, 256, 16, [700, 33], torch.bfloat16, id="d256-gqa4"),
    pytest.param(4, 4, 2, 32, 8, [5, 9, 64, 1], torch.float32, id="fp32-d32-bs8"),
    pytest.param(3, 16, 8, 128, 8, [7, 8, 301], torch.bfloat16, id="d128-bs8-two-boxes"),
]


@pytest.mark.parametrize("mode", [0, 2], ids=["tensor-core", "cuda-core"])
@pytest.mark.parametrize("B,H,Hkv,D,bs,lengths,dtype", CASES)
def test_one_launch_equals_append_then_decode(cuda_device, B, H, Hkv, D, bs, lengths, dtype, mode):
    from model import _native
    from model.triton_decode import paged_decode_plan

    q, k, v, table, k_new, v_new = _disjoint_case(B, H, Hkv, D, bs, lengths, dtype=dtype, seed=B * 7 + D,
                                                  device=cuda_device)
    pos = torch.tensor(lengths, dtype=torch.int64, device=cuda_device)  # append at the end
    seqlen = (pos + 1).to(torch.int32)                                   # ... and attend over it
    k2, v2 = k.clone(), v.clone()

    with decode_mode(mode):
        fused = paged_decode_plan(q, [k], [v], table, seqlen)
        out_fused = fused.run_append(0, q, k_new, v_new, pos)
        split = paged_decode_plan(q, [k2], [v2], table, seqlen)
        _native.append_table(k2, v2, table, pos, k_new, v_new)
        out_split = split.run(0, q)
        torch.cuda.synchronize()
    assert torch.equal(out_fused, out_split), (out_fused.float() - out_split.float()).abs().max()
    assert torch.equal(k, k2) and torch.equal(v, v2)
    ref, _ = oracle.paged_decode(q.cpu(), k.cpu(), v.cpu(), table.cpu(), seqlen.cpu())
    assert_output_close(out_fused, ref, dtype)
    assert _native.device_error() == 0


def test_appending_inside_the_row_patches_the_right_tile(cuda_device):
    """pos < seqlen - 1 (a rewrite of an earlier token) lands in a middle tile; the pool and
    the output still match the two-launch path."""
    from model import _native
    from model.triton_decode import paged_decode_plan

    lengths = [2048, 513, 40]
    q, k, v, table, k_new, v_new = _disjoint_case(3, 16, 8, 128, 16, lengths, dtype=torch.bfloat16, seed=5,
                                                  device=cuda_device)
    pos = torch.tensor([0, 257, 39], dtype=torch.int64, device=cuda_device)
    seqlen = torch.tensor(lengths, dtype=torch.int32, device=cuda_device)
    k2, v2 = k.clone(), v.clone()
    out_fused = paged_decode_plan(q, [k], [v], table, seqlen).run_append(0, q, k_new, v_new, pos)
    _native.append_table(k2, v2, table, pos, k_new, v_new)
    out_split = paged_decode_plan(q, [k2], [v2], table, seqlen).run(0, q)
    torch.cuda.synchronize()
    assert torch.equal(out_fused, out_split) and torch.equal(k, k2) and torch.equal(v, v2)
    assert _native.device_error() == 0


def test_position_outside_the_table_is_skipped_and_flagged(cuda_device):
    from model import _native
    from model.triton_decode import paged_decode_plan

    _native.device_error(clear=True)
    lengths = [40, 20]
    q, k, v, table, k_new, v_new = _disjoint_case(2, 4, 2, 64, 16, lengths, dtype=torch.bfloat16, seed=9,
                                                  device=cuda_device)
    capacity = table.shape[1] * 16
    pos = torch.tensor([capacity + 5, 20], dtype=torch.int64, device=cuda_device)
    seqlen = torch.tensor([40, 21], dtype=torch.int32, device=cuda_device)
    k2, v2 = k.clone(), v.clone()
    out_fused = paged_decode_plan(q, [k], [v], table, seqlen).run_append(0, q, k_new, v_new, pos)
    torch.cuda.synchronize()
    assert _native.device_error(clear=True) == _native.DEVERR_APPEND_RANGE
    _native.append_table(k2, v2, table, pos, k_new, v_new)
    out_split = paged_decode_plan(q, [k2], [v2], table, seqlen).run(0, q)
    assert _native.device_error(clear=True) == _native.DEVERR_APPEND_RANGE
    assert torch.equal(out_fused, out_split) and torch.equal(k, k2) and torch.equal(v, v2)


def _container_steps(device, fuse: bool, steps=3, n_layer=2):
    from model.paged import PagedKV, PagedPool
    from serve.block_manager import BlockManager

    B, Hkv, H, D, bs = 6, 8, 16, 128, 16
    lengths = [17, 300, 1, 64, 1000, 15]
    manager = BlockManager(64 * 4, bs)
    tables = [manager.reserve(manager.blocks_for(n, steps)) for n in lengths]
    pool = PagedPool(n_layer, manager.n_blocks, bs, Hkv, D, dtype=torch.bfloat16, device=device, n_head=H)
    gen = torch.Generator(device=device).manual_seed(3)
    for t in pool.keys + pool.values:
        t.copy_(torch.randn(t.shape, generator=gen, device=device))
    kv = PagedKV(pool, tables, lengths, rope_len=2048, n_head=H, fuse_append=fuse)
    outs = []
    for step in range(steps):
        kv.build_mask(next_token=True)
        for layer in range(n_layer):
            k = torch.randn(B, Hkv, 1, D, generator=gen, device=device).to(torch.bfloat16)
            v = torch.randn(B, Hkv, 1, D, generator=gen, device=device).to(torch.bfloat16)
            q = torch.randn(B, H, 1, D, generator=gen, device=device).to(torch.bfloat16)
            kv.write(layer, k, v)
            outs.append(kv.attend(layer, q))
        kv.advance()
    return kv, pool, outs


def test_paged_kv_fused_steps_equal_unfused_steps(cuda_device):
    kv_f, pool_f, outs_f = _container_steps(cuda_device, fuse=True)
    kv_u, pool_u, outs_u = _container_steps(cuda_device, fuse=False)
    assert kv_f.fuse_append and not kv_u.fuse_append
    for a, b in zip(outs_f, outs_u):
        assert torch.equal(a, b)
    for a, b in zip(pool_f.keys + pool_f.values, pool_u.keys + pool_u.values):
        assert torch.equal(a, b)


def test_a_recorded_append_is_visible_to_every_other_observer(cuda_device):
    from model.paged import PagedKV, PagedPool

    pool = PagedPool(2, 8, 16, 2, 8, dtype=torch.bfloat16, device=cuda_device, n_head=4)
    kv = PagedKV(pool, [[3, 1]], [17], rope_len=64, n_head=4)
    assert kv.fuse_append
    kv.build_mask(next_token=True)
    k = torch.randn(1, 2, 1, 8, device=cuda_device).to(torch.bfloat16)
    kv.write(0, k, k)
    assert pool._pending is not None            # recorded, not launched
    slot = 1 * 16 + 1
    assert torch.equal(pool.keys[0].view(-1, 2, 8)[slot], k[0, :, 0, :])  # reading flushes
    assert pool._pending is None
    kv.write(1, k, k)
    kv.attend(0, torch.randn(1, 4, 1, 8, device=cuda_device).to(torch.bfloat16))  # other layer: flushed
    assert pool._pending is None
    assert torch.equal(pool.values[1].view(-1, 2, 8)[slot], k[0, :, 0, :])


def test_shared_blocks_disable_fusion(cuda_device):
    from model.paged import PagedKV, PagedPool

    pool = PagedPool(1, 8, 16, 2, 8, dtype=torch.bfloat16, device=cuda_device, n_head=4)
    kv = PagedKV(pool, [[3, 1], [3, 2]], [17, 17], rope_len=64, n_head=4)
    assert not kv.fuse_append



GOLDEN = Path(__file__).resolve().parent / "golden"
ROPE_CASES = json.loads((GOLDEN / "golden_meta.json").read_text())["rope"]


@pytest.mark.parametrize("rec", ROPE_CASES, ids=[r["key"] for r in ROPE_CASES])
@pytest.mark.parametrize("fuse", [True, False], ids=["fused", "two-launch"])
def test_rotated_append_stores_the_reference_rotation(cuda_device, rec, fuse):
    """K rows given before RoPE are stored exactly as the reference's apply_rotary_emb_partial
    rotates them (golden vectors from the reference itself), and the decode over them matches
    the oracle."""
    from model.paged import PagedKV, PagedPool

    tensors = torch.load(GOLDEN / "golden_tensors.pt")
    key = rec["key"]
    k_pre, cos, sin, k_ref = (tensors[key + part] for part in ("/k", "/cos", "/sin", "/out"))
    B, _, Hkv, D = k_pre.shape
    dtype = k_pre.dtype
    H, bs = 2 * Hkv, 16
    lengths = [5 + 37 * i for i in range(B)]
    pages = [-(-(n + 2) // bs) for n in lengths]
    pool = PagedPool(1, sum(pages) + 2, bs, Hkv, D, dtype=dtype, device=cuda_device, n_head=H)
    gen = torch.Generator(device=cuda_device).manual_seed(4)
    for t in pool.keys + pool.values:
        t.copy_(torch.randn(t.shape, generator=gen, device=cuda_device).to(dtype))
    tables, at = [], 0
    for n in pages:
        tables.append(list(range(at, at + n)))
        at += n
    kv = PagedKV(pool, tables, lengths, rope_len=max(lengths) + 4, n_head=H, fuse_append=fuse)
    kv.build_mask(next_token=True)
    k_in = k_pre.permute(0, 2, 1, 3).to(cuda_device)  # (B, H_kv, 1, D), as the layer passes it
    v_in = torch.randn(B, Hkv, 1, D, generator=gen, device=cuda_device).to(dtype)
    q = torch.randn(B, H, 1, D, generator=gen, device=cuda_device).to(dtype)
    kv.write(0, k_in, v_in, rope=(cos.to(cuda_device), sin.to(cuda_device)))
    out = kv.attend(0, q)
    torch.cuda.synchronize()

    keys = pool.keys[0].cpu()
    bits = (lambda t: t) if dtype == torch.float32 else (lambda t: t.contiguous().view(torch.uint8))
    for row, n in enumerate(lengths):
        stored = keys[tables[row][n // bs], n % bs]
        assert torch.equal(bits(stored), bits(k_ref[row, 0])), f"row {row}"
    table = torch.zeros(B, max(pages), dtype=torch.int32)
    for row, t in enumerate(tables):
        table[row, : len(t)] = torch.tensor(t, dtype=torch.int32)
    seqlen = torch.tensor([n + 1 for n in lengths], dtype=torch.int32)
    ref, _ = oracle.paged_decode(q[:, :, 0].cpu(), keys, pool.values[0].cpu(), table, seqlen)
    assert_output_close(out[:, :, 0], ref, dtype)
