"""Paged-KV append kernels on a B200: bit-exact against the oracle and the reference's goldens.

Mirrors tests/unit/test_paged_kv.py:99-220 and 441-542 of the reference: prefill writes
(block boundaries, shuffled tables, non-zero start, block size 16/32), the decode slot write
(``PagedKV.write`` -> fused table append) and its bounds behaviour, plus dtype casts.
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest
import torch

from oracle import oracle

pytestmark = pytest.mark.gpu

GOLDEN = Path(__file__).resolve().parent / "golden"
META = json.loads((GOLDEN / "golden_meta.json").read_text())
TENSORS = torch.load(GOLDEN / "golden_tensors.pt")
DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16}


def _pool(n_blocks=8, bs=16, n_layer=2, hkv=2, d=8, dtype=torch.float32, dev="cuda"):
    from model.paged import PagedPool

    return PagedPool(n_layer, n_blocks, bs, hkv, d, dtype=dtype, device=dev, n_head=2 * hkv)


@pytest.mark.parametrize("rec", [r for r in META["append"] if "prefill" in r["key"]], ids=lambda r: r["key"])
def test_prefill_writes_match_the_reference_pool_bytes(cuda_device, rec):
    dtype = DTYPES[rec["dtype"]]
    key = rec["key"]
    pool = _pool(rec["n_blocks"], rec["block_size"], dtype=dtype, dev=cuda_device)
    k = TENSORS[key + "/k"].to(cuda_device).permute(1, 0, 2).contiguous().permute(1, 0, 2)  # engine layout
    v = TENSORS[key + "/v"].to(cuda_device).permute(1, 0, 2).contiguous().permute(1, 0, 2)
    assert not k.is_contiguous()
    pool.write_prefill(0, rec["table0"], rec["start0"], k, v)
    pool.write_prefill(1, rec["table1"], rec["start1"], TENSORS[key + "/k2"].to(cuda_device),
                       TENSORS[key + "/v2"].to(cuda_device))
    torch.cuda.synchronize()
    for layer in range(2):
        assert torch.equal(pool.keys[layer].cpu(), TENSORS[f"{key}/keys{layer}"]), f"layer {layer} keys"
        assert torch.equal(pool.values[layer].cpu(), TENSORS[f"{key}/values{layer}"]), f"layer {layer} values"


@pytest.mark.parametrize("rec", [r for r in META["append"] if "token" in r["key"]], ids=lambda r: r["key"])
def test_decode_write_matches_write_token_reference(cuda_device, rec):
    from model.paged import PagedKV

    dtype = DTYPES[rec["dtype"]]
    pool = _pool(rec["n_blocks"], rec["block_size"], n_layer=1, d=4, dtype=dtype, dev=cuda_device)
    kv = PagedKV(pool, rec["tables"], rec["positions"], rope_len=64, n_head=4)
    k = TENSORS[rec["key"] + "/k"].to(cuda_device).unsqueeze(2)  # (B, H_kv, 1, D)
    v = TENSORS[rec["key"] + "/v"].to(cuda_device).unsqueeze(2)
    kv.write(0, k, v)
    torch.cuda.synchronize()
    assert torch.equal(pool.keys[0].cpu(), TENSORS[rec["key"] + "/keys"])
    assert torch.equal(pool.values[0].cpu(), TENSORS[rec["key"] + "/values"])


@pytest.mark.parametrize("src,dst", [(torch.float32, torch.bfloat16), (torch.bfloat16, torch.bfloat16),
                                     (torch.float32, torch.float16), (torch.bfloat16, torch.float32),
                                     (torch.float16, torch.float16)])
@pytest.mark.parametrize("slot_dtype", [torch.int64, torch.int32])
def test_write_slots_is_bit_exact_with_casts(cuda_device, src, dst, slot_dtype):
    gen = torch.Generator().manual_seed(5)
    n_blocks, bs, hkv, d = 12, 16, 4, 64
    pool = _pool(n_blocks, bs, n_layer=1, hkv=hkv, d=d, dtype=dst, dev=cuda_device)
    perm = torch.randperm(n_blocks * bs, generator=gen)[:37]
    k = (torch.randn(37, hkv, d, generator=gen) * 3).to(src)
    v = (torch.randn(37, hkv, d, generator=gen) * 3).to(src)
    pool.write_slots(0, perm.to(slot_dtype).to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    ref_k = torch.zeros(n_blocks, bs, hkv, d, dtype=dst)
    ref_v = torch.zeros_like(ref_k)
    assert oracle.append_slots(ref_k, ref_v, perm, k, v) == 0
    torch.cuda.synchronize()
    assert torch.equal(pool.keys[0].cpu().view(torch.uint8), ref_k.view(torch.uint8))
    assert torch.equal(pool.values[0].cpu().view(torch.uint8), ref_v.view(torch.uint8))
    # torch's own cast agrees with the oracle's (the reference writes k.to(pool.dtype))
    flat = ref_k.view(-1, hkv, d)
    assert torch.equal(flat[perm].view(torch.uint8), k.to(dst).view(torch.uint8))


def test_unaligned_and_strided_sources_take_the_scalar_path(cuda_device):
    """head_dim 12 (not a multiple of 8) and a non-unit-stride source still copy exactly."""
    from model.paged import PagedPool

    gen = torch.Generator().manual_seed(6)
    pool = PagedPool(1, 4, 16, 2, 12, dtype=torch.float32, device=cuda_device)
    k = torch.randn(5, 2, 12, generator=gen)
    v = torch.randn(5, 2, 12, generator=gen)
    slots = torch.tensor([3, 17, 40, 63, 0])
    pool.write_slots(0, slots.to(cuda_device), k.to(cuda_device), v.to(cuda_device))
    ref_k = torch.zeros(4, 16, 2, 12)
    ref_v = torch.zeros_like(ref_k)
    oracle.append_slots(ref_k, ref_v, slots, k, v)
    torch.cuda.synchronize()
    assert torch.equal(pool.keys[0].cpu(), ref_k) and torch.equal(pool.values[0].cpu(), ref_v)


def test_slot_write_crosses_a_block_boundary_with_a_shuffled_table(cuda_device):
    from model.paged import PagedKV

    pool = _pool(dev=cuda_device, d=4)
    table = [5, 1, 7]
    kv = PagedKV(pool, [table], [15], rope_len=64, n_head=4)
    before = pool.keys[0].clone()
    k = torch.randn(1, 2, 1, 4, device=cuda_device)
    kv.write(0, k, torch.randn(1, 2, 1, 4, device=cuda_device))
    flat = pool.keys[0].view(-1, 2, 4)
    slot = 5 * 16 + 15
    assert torch.equal(flat[slot], k[0, :, 0, :])
    changed = (pool.keys[0] != before).any(dim=-1).any(dim=-1).view(-1).nonzero().tolist()
    assert changed == [[slot]]


def test_rebuilt_container_writes_through_its_own_table(cuda_device):
    from model.paged import PagedKV

    pool = _pool(dev=cuda_device, d=4)
    k_a = torch.randn(1, 2, 1, 4, device=cuda_device)
    k_b = torch.randn(1, 2, 1, 4, device=cuda_device)
    v = torch.zeros(1, 2, 1, 4, device=cuda_device)
    PagedKV(pool, [[0, 1, 2]], [5], rope_len=64, n_head=4).write(0, k_a, v)
    PagedKV(pool, [[3, 4, 5]], [5], rope_len=64, n_head=4).write(0, k_b, v)
    flat = pool.keys[0].view(-1, 2, 4)
    assert torch.equal(flat[5], k_a[0, :, 0, :]) and torch.equal(flat[3 * 16 + 5], k_b[0, :, 0, :])


def test_write_past_the_block_table_raises_before_touching_the_pool(cuda_device):
    from model.paged import PagedKV

    pool = _pool(n_blocks=4, dev=cuda_device, d=4)
    kv = PagedKV(pool, [[0]], [16], rope_len=32, n_head=4)
    before = pool.keys[0].clone()
    k = torch.randn(1, 2, 1, 4, device=cuda_device)
    with pytest.raises(IndexError, match="block table has 1 blocks"):
        kv.write(0, k, k)
    assert torch.equal(pool.keys[0], before)
    kv2 = PagedKV(pool, [[1]], [15], rope_len=32, n_head=4)
    kv2.build_mask(next_token=True)
    kv2.write(0, k, k)
    kv2.advance()
    assert kv2._slot_ids is None
    with pytest.raises(IndexError, match="needs block 1"):
        kv2.write(0, k, k)


def test_out_of_pool_slot_is_skipped_and_flagged_not_faulted(cuda_device):
    """The reference's index_copy_ would device-assert; the append kernel skips the slot and
    records PD_DEVERR_APPEND_RANGE in the device error word (the context stays usable)."""
    from model import _native

    _native.device_error(clear=True)
    pool = _pool(n_blocks=4, dev=cuda_device, d=8)
    k = torch.randn(2, 2, 8, device=cuda_device)
    pool.write_slots(0, torch.tensor([0, 10_000], device=cuda_device), k, k)
    assert _native.device_error(clear=True) == _native.DEVERR_APPEND_RANGE
    assert torch.equal(pool.keys[0].view(-1, 2, 8)[0], k[0])
    assert _native.device_error() == 0
