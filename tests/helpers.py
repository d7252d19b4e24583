"""Shared builders and tolerance checks for the parity tests."""

from __future__ import annotations

import contextlib

import torch

#: Output tolerance for bf16/fp16 results against the fp32 oracle. 2e-3 absolute is the
#: bar for |out| < 1 (half a bf16 ulp is <= 1.95e-3 there); above 1 the bound is half an
#: ulp of the reference value plus fp32 slack, i.e. a correctly rounded result.
HALF_TOL_ABS = 2e-3
FP32_TOL = 1e-4


def build_case(B, H, Hkv, D, block_size, lengths, *, device="cpu", dtype=torch.float32, seed=0,
               n_blocks=None):
    """Random pool plus per-row random block tables (rows may share blocks).

    Mirrors the reference's test builder (tests/unit/test_triton_decode.py:48-72): one
    column per logical page of the longest row, unused tail entries left 0 (a valid id),
    K, V, q drawn in that order from one CPU generator.
    """
    gen = torch.Generator().manual_seed(seed)
    pages = [(int(n) + block_size - 1) // block_size for n in lengths]
    max_pages = max(max(pages), 1)
    if n_blocks is None:
        n_blocks = max(B * max_pages, max_pages + 4)
    k = torch.randn(n_blocks, block_size, Hkv, D, generator=gen).to(device=device, dtype=dtype)
    v = torch.randn(n_blocks, block_size, Hkv, D, generator=gen).to(device=device, dtype=dtype)
    q = torch.randn(B, H, D, generator=gen).to(device=device, dtype=dtype)
    table = torch.zeros(B, max_pages, dtype=torch.int32)
    for row, n_pages in enumerate(pages):
        if n_pages:
            table[row, :n_pages] = torch.randperm(n_blocks, generator=gen)[:n_pages].to(torch.int32)
    seqlen = torch.tensor(lengths, dtype=torch.int32)
    return q, k, v, table.to(device), seqlen.to(device)


def max_abs(a, b) -> float:
    return (a.float().cpu() - b.float().cpu()).abs().max().item() if a.numel() else 0.0


def assert_output_close(got, ref_f32, dtype):
    """got (kernel, in dtype) vs the fp32 oracle result."""
    got = got.float().cpu()
    ref = ref_f32.float().cpu()
    assert torch.isfinite(got).all(), "a finite input produced NaN/Inf"
    diff = (got - ref).abs()
    if dtype == torch.float32:
        assert diff.max().item() <= FP32_TOL, f"max|delta| {diff.max().item()} > {FP32_TOL}"
        return diff.max().item()
    ulp_half = (2.0 ** (torch.floor(torch.log2(ref.abs().clamp_min(1e-30))) - (8 if dtype == torch.bfloat16 else 11)))
    bound = torch.maximum(torch.full_like(ref, HALF_TOL_ABS), ulp_half * 1.001 + 1e-5)
    bad = diff > bound
    assert not bad.any(), (
        f"{int(bad.sum())} elements beyond tolerance; max|delta| {diff.max().item()}"
    )
    return diff.max().item()


@contextlib.contextmanager
def decode_mode(mode: int, shared_stages: int = 0, row_cost: int = -1):
    """Runs the body with pd_set_decode_mode(mode, ...) and restores the previous choice.
    0: per-warp kernel with tensor-core tile math where it applies, 1: shared stages where
    they apply, 2: per-warp kernel with CUDA-core tile math."""
    from model import _native

    before = _native.get_decode_mode()
    _native.set_decode_mode(mode, shared_stages, row_cost)
    try:
        yield
    finally:
        _native.set_decode_mode(*before)


def oracle_rows(oracle, q, k, v, table, seqlen, rows):
    """fp32 oracle output of ``rows`` only, from a CPU copy of just the pool blocks those rows
    use (the full pools of the large configs are GBs)."""
    tab = table[rows].long()
    ids = torch.unique(tab)
    remap = torch.full((int(ids.max()) + 1,), -1, dtype=torch.long, device=tab.device)
    remap[ids] = torch.arange(ids.numel(), device=tab.device)
    local = remap[tab].to(torch.int32).cpu()
    ref, _ = oracle.paged_decode(q[rows].cpu(), k[ids].cpu(), v[ids].cpu(), local, seqlen[rows].cpu())
    return ref
