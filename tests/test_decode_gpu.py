"""Decode kernel (``pd_decode`` through ``paged_decode``) against the CPU oracle on a B200.

Shapes are the reference's kernel grid (tests/unit/test_triton_decode.py:263-292) plus the
Qwen3-0.6B head shape; tolerances: fp32 1e-4, bf16 <= 2e-3 absolute (|out| < 1) or a
correctly rounded bf16 result, and argmax equality for bf16 as in the reference.
"""

from __future__ import annotations

import pytest
import torch

from helpers import assert_output_close, build_case
from oracle import oracle

pytestmark = pytest.mark.gpu

SHAPES = [
    pytest.param(1, 2, 2, 64, 16, [1], id="b1-gqa1-d64-l1-bs16"),
    pytest.param(3, 8, 4, 128, 16, [15, 16, 17], id="b3-gqa2-d128-l15-17-bs16"),
    pytest.param(8, 8, 2, 64, 32, [1, 15, 16, 17, 100, 1, 15, 16], id="b8-gqa4-d64-bs32"),
    pytest.param(1, 8, 1, 256, 16, [1664], id="b1-gqa8-d256-l1664-bs16"),
    pytest.param(3, 8, 1, 256, 32, [100, 1664, 1], id="b3-gqa8-d256-bs32"),
    pytest.param(8, 16, 8, 128, 16, [1664] * 8, id="qwen3-b8-l1664"),
    pytest.param(4, 16, 8, 128, 16, [0, 5, 3000, 129], id="qwen3-ragged-zero"),
    pytest.param(2, 8, 2, 256, 16, [700, 33], id="qwen35-d256-gqa4"),
    pytest.param(2, 4, 2, 32, 16, [40, 7], id="d32"),
    pytest.param(2, 4, 4, 16, 8, [40, 7], id="d16-bs8"),
    pytest.param(2, 6, 2, 64, 16, [90, 300], id="gqa3-chunks"),
    pytest.param(2, 32, 2, 64, 16, [90, 300], id="gqa16-chunks"),
    # one warp per (kv head, q chunk) item: the column split, with fewer columns than CTAs
    pytest.param(3, 16, 8, 128, 16, [1, 17, 40], id="qwen3-columns-lt-ctas"),
    pytest.param(2, 16, 8, 64, 16, [4000, 2], id="qwen3-d64-columns"),
    pytest.param(5, 64, 8, 128, 16, [33, 700, 1, 2500, 64], id="gqa8-columns"),
    # tensor-core tiles made of several TMA boxes (blocks smaller than a tile), and a block
    # size below 8 tokens (CUDA-core tile math)
    pytest.param(2, 16, 8, 128, 8, [300, 17], id="d128-bs8-two-boxes"),
    pytest.param(2, 8, 2, 64, 8, [301, 9], id="d64-bs8-four-boxes"),
    pytest.param(2, 8, 2, 256, 8, [129, 8], id="d256-bs8"),
    pytest.param(2, 8, 2, 128, 4, [50, 3], id="d128-bs4"),
]


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16], ids=["fp32", "bf16", "fp16"])
@pytest.mark.parametrize("B,H,Hkv,D,bs,lengths", SHAPES)
def test_decode_matches_oracle(cuda_device, B, H, Hkv, D, bs, lengths, dtype):
    from model.triton_decode import paged_decode

    q, k, v, table, seqlen = build_case(B, H, Hkv, D, bs, lengths, dtype=dtype, seed=13)
    ref_f32, ref = oracle.paged_decode(q, k, v, table, seqlen)
    got = paged_decode(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), table.to(cuda_device),
                       seqlen.to(cuda_device))
    torch.cuda.synchronize()
    assert got.shape == (B, H, D) and got.dtype == dtype
    assert_output_close(got, ref_f32, dtype)
    if dtype != torch.float32:
        # argmax agreement as in the reference's tests, up to rounding: the element the kernel
        # ranks first must be within one output ulp (or 4e-3) of the true maximum
        nz = seqlen > 0
        g, r = got.cpu()[nz].float(), ref_f32[nz]
        picked = r.gather(-1, g.argmax(-1, keepdim=True)).squeeze(-1)
        top = r.max(-1).values
        ulp = 2.0 ** (torch.floor(torch.log2(top.abs().clamp_min(1e-30))) - (7 if dtype == torch.bfloat16 else 10))
        assert (top - picked <= torch.maximum(ulp, torch.full_like(ulp, 4e-3))).all()
    from model import _native
    assert _native.device_error() == 0


@pytest.mark.parametrize("mode,row_cost", [(0, 2), (1, 2), (2, 2), (0, 0), (0, 7), (2, 0)],
                         ids=["tensor-core", "shared-stage", "cuda-core", "tensor-core-rowcost0",
                              "tensor-core-rowcost7", "cuda-core-rowcost0"])
@pytest.mark.parametrize("B,H,Hkv,D,bs,lengths", [
    (8, 16, 8, 128, 16, [1664] * 8),
    (6, 16, 8, 128, 16, [0, 5, 3000, 129, 16, 17]),
    (3, 16, 8, 128, 16, [1, 17, 40]),
    (4, 32, 8, 128, 16, [700, 33, 2048, 1]),     # 4 q heads per kv head
    (2, 16, 8, 64, 32, [4000, 2]),
    (2, 16, 8, 256, 16, [900, 77]),
    (3, 16, 4, 128, 16, [300, 1, 2100]),         # 4 items per row: per-warp kernel in every mode
    (3, 8, 2, 256, 16, [2048, 5, 700]),          # Qwen3.5 full-attention heads
    (2, 64, 8, 128, 16, [1000, 3]),              # 8 q heads per kv head
])
def test_both_decode_kernels_match_the_oracle(cuda_device, mode, row_cost, B, H, Hkv, D, bs, lengths):
    from model import _native
    from model.triton_decode import paged_decode

    before = _native.get_decode_mode()
    try:
        _native.set_decode_mode(mode, 0, row_cost)
        for dtype in (torch.bfloat16, torch.float16):
            q, k, v, table, seqlen = build_case(B, H, Hkv, D, bs, lengths, dtype=dtype, seed=29)
            ref_f32, _ = oracle.paged_decode(q, k, v, table, seqlen)
            got = paged_decode(q.to(cuda_device), k.to(cuda_device), v.to(cuda_device), table.to(cuda_device),
                               seqlen.to(cuda_device))
            torch.cuda.synchronize()
            assert_output_close(got, ref_f32, dtype)
            assert not got[seqlen.to(cuda_device) == 0].any()
    finally:
        _native.set_decode_mode(*before)
    assert _native.device_error() == 0


def test_one_workspace_serves_any_shape_sequence_without_clearing(cuda_device):
    """A workspace reused across shapes (and pre-filled with garbage) needs no clearing: the
    split-row counters carry a per-launch epoch. Regression for a cached workspace whose
    counter region grew over the previous shape's partials."""
    from model import _native

    ws = torch.full((64 << 20,), 0xFF, dtype=torch.uint8, device=cuda_device)
    ws[::7] = 0x3C
    cases = [(8, 16, 8, 128, 16, [700] * 8), (32, 16, 8, 128, 16, [2100] * 32),
             (2, 16, 8, 128, 16, [5000, 10]), (32, 16, 8, 128, 16, [2100] * 32)]
    for i, (B, H, Hkv, D, bs, lengths) in enumerate(cases):
        q, k, v, table, seqlen = build_case(B, H, Hkv, D, bs, lengths, dtype=torch.bfloat16, seed=40 + i)
        ref_f32, _ = oracle.paged_decode(q, k, v, table, seqlen)
        qd = q.to(cuda_device)
        out = torch.empty_like(qd)
        assert _native.workspace_bytes(B, H, Hkv, D, q.dtype) <= ws.numel()
        _native.decode(qd, k.to(cuda_device), v.to(cuda_device), table.to(cuda_device), seqlen.to(cuda_device),
                       out, _native.log2e_scale(1 / D ** 0.5), ws)
        torch.cuda.synchronize()
        assert_output_close(out, ref_f32, torch.bfloat16)
    assert _native.device_error() == 0
