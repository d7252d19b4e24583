"""Block-table-aware chunked prefill (``pd_prefill`` through ``paged_prefill``).

CPU tests pin the oracle (a one-token chunk is the paged decode; a long chunk equals the
same rows processed as separate shorter chunks) and the entry point's refusals. GPU tests
compare the sm_100a kernel with the oracle on the same seeded inputs: several group sizes,
head dims (64, 128, 256), block sizes (one and several TMA boxes per key tile, and key
tiles within a block), ragged chunks and contexts,
empty rows, and pools whose unused slots hold NaN. Tolerance: the decode suite's (fp32-exact
reference, output rounded to the pool dtype).
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

from helpers import assert_output_close
from oracle import oracle


def prefill_case(H, Hkv, D, bs, ctx, chunks, *, dtype=torch.bfloat16, seed=0, nan_fill=False):
    """Rows with `ctx[b]` earlier tokens and a chunk of `chunks[b]` new ones (K/V of all already
    in the pool). Returns q (total_q, H, D), k, v, table, cu_seqlens_q, seqlen_k."""
    gen = torch.Generator().manual_seed(seed)
    B = len(ctx)
    lens = [c + s for c, s in zip(ctx, chunks)]
    pages = [max(1, -(-n // bs)) for n in lens]
    n_blocks = sum(pages) + 2
    k = torch.randn(n_blocks, bs, Hkv, D, generator=gen).to(dtype)
    v = torch.randn(n_blocks, bs, Hkv, D, generator=gen).to(dtype)
    perm = torch.randperm(n_blocks, generator=gen)
    table = torch.zeros(B, max(pages) + 1, dtype=torch.int32)
    at = 0
    for row, n in enumerate(pages):
        table[row, :n] = perm[at:at + n].to(torch.int32)
        at += n
    if nan_fill:  # slots no row reads: past each row's length, and the spare blocks
        for row, n in enumerate(lens):
            for t in range(n, pages[row] * bs):
                blk = int(table[row, t // bs])
                k[blk, t % bs] = float("nan")
                v[blk, t % bs] = float("nan")
        for blk in perm[at:].tolist():
            k[blk] = float("nan")
            v[blk] = float("nan")
    cu = torch.tensor([0] + list(torch.tensor(chunks).cumsum(0).tolist()), dtype=torch.int32)
    q = torch.randn(int(cu[-1]), H, D, generator=gen).to(dtype)
    return q, k, v, table, cu, torch.tensor(lens, dtype=torch.int32)


# ------------------------------------------------------------------ oracle (CPU)


def test_oracle_one_token_chunks_are_the_decode():
    q, k, v, table, cu, sk = prefill_case(8, 2, 64, 16, [0, 30, 200], [1, 1, 1], seed=1)
    got, _ = oracle.paged_prefill(q, k, v, table, cu, sk)
    ref = oracle.dense_decode_py(q, k, v, table, sk)
    assert (got.double() - ref).abs().max().item() < 1e-6


def test_oracle_chunk_equals_its_tokens_one_by_one():
    """Causality: token i of a chunk sees exactly what a one-token chunk at its position sees."""
    q, k, v, table, cu, sk = prefill_case(4, 2, 64, 16, [37], [9], seed=2)
    whole, _ = oracle.paged_prefill(q, k, v, table, cu, sk)
    for i in range(9):
        one, _ = oracle.paged_prefill(q[i:i + 1], k, v, table, torch.tensor([0, 1], dtype=torch.int32),
                                      torch.tensor([37 + i + 1], dtype=torch.int32))
        assert (one[0] - whole[i]).abs().max().item() < 1e-6


def test_entry_point_refuses_unsupported_shapes_without_touching_memory():
    from model import _native

    lib = _native.require()
    strides = (ctypes.c_int64 * 3)(16 * 8 * 256, 8 * 256, 256)
    args = dict(batch=1, max_q=4, n_head=8, n_kv=8, head_dim=512, dtype=2)

    def call(**kw):
        a = {**args, **kw}
        return lib.pd_prefill(None, 0, 0, None, None, 4, 16, strides, strides, None, 0, 0, None, None,
                              None, 0, 0, a["batch"], a["max_q"], a["n_head"], a["n_kv"], a["head_dim"],
                              a["dtype"], 1.0, None)

    assert call() == 2                      # head_dim 512: PD_ERR_UNSUPPORTED
    assert call(head_dim=128, dtype=0) == 2  # fp32 pools
    assert call(head_dim=128, n_head=24, n_kv=2) == 2  # 12 q heads per kv head
    assert call(head_dim=128, n_head=12, n_kv=8) == 1  # heads not a multiple: PD_ERR_INVALID
    assert call(head_dim=96) == 1          # not a power of two


# ------------------------------------------------------------------ kernel (GPU)


@pytest.fixture(params=[0, 1], ids=["tcgen05", "mma_sync"])
def kernel(request):
    """Runs the test with the tcgen05 / TMEM prefill kernel (mode 0, the default) and with the
    mma.sync kernel (mode 1); both compute the same function."""
    from model import _native

    before = _native.get_prefill_mode()
    _native.set_prefill_mode(request.param)
    try:
        yield request.param
    finally:
        _native.set_prefill_mode(before)


CASES = [
    # H, Hkv, D, bs, ctx, chunks
    pytest.param(16, 8, 128, 16, [0, 100, 1000], [64, 7, 129], id="qwen3-g2-d128-bs16"),
    pytest.param(8, 2, 64, 32, [5, 0, 300, 63], [1, 33, 200, 64], id="g4-d64-bs32"),
    pytest.param(4, 4, 128, 64, [0, 700], [150, 65], id="g1-d128-bs64"),
    pytest.param(16, 2, 128, 8, [17, 0], [40, 8], id="g8-d128-bs8"),
    pytest.param(16, 8, 64, 128, [2000, 3], [300, 3], id="qwen3-d64-bs128"),
    pytest.param(8, 8, 128, 16, [0, 9], [0, 20], id="empty-row"),
    pytest.param(8, 2, 256, 16, [0, 700, 33], [96, 40, 1], id="qwen35-d256-g4"),
    pytest.param(16, 2, 256, 64, [100, 0], [70, 33], id="d256-g8-bs64"),
]


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16], ids=["bf16", "fp16"])
@pytest.mark.parametrize("H,Hkv,D,bs,ctx,chunks", CASES)
def test_prefill_matches_the_oracle(cuda_device, kernel, H, Hkv, D, bs, ctx, chunks, dtype):
    from model import _native
    from model.triton_decode import paged_prefill

    q, k, v, table, cu, sk = prefill_case(H, Hkv, D, bs, ctx, chunks, dtype=dtype, seed=len(ctx) + D)
    ref_f32, _ = oracle.paged_prefill(q, k, v, table, cu, sk)
    dev = [t.to(cuda_device) for t in (q, k, v, table, cu, sk)]
    got = paged_prefill(*dev, max(chunks))
    torch.cuda.synchronize()
    assert got.shape == q.shape and got.dtype == dtype
    assert_output_close(got, ref_f32, dtype)
    assert _native.device_error() == 0


@pytest.mark.gpu
def test_prefill_ignores_nan_in_slots_no_row_reads(cuda_device, kernel):
    from model import _native
    from model.triton_decode import paged_prefill

    q, k, v, table, cu, sk = prefill_case(16, 8, 128, 16, [3, 90], [50, 11], seed=5, nan_fill=True)
    ref_f32, _ = oracle.paged_prefill(q, k, v, table, cu, sk)
    got = paged_prefill(*[t.to(cuda_device) for t in (q, k, v, table, cu, sk)], 50)
    torch.cuda.synchronize()
    assert_output_close(got, ref_f32, torch.bfloat16)
    assert _native.device_error() == 0


@pytest.mark.gpu
@pytest.mark.parametrize("pad", ["block", "row"])
@pytest.mark.parametrize("D,bs", [(128, 16), (256, 32), (64, 8)])
def test_strided_pool_views(cuda_device, kernel, pad, D, bs):
    """Pools that are views of larger tensors. With padding between blocks (block stride
    above block_size x token stride) the tcgen05 kernel copies one 128-byte piece per box; with
    padded rows (token stride above n_kv_head x head_dim) it keeps the grouped boxes. Both
    layouts must give the oracle's output."""
    from model import _native
    from model.triton_decode import paged_prefill

    H, Hkv = 8, 2
    q, k, v, table, cu, sk = prefill_case(H, Hkv, D, bs, [70, 0, 333], [45, 130, 9], seed=D + bs)
    ref_f32, _ = oracle.paged_prefill(q, k, v, table, cu, sk)

    def padded(x):
        n = x.shape[0]
        if pad == "block":
            big = torch.full((n, bs + 8, Hkv, D), float("nan"), dtype=x.dtype)
            big[:, :bs] = x
            return big.to(cuda_device)[:, :bs]
        big = torch.full((n, bs, Hkv + 1, D), float("nan"), dtype=x.dtype)
        big[:, :, :Hkv] = x
        return big.to(cuda_device)[:, :, :Hkv]

    kp, vp = padded(k), padded(v)
    assert not kp.is_contiguous()
    got = paged_prefill(q.to(cuda_device), kp, vp, table.to(cuda_device), cu.to(cuda_device),
                        sk.to(cuda_device), 130)
    torch.cuda.synchronize()
    assert_output_close(got, ref_f32, torch.bfloat16)
    assert _native.device_error() == 0


@pytest.mark.gpu
def test_queries_that_see_no_key_give_zeros(cuda_device, kernel):
    """seqlen_k below the chunk length puts the first query tokens at negative positions: they
    see no key and their output is exact zeros (acc / max(l, 1) with l = 0), whole query tiles
    of them included; a row with seqlen_k 0 is all zeros."""
    from model import _native
    from model.triton_decode import paged_prefill

    q, k, v, table, cu, sk = prefill_case(16, 8, 128, 16, [0, 0, 5], [200, 70, 10], seed=12)
    sk = torch.tensor([50, 0, 12], dtype=torch.int32)
    ref_f32, _ = oracle.paged_prefill(q, k, v, table, cu, sk)
    got = paged_prefill(*[t.to(cuda_device) for t in (q, k, v, table, cu, sk)], 200)
    torch.cuda.synchronize()
    assert_output_close(got, ref_f32, torch.bfloat16)
    assert torch.count_nonzero(got[:150].float()) == 0  # row 0's tokens 0..149
    assert torch.count_nonzero(got[200:270].float()) == 0  # row 1
    assert torch.count_nonzero(got[150:200].float()) > 0
    assert _native.device_error() == 0


@pytest.mark.gpu
def test_a_larger_max_seqlen_q_bound_changes_nothing(cuda_device, kernel):
    """Engines pass a bucketed bound; the extra query tiles of the grid have no tokens."""
    from model import _native
    from model.triton_decode import paged_prefill

    q, k, v, table, cu, sk = prefill_case(16, 8, 128, 16, [40, 0, 500], [3, 70, 33], seed=9)
    dev = [t.to(cuda_device) for t in (q, k, v, table, cu, sk)]
    tight = paged_prefill(*dev, 70)
    loose = paged_prefill(*dev, 1000)
    torch.cuda.synchronize()
    assert torch.equal(tight, loose)
    ref_f32, _ = oracle.paged_prefill(q, k, v, table, cu, sk)
    assert_output_close(loose, ref_f32, torch.bfloat16)
    assert _native.device_error() == 0


@pytest.mark.gpu
def test_one_token_chunks_agree_with_the_decode_kernel(cuda_device, kernel):
    from model.triton_decode import paged_decode, paged_prefill

    q, k, v, table, cu, sk = prefill_case(16, 8, 128, 16, [31, 600, 2047, 0], [1, 1, 1, 1], seed=6)
    dev = [t.to(cuda_device) for t in (q, k, v, table, cu, sk)]
    pre = paged_prefill(*dev, 1)
    dec = paged_decode(dev[0], dev[1], dev[2], dev[3], dev[5])
    torch.cuda.synchronize()
    ref_f32, _ = oracle.paged_prefill(q, k, v, table, cu, sk)
    assert_output_close(pre, ref_f32, torch.bfloat16)
    assert_output_close(dec, ref_f32, torch.bfloat16)
    assert (pre.float() - dec.float()).abs().max().item() <= 2 * 2.0 ** -8 * max(1.0, ref_f32.abs().max().item())


@pytest.mark.gpu
def test_long_chunk_over_a_long_context(cuda_device, kernel):
    """A 1,000-token chunk after 3,000 cached tokens: many query tiles and key tiles per CTA."""
    from model import _native
    from model.triton_decode import paged_prefill

    q, k, v, table, cu, sk = prefill_case(16, 8, 128, 16, [3000, 0], [1000, 777], seed=7)
    ref_f32, _ = oracle.paged_prefill(q, k, v, table, cu, sk)
    got = paged_prefill(*[t.to(cuda_device) for t in (q, k, v, table, cu, sk)], 1000)
    torch.cuda.synchronize()
    assert_output_close(got, ref_f32, torch.bfloat16)
    assert _native.device_error() == 0
    assert math.isfinite(got.float().abs().max().item())


@pytest.mark.gpu
def test_chunked_prefill_through_the_engine_pool(cuda_device, kernel):
    """The engine's flow: a request's prompt K/V go into the pool with
    ``PagedPool.write_prefill`` chunk by chunk, and each chunk's queries attend over the pool
    with ``paged_prefill`` (earlier chunks included)."""
    from model import _native
    from model.paged import PagedPool
    from model.triton_decode import paged_prefill

    gen = torch.Generator().manual_seed(8)
    H, Hkv, D, bs = 16, 8, 128, 16
    pool = PagedPool(1, 64, bs, Hkv, D, dtype=torch.bfloat16, device=cuda_device, n_head=H)
    tables = [list(range(0, 64, 2)), list(range(1, 31, 2))]  # 32 and 15 interleaved, disjoint blocks
    table = torch.zeros(2, 32, dtype=torch.int32)
    for row, t in enumerate(tables):
        table[row, :len(t)] = torch.tensor(t, dtype=torch.int32)
    done = [0, 0]
    for chunks in ([300, 150], [200, 90]):
        qs = []
        for row, n in enumerate(chunks):
            k = torch.randn(n, Hkv, D, generator=gen).to(torch.bfloat16).to(cuda_device)
            v = torch.randn(n, Hkv, D, generator=gen).to(torch.bfloat16).to(cuda_device)
            pool.write_prefill(0, tables[row], done[row], k, v)
            qs.append(torch.randn(n, H, D, generator=gen).to(torch.bfloat16))
        for row, n in enumerate(chunks):
            done[row] += n
        q = torch.cat(qs)
        cu = torch.tensor([0, chunks[0], chunks[0] + chunks[1]], dtype=torch.int32)
        sk = torch.tensor(done, dtype=torch.int32)
        kp, vp = pool.keys[0], pool.values[0]
        got = paged_prefill(q.to(cuda_device), kp, vp, table.to(cuda_device), cu.to(cuda_device),
                            sk.to(cuda_device), max(chunks))
        torch.cuda.synchronize()
        ref_f32, _ = oracle.paged_prefill(q, kp.cpu(), vp.cpu(), table, cu, sk)
        assert_output_close(got, ref_f32, torch.bfloat16)
    assert _native.device_error() == 0
