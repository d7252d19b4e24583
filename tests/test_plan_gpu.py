"""Launch plan and decode container on a B200 (reference tests/unit/test_triton_decode.py:295-567
and tests/unit/test_paged_kv.py:351-404): the plan launches exactly what ``paged_decode``
launches, tracks in-place seqlen updates, refuses foreign layouts; error types and messages."""

from __future__ import annotations

import pytest
import torch

from helpers import build_case
from oracle import oracle

pytestmark = pytest.mark.gpu


def _cuda_case(*args, dtype=torch.float32, seed=0, **kw):
    q, k, v, table, seqlen = build_case(*args, dtype=dtype, seed=seed, **kw)
    return q.cuda(), k.cuda(), v.cuda(), table.cuda(), seqlen.cuda()


def test_plan_matches_paged_decode_for_every_layer(cuda_device):
    from model.triton_decode import paged_decode, paged_decode_plan

    q, k, v, table, seqlen = _cuda_case(3, 8, 4, 64, 16, [17, 15, 32], seed=43)
    gen = torch.Generator(device="cuda").manual_seed(44)
    ks = [torch.randn(k.shape, generator=gen, device="cuda") for _ in range(4)]
    vs = [torch.randn(v.shape, generator=gen, device="cuda") for _ in range(4)]
    plan = paged_decode_plan(q, ks, vs, table, seqlen)
    for layer in range(4):
        assert torch.equal(plan.run(layer, q), paged_decode(q, ks[layer], vs[layer], table, seqlen))


def test_plan_error_surface(cuda_device):
    from model.triton_decode import paged_decode_plan

    q, k, v, table, seqlen = _cuda_case(2, 4, 2, 64, 16, [17, 15], seed=59)
    with pytest.raises(ValueError, match="int32 seqlen"):
        paged_decode_plan(q, [k], [v], table, seqlen.to(torch.int64))
    with pytest.raises(ValueError, match="column-contiguous block table"):
        paged_decode_plan(q, [k], [v], table[:, ::2], seqlen)
    with pytest.raises(ValueError, match="contiguous 1-D seqlen"):
        paged_decode_plan(q, [k], [v], table, seqlen.repeat(2)[::2])
    plan = paged_decode_plan(q, [k, k], [v, v], table, seqlen)
    with pytest.raises(ValueError, match="does not match the validated layout"):
        plan.run(0, q.transpose(1, 2).contiguous().transpose(1, 2))
    with pytest.raises(ValueError, match="does not match the validated layout"):
        plan.run(0, q[:, :2, :].contiguous())
    with pytest.raises(ValueError, match="does not match the validated layout"):
        plan.run(0, q.double())
    with pytest.raises(IndexError, match="outside the plan"):
        plan.run(2, q)
    with pytest.raises(ValueError, match="head_dim"):
        paged_decode_plan(q, [k, k[..., :-1].contiguous()], [v, v[..., :-1].contiguous()], table, seqlen)


def test_paged_decode_error_surface(cuda_device):
    from model.triton_decode import paged_decode

    q, k, v, table, seqlen = _cuda_case(2, 4, 2, 64, 16, [17, 15], seed=29)
    with pytest.raises(ValueError, match="int32"):
        paged_decode(q, k, v, table.long(), seqlen)
    with pytest.raises(RuntimeError, match="CUDA tensors"):
        paged_decode(q, k, v, table.cpu(), seqlen)
    with pytest.raises(ValueError, match="capacity"):
        paged_decode(q, k, v, table, torch.full((2,), table.shape[1] * 16 + 1, dtype=torch.int32, device="cuda"))
    with pytest.raises(ValueError, match="head_dim"):
        paged_decode(q, k[..., :-1].contiguous(), v[..., :-1].contiguous(), table, seqlen)


def test_no_input_mutation_int64_seqlen_and_noncontiguous_query(cuda_device):
    from model.triton_decode import paged_decode

    q, k, v, table, seqlen = _cuda_case(3, 8, 4, 64, 16, [17, 15, 1], seed=17)
    snaps = [t.clone() for t in (q, k, v, table, seqlen)]
    qn = q.transpose(1, 2).contiguous().transpose(1, 2)
    got = paged_decode(qn, k, v, table, seqlen.to(torch.int64))
    for t, s in zip((q, k, v, table, seqlen), snaps):
        assert torch.equal(t, s)
    ref, _ = oracle.paged_decode(q, k, v, table, seqlen)
    torch.testing.assert_close(got.cpu(), ref, rtol=0, atol=1e-4)


def test_zero_length_rows_and_stale_bytes(cuda_device):
    from model.triton_decode import paged_decode

    q, k, v, table, seqlen = _cuda_case(3, 4, 2, 64, 16, [0, 16, 17], seed=23)
    out = paged_decode(q, k, v, table, seqlen)
    assert torch.isfinite(out).all() and not out[0].any()
    # stale (and NaN) bytes past seqlen in a reused block never reach the output
    k2 = torch.full((1, 16, 2, 64), float("nan"), device="cuda")
    v2 = torch.full_like(k2, float("nan"))
    g = torch.Generator(device="cuda").manual_seed(107)
    k2[:, :5] = torch.randn(5, 2, 64, generator=g, device="cuda")
    v2[:, :5] = torch.randn(5, 2, 64, generator=g, device="cuda")
    q2 = torch.randn(2, 4, 64, generator=g, device="cuda")
    t2 = torch.zeros(2, 1, dtype=torch.int32, device="cuda")
    s2 = torch.tensor([5, 3], dtype=torch.int32, device="cuda")
    got = paged_decode(q2, k2, v2, t2, s2)
    ref, _ = oracle.paged_decode(q2, k2, v2, t2, s2)
    assert torch.isfinite(got).all()
    torch.testing.assert_close(got.cpu(), ref, rtol=0, atol=1e-4)


def test_revalidation_after_in_place_seqlen_change_and_inference_tensors(cuda_device):
    from model.triton_decode import paged_decode

    q, k, v, table, seqlen = _cuda_case(2, 4, 2, 64, 16, [17, 15], seed=43)
    paged_decode(q, k, v, table, seqlen)
    seqlen[0] = 1
    got = paged_decode(q, k, v, table, seqlen)
    ref, _ = oracle.paged_decode(q, k, v, table, seqlen)
    torch.testing.assert_close(got.cpu(), ref, rtol=0, atol=1e-4)
    with torch.inference_mode():
        s_inf = torch.tensor([17, 15], dtype=torch.int32, device="cuda")
        got = paged_decode(q, k, v, table, s_inf)
    ref, _ = oracle.paged_decode(q, k, v, table, s_inf)
    torch.testing.assert_close(got.cpu(), ref, rtol=0, atol=1e-4)


def test_container_plan_tracks_in_place_seqlen_updates(cuda_device):
    from model.paged import PagedKV, PagedPool
    from model.triton_decode import paged_decode

    torch.manual_seed(0)
    pool = PagedPool(1, 4, 16, 2, 32, dtype=torch.float32, device="cuda", n_head=4)
    kv = PagedKV(pool, [[0, 1, 2, 3]], [10], rope_len=64, n_head=4)
    q = torch.randn(1, 4, 1, 32, device="cuda")
    outs = []
    for step in range(3):
        kv.build_mask(next_token=True)
        kv.write(0, torch.randn(1, 2, 1, 32, device="cuda"), torch.randn(1, 2, 1, 32, device="cuda"))
        outs.append(kv.attend(0, q))
        expected = paged_decode(q[:, :, 0, :].contiguous(), pool.keys[0], pool.values[0],
                                kv._block_table_tensor, kv._seqlen).unsqueeze(2)
        assert torch.equal(outs[-1], expected), f"step {step}"
        kv.advance()
    assert not torch.equal(outs[0], outs[-1])


def test_container_protocol_and_step_order(cuda_device):
    from model.paged import PagedKV, PagedPool

    pool = PagedPool(2, 12, 16, 2, 64, dtype=torch.bfloat16, device="cuda", n_head=4)
    kv = PagedKV(pool, [[0, 1, 2, 3], [4, 5, 6, 7], [8, 9, 10, 11]], [5, 9, 13], rope_len=100, n_head=4)
    assert kv.decode_container and kv.block_table_decode and kv._seqlen.dtype == torch.int32
    q = torch.randn(3, 4, 1, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="before build_mask"):
        kv.attend(0, q)
    kv.build_mask(next_token=True)
    assert torch.equal(kv._seqlen, (kv.pos + 1).to(torch.int32))
    with pytest.raises(RuntimeError, match="before write"):
        kv.attend(0, q)
    with pytest.raises(ValueError):
        kv.write(0, torch.zeros(4, 2, 1, 64, device="cuda"), torch.zeros(4, 2, 1, 64, device="cuda"))
    assert kv.build_mask(next_token=False) is None
    assert torch.equal(kv._seqlen, kv.pos.to(torch.int32))
    for name in ("lpad", "mask", "bias", "get", "set_buffers"):
        assert not hasattr(kv, name)
    with pytest.raises((IndexError, ValueError)):
        PagedKV(PagedPool(1, 2, 16, 2, 64, device="cuda"), [[0]], [21], rope_len=16)


def test_engine_style_decode_steps_match_the_oracle(cuda_device):
    """Several steps of the engine's protocol (write then attend per layer) against the oracle
    applied to the same pools, with per-row lengths that cross block boundaries."""
    from model.paged import PagedKV, PagedPool

    gen = torch.Generator(device="cuda").manual_seed(3)
    pool = PagedPool(3, 40, 16, 8, 128, dtype=torch.bfloat16, device="cuda", n_head=16)
    for t in pool.keys + pool.values:
        t.copy_(torch.randn(t.shape, generator=gen, device="cuda"))
    tables = [list(range(0, 10)), list(range(10, 20)), list(range(20, 40))]
    kv = PagedKV(pool, tables, [14, 47, 300], rope_len=400, n_head=16)
    for _ in range(4):
        kv.build_mask(next_token=True)
        for layer in range(3):
            k = torch.randn(3, 8, 1, 128, generator=gen, device="cuda").to(torch.bfloat16)
            v = torch.randn(3, 8, 1, 128, generator=gen, device="cuda").to(torch.bfloat16)
            q = torch.randn(3, 16, 1, 128, generator=gen, device="cuda").to(torch.bfloat16)
            kv.write(layer, k, v)
            got = kv.attend(layer, q)[:, :, 0, :]
            ref, _ = oracle.paged_decode(q[:, :, 0, :], pool.keys[layer], pool.values[layer],
                                         kv._block_table_tensor, kv._seqlen)
            assert (got.float().cpu() - ref).abs().max() < 4e-3
        kv.advance()
    assert kv.pos.tolist() == [18, 51, 304]
