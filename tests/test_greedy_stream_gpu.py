"""Greedy decode of random-init models through ``PagedKV`` at the two attention shapes the
engines drive: config 2's 28-layer Qwen3-0.6B (16 q / 8 kv heads, head_dim 128, full RoPE), and
Qwen3.5-0.8B's 6 full-attention layers (8 q / 2 kv heads, head_dim 256, RoPE on the first 64
dims; its linear-attention layers are outside this path and left out).

The models have no checkpoint: hidden 1024, SwiGLU 3072, vocab 151936, RMSNorm with per-head
q/k norms, RoPE theta 1e6, bf16, tied embeddings. Each runs B=32 requests, each with a
2048-token prompt in paged KV (block size 16, blocks assigned by a seeded permutation), for
64 greedy steps. The arms share every tensor op except attention:

* the product arm appends each step's K/V and attends through ``PagedKV.write`` /
  ``PagedKV.attend``: the fused sm_100a append + decode launch, overlapped launches included.
  It hands K over *before* its rotary embedding with ``rope=(cos, sin)``, so the append
  rotates it on the way into the pool (the reference arms rotate K in torch, in the
  reference's arithmetic);
* the reference arm keeps a dense per-request cache and attends in fp32 over the gathered
  keys (softmax(q k^T / sqrt(d)) V, rounded to bf16), which is the reference's torch
  paged-gather attention.

A third arm, the same gather attention in float64, is the noise floor: it is as correct
as the fp32 reference, and it still differs from it by a bf16 ulp in some attention outputs.
Each arm computes its new K/V from its own hidden state, so such differences compound over
the layers and 64 steps. Random weights give flat logits (top-2 gaps of a few thousandths
are common), so near-ties flip in the floor arm too.

The prompt K/V come from one shared bf16 prefill and are written into every arm. Decoding is
teacher-forced: all arms take the fp32 reference's token as the next input, so all 64 x 32
decisions are compared. The product arm must stay within the floor: its largest logit
deviation from the fp32 reference at most FLOOR_FACTOR times the float64 arm's, its
mismatched decisions no more than FLOOR_FACTOR times the float64 arm's (plus a small count
for the statistics of rare events), and each of its mismatches at a top-2 gap that the
floor's own deviation could flip.
"""

from __future__ import annotations

import math
from typing import NamedTuple

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

VOCAB, HIDDEN, INTER = 151936, 1024, 3072
THETA, EPS = 1e6, 1e-6
B, PROMPT, STEPS, BS = 32, 2048, 64, 16

FLOOR_FACTOR = 2.0
MISMATCH_SLACK = 8


class Shape(NamedTuple):
    n_layer: int
    h: int       # q heads
    hkv: int     # kv heads
    d: int       # head_dim
    rotary: int  # leading dims that RoPE rotates


SHAPES = [
    pytest.param(Shape(28, 16, 8, 128, 128), id="qwen3-28-layers"),
    pytest.param(Shape(6, 8, 2, 256, 64), id="qwen35-6-full-attention-layers"),
]


def _rms(x, w):
    xf = x.float()
    return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + EPS)).to(x.dtype) * w


def _rope_tables(n_pos, rot, device):
    inv = 1.0 / (THETA ** (torch.arange(0, rot, 2, device=device, dtype=torch.float32) / rot))
    freqs = torch.outer(torch.arange(n_pos, device=device, dtype=torch.float32), inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


def _rope(x, cos, sin):
    """x (..., n, D) with cos/sin (n, R): GPT-NeoX rotation of the first R dims, the rest kept."""
    r = cos.shape[-1]
    xr, half = x[..., :r], r // 2
    rotated = torch.cat([-xr[..., half:], xr[..., :half]], dim=-1)
    return torch.cat([xr * cos + rotated * sin, x[..., r:]], dim=-1)


class _Model:
    def __init__(self, device, shape: Shape, seed=0):
        self.s = S = shape
        H, HKV, D = S.h, S.hkv, S.d
        gen = torch.Generator(device=device).manual_seed(seed)

        def w(*shape):
            return (torch.randn(*shape, generator=gen, device=device) * 0.02).to(torch.bfloat16)

        ones = lambda n: torch.ones(n, device=device, dtype=torch.bfloat16)  # noqa: E731
        self.embed = w(VOCAB, HIDDEN)
        self.embed_f32 = self.embed.float()
        self.layers = [
            dict(ln1=ones(HIDDEN), wq=w(H * D, HIDDEN), wk=w(HKV * D, HIDDEN), wv=w(HKV * D, HIDDEN),
                 qn=ones(D), kn=ones(D), wo=w(HIDDEN, H * D), ln2=ones(HIDDEN), wg=w(INTER, HIDDEN),
                 wu=w(INTER, HIDDEN), wd=w(HIDDEN, INTER))
            for _ in range(S.n_layer)
        ]
        self.norm = ones(HIDDEN)
        self.cos, self.sin = _rope_tables(PROMPT + STEPS, S.rotary, device)

    def qkv(self, L, x, pos, rotate_k=True):
        """x (B, n, HIDDEN) at positions pos (n,) -> q (B, H, n, D), k / v (B, HKV, n, D);
        k is returned before its rotary embedding when ``rotate_k`` is False."""
        H, HKV, D = self.s.h, self.s.hkv, self.s.d
        h = _rms(x, L["ln1"])
        n = x.shape[1]
        q = _rms((h @ L["wq"].T).view(B, n, H, D), L["qn"]).transpose(1, 2)
        k = _rms((h @ L["wk"].T).view(B, n, HKV, D), L["kn"]).transpose(1, 2)
        v = (h @ L["wv"].T).view(B, n, HKV, D).transpose(1, 2)
        cos, sin = self.cos[pos], self.sin[pos]
        return _rope(q, cos, sin), (_rope(k, cos, sin) if rotate_k else k), v

    def rope_rows(self, p):
        """The (B, R/2) cos/sin rows of position p that a rotated ``PagedKV.write`` takes."""
        half = self.s.rotary // 2
        return (self.cos[p, :half].expand(B, half).contiguous(),
                self.sin[p, :half].expand(B, half).contiguous())

    def finish(self, L, x, attn):
        """attn (B, H, n, D): output projection, residual and the MLP."""
        n = x.shape[1]
        x = x + attn.transpose(1, 2).reshape(B, n, self.s.h * self.s.d) @ L["wo"].T
        h = _rms(x, L["ln2"])
        return x + (F.silu(h @ L["wg"].T) * (h @ L["wu"].T)) @ L["wd"].T

    def logits(self, x):
        """Last position's fp32 logits (B, VOCAB)."""
        return _rms(x[:, -1], self.norm).float() @ self.embed_f32.T


def _ref_attend(q, kc, vc, n_keys, dtype=torch.float32):
    """Attention of q (B, H, 1, D) over the first n_keys of the dense cache, computed in
    `dtype` and rounded to bf16."""
    H, HKV, D = q.shape[1], kc.shape[1], q.shape[-1]
    k = kc[:, :, :n_keys].to(dtype)
    v = vc[:, :, :n_keys].to(dtype)
    qg = q.to(dtype).view(B, HKV, H // HKV, D)
    p = torch.softmax(torch.einsum("bkgd,bktd->bkgt", qg, k) / math.sqrt(D), dim=-1)
    return torch.einsum("bkgt,bktd->bkgd", p, v).reshape(B, H, 1, D).to(torch.bfloat16)


def run_streams(device, shape: Shape):
    """All arms over the 64 steps; returns per-step tensors (steps, B) of the product and
    float64 arms' tokens, the fp32 reference's tokens and top-2 gaps, and each arm's largest
    logit deviation from the fp32 reference."""
    from model.paged import PagedKV, PagedPool

    H, HKV, D, N_LAYER = shape.h, shape.hkv, shape.d, shape.n_layer
    model = _Model(device, shape)
    gen = torch.Generator(device=device).manual_seed(1)
    prompt = torch.randint(0, VOCAB, (B, PROMPT), generator=gen, device=device)

    pages = -(-(PROMPT + STEPS) // BS)
    n_blocks = B * pages + 7
    perm = torch.randperm(n_blocks, generator=torch.Generator().manual_seed(2)).tolist()
    tables = [perm[r * pages:(r + 1) * pages] for r in range(B)]
    pool = PagedPool(N_LAYER, n_blocks, BS, HKV, D, dtype=torch.bfloat16, device=device, n_head=H)
    kc = [torch.zeros(B, HKV, PROMPT + STEPS, D, dtype=torch.bfloat16, device=device) for _ in range(N_LAYER)]
    vc = [torch.zeros_like(t) for t in kc]
    kx = [torch.zeros_like(t) for t in kc]  # the float64 arm's cache
    vx = [torch.zeros_like(t) for t in kc]

    # shared prefill (bf16 SDPA); its K/V go into every arm
    with torch.no_grad():
        x = model.embed[prompt]
        pos = torch.arange(PROMPT, device=device)
        for li, L in enumerate(model.layers):
            q, k, v = model.qkv(L, x, pos)
            for cache, val in ((kc, k), (vc, v), (kx, k), (vx, v)):
                cache[li][:, :, :PROMPT] = val
            for r in range(B):
                pool.write_prefill(li, tables[r], 0, k[r].transpose(0, 1).contiguous(),
                                   v[r].transpose(0, 1).contiguous())
            a = F.scaled_dot_product_attention(q, k.repeat_interleave(H // HKV, 1),
                                               v.repeat_interleave(H // HKV, 1), is_causal=True)
            x = model.finish(L, x, a)
        tok = model.logits(x).argmax(-1)

        kv = PagedKV(pool, tables, [PROMPT] * B, rope_len=PROMPT + STEPS, n_head=H)
        ours_tok, ref_tok, x_tok, gaps, deltas, x_deltas = [], [], [], [], [], []
        for step in range(STEPS):
            p = PROMPT + step
            pos = torch.tensor([p], device=device)
            kv.build_mask(next_token=True)
            xo = xr = xx = model.embed[tok].unsqueeze(1)
            for li, L in enumerate(model.layers):
                q, k, v = model.qkv(L, xo, pos, rotate_k=False)
                kv.write(li, k, v, rope=model.rope_rows(p))
                xo = model.finish(L, xo, kv.attend(li, q))
                q, k, v = model.qkv(L, xr, pos)
                kc[li][:, :, p:p + 1] = k
                vc[li][:, :, p:p + 1] = v
                xr = model.finish(L, xr, _ref_attend(q, kc[li], vc[li], p + 1))
                q, k, v = model.qkv(L, xx, pos)
                kx[li][:, :, p:p + 1] = k
                vx[li][:, :, p:p + 1] = v
                xx = model.finish(L, xx, _ref_attend(q, kx[li], vx[li], p + 1, torch.float64))
            kv.advance()
            if step == 0:  # layer 0 of step 0 sees the same hidden state in every arm
                rope_bitwise = all(
                    torch.equal(pool.keys[0][tables[r][p // BS], p % BS], kc[0][r, :, p]) for r in range(B))
            lo, lr, lx = model.logits(xo), model.logits(xr), model.logits(xx)
            top2 = lr.topk(2, dim=-1).values
            ours_tok.append(lo.argmax(-1))
            ref_tok.append(lr.argmax(-1))
            x_tok.append(lx.argmax(-1))
            gaps.append(top2[:, 0] - top2[:, 1])
            deltas.append((lo - lr).abs().amax(-1))
            x_deltas.append((lx - lr).abs().amax(-1))
            tok = ref_tok[-1]  # teacher forcing: every arm continues from the reference's token
    torch.cuda.synchronize()
    return dict(ours=torch.stack(ours_tok), ref=torch.stack(ref_tok), exact=torch.stack(x_tok),
                gap=torch.stack(gaps), delta=torch.stack(deltas), exact_delta=torch.stack(x_deltas),
                logit_std=lr.std().item(), rope_bitwise=rope_bitwise)


@pytest.mark.parametrize("shape", SHAPES)
def test_greedy_streams_agree_through_paged_kv(cuda_device, shape):
    from model import _native

    s = run_streams(cuda_device, shape)
    mismatch = s["ours"] != s["ref"]
    n_mis, n_floor = int(mismatch.sum()), int((s["exact"] != s["ref"]).sum())
    worst_gap = float(s["gap"][mismatch].max()) if n_mis else 0.0
    delta, floor = float(s["delta"].max()), float(s["exact_delta"].max())
    detail = (f"{n_mis} of {mismatch.numel()} decisions differ from the fp32 reference (float64 "
              f"arm: {n_floor}); worst top-2 gap at a mismatch {worst_gap:.4f}; max |logit delta| "
              f"{delta:.4f} (float64 arm: {floor:.4f}); logit std {s['logit_std']:.3f}")
    assert _native.device_error() == 0
    assert s["rope_bitwise"], "K rotated by the fused append differs from K rotated in torch"
    assert delta <= FLOOR_FACTOR * floor, detail
    assert n_mis <= FLOOR_FACTOR * n_floor + MISMATCH_SLACK, detail
    assert worst_gap < 2 * floor, detail
