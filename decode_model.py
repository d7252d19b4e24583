"""A random-init Qwen3-0.6B-shaped decoder that drives ``PagedKV``: benchmark and test input.

BASELINE config 2 times the whole decode step of the reference's serve engine on Qwen3-0.6B
(``MiniLLMConfig`` with 28 layers, hidden 1024, 16 q / 8 kv heads, head_dim 128, SwiGLU 3072,
vocab 151936, RMSNorm eps 1e-6 with per-head q/k norms, RoPE theta 1e6, tied embeddings;
model/minillm.py, model/layers.py of the reference). The model and its weights are outside the
rebuilt path and no checkpoint exists here, so this module restates the architecture in plain
torch with random weights (std 0.02, the reference's ``_init_weights``) to give the attention
path its real callers: per layer RMSNorm, one fused q/k/v projection, q/k RMSNorm, RoPE on q,
``PagedKV.write`` with K handed over before its rotary embedding (the fused append rotates
it), ``PagedKV.attend``, the output projection, RMSNorm, a fused gate/up projection, SiLU,
the down projection; then the final norm, the tied lm_head and a greedy argmax.

:meth:`PagedDecoder.step` only reads and writes fixed buffers, so a whole step can be captured
with :class:`serve.graph.DecodeStepGraph`; the next step's input token is this step's argmax on
the device. This is not part of the library (``bench.py`` and ``tests/`` import it).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F

VOCAB, HIDDEN, INTER = 151936, 1024, 3072
THETA, EPS = 1e6, 1e-6


def rope_tables(n_pos: int, rotary: int, device):
    """cos/sin (n_pos, rotary) in bf16, GPT-NeoX layout (the two halves repeat the freqs)."""
    inv = 1.0 / (THETA ** (torch.arange(0, rotary, 2, device=device, dtype=torch.float32) / rotary))
    freqs = torch.outer(torch.arange(n_pos, device=device, dtype=torch.float32), inv)
    emb = torch.cat([freqs, freqs], dim=-1)
    return emb.cos().to(torch.bfloat16), emb.sin().to(torch.bfloat16)


class PagedDecoder:
    """Random-init decoder of ``n_layer`` layers over a :class:`PagedKV` of matching heads."""

    def __init__(self, kv, *, n_layer: int, n_head: int, n_kv_head: int, head_dim: int, rotary: int,
                 max_pos: int, seed: int = 0, device="cuda"):
        self.kv = kv
        self.n_layer, self.h, self.hkv, self.d, self.rotary = n_layer, n_head, n_kv_head, head_dim, rotary
        gen = torch.Generator(device=device).manual_seed(seed)

        def w(*shape):
            return (torch.randn(*shape, generator=gen, device=device) * 0.02).to(torch.bfloat16)

        ones = lambda n: torch.ones(n, device=device, dtype=torch.bfloat16)  # noqa: E731
        qd, kd = n_head * head_dim, n_kv_head * head_dim
        self.embed = w(VOCAB, HIDDEN)
        self.layers = [dict(ln1=ones(HIDDEN), wqkv=w(qd + 2 * kd, HIDDEN), qn=ones(head_dim), kn=ones(head_dim),
                            wo=w(HIDDEN, qd), ln2=ones(HIDDEN), wgu=w(2 * INTER, HIDDEN), wd=w(HIDDEN, INTER))
                       for _ in range(n_layer)]
        self.norm = ones(HIDDEN)
        self.cos, self.sin = rope_tables(max_pos, rotary, device)
        B = kv.batch
        self.tok = torch.zeros(B, dtype=torch.long, device=device)   # input token of the step
        self.next = torch.zeros(B, dtype=torch.long, device=device)  # greedy output of the step
        self.prepare_q = torch.zeros(B, n_head, 1, head_dim, dtype=torch.bfloat16, device=device)

    @staticmethod
    def _rms(x, w):
        return F.rms_norm(x, (x.shape[-1],), w, EPS)

    def _rope_q(self, q, cos, sin):
        """q (B, H, 1, D); cos/sin (B, 1, 1, R): GPT-NeoX rotation of the first R dims."""
        r = self.rotary
        half = r // 2
        qr = q[..., :r]
        rotated = torch.cat([-qr[..., half:], qr[..., :half]], dim=-1)
        out = qr * cos + rotated * sin
        return out if r == q.shape[-1] else torch.cat([out, q[..., r:]], dim=-1)

    def step(self) -> None:
        """One greedy decode step of every row: reads :attr:`tok`, writes :attr:`next`. Call it
        between ``kv.build_mask(next_token=True)`` and ``kv.advance()``."""
        kv = self.kv
        B, H, HKV, D = kv.batch, self.h, self.hkv, self.d
        pos = kv.pos  # the position this step's token is written at
        cos, sin = self.cos[pos], self.sin[pos]  # (B, R)
        half = self.rotary // 2
        rope_rows = (cos[:, :half].contiguous(), sin[:, :half].contiguous())
        cos4, sin4 = cos.view(B, 1, 1, -1), sin.view(B, 1, 1, -1)
        x = self.embed[self.tok]  # (B, HIDDEN)
        for li, L in enumerate(self.layers):
            h = self._rms(x, L["ln1"])
            qkv = h @ L["wqkv"].T
            q = self._rms(qkv[:, :H * D].view(B, H, 1, D), L["qn"])
            k = self._rms(qkv[:, H * D:(H + HKV) * D].view(B, HKV, 1, D), L["kn"])
            v = qkv[:, (H + HKV) * D:].view(B, HKV, 1, D)
            kv.write(li, k, v, rope=rope_rows)
            a = kv.attend(li, self._rope_q(q, cos4, sin4))
            x = x + a.reshape(B, H * D) @ L["wo"].T
            h = self._rms(x, L["ln2"])
            gu = h @ L["wgu"].T
            x = x + (F.silu(gu[:, :INTER]) * gu[:, INTER:]) @ L["wd"].T
        logits = self._rms(x, self.norm) @ self.embed.T
        torch.argmax(logits, dim=-1, out=self.next)
        self.tok.copy_(self.next)
