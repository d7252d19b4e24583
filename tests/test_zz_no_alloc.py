"""``pd_decode_noalloc``: the decode entry point for callers that cannot allocate device memory.

Some hosts bind this library's C ABI without owning a device allocator (a Go, Java or Node
process handed raw pointers) or with every byte already reserved by another allocator; they
cannot supply the workspace ``pd_decode`` needs. ``pd_decode_noalloc`` takes none and uses a
fixed scratch array built into the library instead. Here it is called through the C ABI
twice in a row -- the second call reuses whatever the first left in the shared array -- and
each result must agree with ``pd_decode`` on the same inputs within the suite's tolerance.
Shapes that need more scratch than the array holds must be refused with a clear error.

Collected last on purpose (``zz``) so that a failure here, in a run that stops at the first
failure, comes after every other test has run.
"""

from __future__ import annotations

import math

import pytest
import torch

from helpers import assert_output_close, build_case

pytestmark = pytest.mark.gpu


def _decode_both(q, k, v, table, seqlen):
    from model import _native

    scale = _native.log2e_scale(1.0 / math.sqrt(q.shape[2]))
    ref = torch.empty_like(q)
    ws = torch.empty(_native.workspace_bytes(*q.shape[:2], k.shape[2], q.shape[2], q.dtype),
                     dtype=torch.uint8, device=q.device)
    _native.decode(q, k, v, table, seqlen, ref, scale, ws)
    got = torch.empty_like(q)
    _native.decode_noalloc(q, k, v, table, seqlen, got, scale)
    torch.cuda.synchronize()
    return got, ref


def test_noalloc_decode_matches_pd_decode_on_two_calls_in_a_row(cuda_device):
    from model import _native

    # Long rows so items are split across workers and the scratch (partials + counters) is used.
    cases = [
        (4, 16, 8, 128, 16, [3000, 17, 1, 2048], 71),
        (32, 16, 8, 128, 16, [2100] * 31 + [0], 72),
    ]
    for B, H, Hkv, D, bs, lengths, seed in cases:
        q, k, v, table, seqlen = build_case(B, H, Hkv, D, bs, lengths, dtype=torch.bfloat16, seed=seed)
        q, k, v, table, seqlen = (t.to(cuda_device) for t in (q, k, v, table, seqlen))
        got, ref = _decode_both(q, k, v, table, seqlen)
        assert_output_close(got, ref.float(), torch.bfloat16)
        assert not got[seqlen == 0].any()
    assert _native.device_error() == 0


def test_noalloc_refuses_shapes_beyond_its_scratch(cuda_device):
    from model import _native

    B, H, Hkv, D = 1, 64, 8, 256  # 8 q heads per kv head at head_dim 256: > 8 MiB of scratch
    assert _native.workspace_bytes(B, H, Hkv, D, torch.bfloat16) > 8 << 20
    q, k, v, table, seqlen = build_case(B, H, Hkv, D, 16, [40], dtype=torch.bfloat16, seed=3)
    q, k, v, table, seqlen = (t.to(cuda_device) for t in (q, k, v, table, seqlen))
    out = torch.empty_like(q)
    with pytest.raises(ValueError, match="scratch"):
        _native.decode_noalloc(q, k, v, table, seqlen, out, 1.0)
