"""``pd_decode_noalloc``: the decode entry point for callers that cannot allocate device memory.

Some hosts bind this library's C ABI without owning a device allocator (a Go, Java or Node
process handed raw pointers) or with every byte already reserved by another allocator; they
cannot supply the workspace ``pd_decode`` needs. ``pd_decode_noalloc`` takes none and uses a
fixed scratch array built into the library instead. Here it is called through the C ABI
twice in a row -- the second call reuses whatever the first left in the shared array -- and
each result must equal ``pd_decode``'s on the same inputs bit for bit: both run the same
deterministic kernel with the same work split, so any difference would be a scratch-layout
bug that a tolerance could hide. The array starts out zero-filled; that start state is
reproduced for ``pd_decode`` with a zeroed workspace on a split-heavy shape. Shapes that need
more scratch than the array holds must be refused with an error that names the limit.

Collected last on purpose (``zz``) so that a failure here, in a run that stops at the first
failure, comes after every other test has run.
"""

from __future__ import annotations

import math

import pytest
import torch

from helpers import build_case

pytestmark = pytest.mark.gpu


def _decode_both(q, k, v, table, seqlen, *, zero_workspace=False):
    from model import _native

    scale = _native.log2e_scale(1.0 / math.sqrt(q.shape[2]))
    ref = torch.empty_like(q)
    need = _native.workspace_bytes(*q.shape[:2], k.shape[2], q.shape[2], q.dtype)
    alloc = torch.zeros if zero_workspace else torch.empty
    ws = alloc(need, dtype=torch.uint8, device=q.device)
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
        assert torch.equal(got, ref)
        assert not got[seqlen == 0].any()
    assert _native.device_error() == 0


def test_zero_filled_workspace_decodes_a_split_heavy_shape(cuda_device):
    """A zero-filled workspace -- the state of a fresh allocation and of the library's scratch
    array before its first call -- must decode correctly when rows are split into many pieces
    (4 long rows over ~1,200 warps), for pd_decode and for pd_decode_noalloc."""
    from model import _native

    q, k, v, table, seqlen = build_case(4, 16, 8, 128, 16, [8192, 6000, 7777, 4096], dtype=torch.bfloat16,
                                        seed=91)
    q, k, v, table, seqlen = (t.to(cuda_device) for t in (q, k, v, table, seqlen))
    first, ref = _decode_both(q, k, v, table, seqlen, zero_workspace=True)
    again, ref2 = _decode_both(q, k, v, table, seqlen, zero_workspace=True)
    assert torch.equal(ref, ref2)
    assert torch.equal(first, ref) and torch.equal(again, ref)
    assert _native.device_error() == 0


def test_noalloc_refuses_shapes_beyond_its_scratch(cuda_device):
    from model import _native

    B, H, Hkv, D = 1, 64, 8, 256  # 8 q heads per kv head at head_dim 256: > 8 MiB of scratch
    need = _native.workspace_bytes(B, H, Hkv, D, torch.bfloat16)
    assert need > 8 << 20
    q, k, v, table, seqlen = build_case(B, H, Hkv, D, 16, [40], dtype=torch.bfloat16, seed=3)
    q, k, v, table, seqlen = (t.to(cuda_device) for t in (q, k, v, table, seqlen))
    out = torch.empty_like(q)
    with pytest.raises(ValueError, match=rf"needs {need} bytes of scratch .* holds {8 << 20}"):
        _native.decode_noalloc(q, k, v, table, seqlen, out, 1.0)
