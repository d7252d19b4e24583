"""The bounded-wait error path, exercised on the GPU without a hang or a fault.

Every wait in the decode and prefill kernels (a pipeline stage's mbarrier, a split item's
arrival counter) gives up after a time limit, records ``PD_DEVERR_WAIT_TIMEOUT`` in the device
error word, waits for its own copies still in flight and returns, so the launch ends and the
context stays usable. ``pd_set_wait_limit`` shortens that limit for later launches; below 1 µs
every wait gives up at once, so the first wait of every warp runs out on purpose while its
copies are still in flight. The test checks that such launches return with the bit set, and
that after the limit is restored the next launches (same workspace, same pools) equal the
oracle. The reference kernel has no device status (model/triton_decode.py:63-66).
"""

from __future__ import annotations

import math

import pytest
import torch

from helpers import assert_output_close, build_case
from oracle import oracle

pytestmark = pytest.mark.gpu

#: Launches made with the short limit; every one must record the timeout.
_TRIES = 2


@pytest.fixture
def short_waits():
    from model import _native

    _native.device_error(clear=True)
    _native.set_wait_limit(1)
    try:
        yield
    finally:
        _native.set_wait_limit(0)
        torch.cuda.synchronize()
        _native.device_error(clear=True)
    assert _native.get_wait_limit() == 1_000_000_000


def _timed_out(run) -> bool:
    from model import _native

    for _ in range(_TRIES):
        run()
        bits = _native.device_error(clear=True)  # synchronises: the launch has returned
        if bits != _native.DEVERR_WAIT_TIMEOUT:
            return False
    return True


def test_decode_wait_runs_out_and_the_next_launch_is_correct(cuda_device, short_waits):
    from model import _native

    q, k, v, table, seqlen = build_case(8, 16, 8, 128, 16, [4096, 3000, 1, 2048, 0, 777, 5000, 4096],
                                        dtype=torch.bfloat16, seed=41)
    ref_f32, _ = oracle.paged_decode(q, k, v, table, seqlen)
    qd, kd, vd, td, sd = (t.to(cuda_device) for t in (q, k, v, table, seqlen))
    scale = _native.log2e_scale(1.0 / math.sqrt(128))
    ws = torch.empty(_native.workspace_bytes(8, 16, 8, 128, torch.bfloat16), dtype=torch.uint8,
                     device=cuda_device)
    out = torch.empty_like(qd)
    assert _timed_out(lambda: _native.decode(qd, kd, vd, td, sd, out, scale, ws))
    _native.set_wait_limit(0)
    for _ in range(2):  # the workspace the timed-out launches used, as they left it
        out = torch.empty_like(qd)
        _native.decode(qd, kd, vd, td, sd, out, scale, ws)
        assert _native.device_error(clear=True) == 0
        assert_output_close(out, ref_f32, torch.bfloat16)


@pytest.mark.parametrize("kernel", [0, 1], ids=["tcgen05", "mma_sync"])
def test_prefill_wait_runs_out_and_the_next_launch_is_correct(cuda_device, short_waits, kernel):
    from model import _native
    from model.triton_decode import paged_prefill

    before = _native.get_prefill_mode()
    _native.set_prefill_mode(kernel)
    try:
        _prefill_case(cuda_device, paged_prefill)
    finally:
        _native.set_prefill_mode(before)


def _prefill_case(cuda_device, paged_prefill):
    from model import _native

    from test_prefill import prefill_case

    chunk = [256, 129, 200, 64]
    q, k, v, table, cu, seqlen_k = prefill_case(16, 8, 128, 16, [1500, 700, 2048, 64], chunk, seed=42)
    ref, _ = oracle.paged_prefill(q, k, v, table, cu, seqlen_k)
    qd, kd, vd, td, cud, skd = (t.to(cuda_device) for t in (q, k, v, table, cu, seqlen_k))
    assert _timed_out(lambda: paged_prefill(qd, kd, vd, td, cud, skd, max(chunk)))
    _native.set_wait_limit(0)
    out = paged_prefill(qd, kd, vd, td, cud, skd, max(chunk))
    assert _native.device_error(clear=True) == 0
    assert_output_close(out, ref, torch.bfloat16)
