"""The plan's step cache of the work split: bitwise the same outputs, whatever the cache holds.

A plan records each launch's work split (each warp's range, starting cursor and, with a static
block table, its first table windows) in its workspace, keyed by a hash of the clamped lengths
and the plan's shape. Later launches with the same lengths -- the other layers of a decode step
-- reuse it instead of recomputing it. The cached split is the computed one, so every output must
equal ``paged_decode`` (which computes its split every time) bit for bit: on every benchmark
config, for the first layer (which writes the records) and the later ones (which read them),
with overlapped launches, after the lengths change in place (the key must miss), and when the
workspace starts zero-filled. Reference: the step updates seqlen once and every layer reads it
(model/paged.py:454-472).
"""

from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu


def _fresh(wl, layer, seqlen):
    from model.triton_decode import paged_decode

    return paged_decode(wl.q[layer], wl.k_pools[layer], wl.v_pools[layer], wl.block_table, seqlen)


@pytest.mark.parametrize("static_table", [False, True], ids=["table-reread", "static-table"])
@pytest.mark.parametrize("name,n_layer", [("config1", 4), ("config2", 3), ("config3", 3), ("qwen35", 3)])
def test_cached_split_gives_the_computed_outputs(cuda_device, name, n_layer, static_table):
    import workloads
    from model import _native
    from model.triton_decode import paged_decode_plan

    wl = getattr(workloads, name)(cuda_device, n_layer=n_layer)
    plan = paged_decode_plan(wl.q[0], wl.k_pools, wl.v_pools, wl.block_table, wl.seqlen)
    plan._native_plan.set_static_table(static_table)
    for overlap in (False, True):
        outs = [plan.run(layer, wl.q[layer], overlap=overlap and layer > 0) for layer in range(n_layer)]
        for layer in range(n_layer):
            assert torch.equal(outs[layer], _fresh(wl, layer, wl.seqlen)), (overlap, layer)
    # the lengths change in place (the next step): the recorded split no longer applies
    wl.seqlen.sub_(torch.arange(wl.seqlen.numel(), device=cuda_device, dtype=torch.int32) % 3)
    wl.seqlen.clamp_(min=0)
    outs = [plan.run(layer, wl.q[layer]) for layer in range(n_layer)]
    for layer in range(n_layer):
        assert torch.equal(outs[layer], _fresh(wl, layer, wl.seqlen)), ("after update", layer)
    assert _native.device_error() == 0


def test_zero_filled_plan_workspace(cuda_device):
    """A record of zeros never matches a key (keys are odd), so a zeroed workspace computes."""
    import workloads
    from model.triton_decode import paged_decode_plan

    wl = workloads.config2(cuda_device, n_layer=2)
    plan = paged_decode_plan(wl.q[0], wl.k_pools, wl.v_pools, wl.block_table, wl.seqlen)
    plan._workspace.zero_()
    for layer in range(2):
        assert torch.equal(plan.run(layer, wl.q[layer]), _fresh(wl, layer, wl.seqlen))
