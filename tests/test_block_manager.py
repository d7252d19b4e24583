"""``serve/block_manager.py`` against the reference allocator's recorded behaviour.

``tests/golden/block_manager.json`` holds a 200-call seeded reserve/free trace of the
reference's ``BlockManager`` (ids returned and the stats after every call), its
``blocks_for`` values, and the fragmented config-3 block tables the workload recipe produced
on the reference allocator. This allocator must reproduce all of them exactly; the remaining
tests restate the reference's unit tests (tests/unit/test_block_manager.py).
"""

from __future__ import annotations

import json
from pathlib import Path

import pytest

import workloads
from serve.block_manager import BlockManager, FragStats

GOLDEN = json.loads((Path(__file__).resolve().parent / "golden" / "block_manager.json").read_text())


def test_reproduces_the_reference_trace():
    bm = BlockManager(64, 16)
    for step in GOLDEN["trace"]:
        if step["op"] == "free":
            bm.free(step["ids"])
        else:
            assert bm.reserve(step["n"]) == step["ids"]
        assert bm.stats() == step["stats"]
    for prompt, budget, expected in GOLDEN["blocks_for"]:
        assert bm.blocks_for(prompt, budget) == expected


@pytest.mark.parametrize("case", GOLDEN["config3"], ids=lambda c: f"seed{c['seed']}")
def test_config3_fragmented_tables_match_the_reference_allocator(case):
    lengths = workloads.lognormal_lengths(64, case["seed"])
    assert lengths == case["lengths"]
    tables = workloads.fragmented_tables(lengths, case["n_blocks"], 16, case["seed"])
    assert tables == case["tables"]
    # fragmentation is real: some row's blocks are not one ascending run
    assert any(t != list(range(t[0], t[0] + len(t))) for t in tables)


def test_smallest_first_atomic_and_validated():
    with pytest.raises(ValueError):
        BlockManager(0, 16)
    with pytest.raises(ValueError):
        BlockManager(8, -1)
    bm = BlockManager(4, 16)
    assert bm.reserve(0) == [] and bm.stats()["alloc_calls"] == 0
    assert bm.reserve(3) == [0, 1, 2]
    before = bm.stats()
    assert bm.reserve(2) is None and bm.stats() == before
    assert bm.reserve(1) == [3]
    with pytest.raises(ValueError):
        bm.reserve(-1)
    with pytest.raises(ValueError, match="duplicate"):
        bm.free([1, 1])
    bm.free([2, 0])
    with pytest.raises(ValueError, match="not allocated"):
        bm.free([0])
    with pytest.raises(ValueError, match="not allocated"):
        bm.free([1, 2])  # validated as a whole: 1 stays allocated
    assert bm.in_use == 2 and bm.peak == 4
    assert bm.reserve(2) == [0, 2]
    bm.free([])
    assert bm.stats()["free_calls"] == 1
    assert bm.blocks_for(0, 0) == 1 and bm.blocks_for(17, 0) == 2 and bm.blocks_for(2048, 64) == 132


def test_frag_stats_arithmetic():
    fs = FragStats(16)
    assert fs.internal_frag() is None
    fs.observe(1.0, 24, 2)   # 24 of 32 slots
    fs.observe(0.0, 0, 5)    # no time: ignored
    fs.observe(3.0, 16, 1)   # full block
    assert fs.internal_frag() == pytest.approx(1 - (24 + 48) / (32 + 48))
    assert fs.reservation_slack(100, 75) == pytest.approx(0.25)
    assert fs.reservation_slack(0, 5) is None
    assert fs.seat_row_slack(10, 0, 1.0) is None
    assert fs.seat_row_slack(32, 64, 2.0) == pytest.approx(0.5)
    with pytest.raises(ValueError):
        fs.observe(1.0, -1, 1)
