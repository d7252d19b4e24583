"""Generate the golden vectors that pin the oracle (and through it the kernels).

Run once in a container that has the reference checkout (read-only) at ``--reference``:

    python tests/golden/make_golden.py --reference /path/to/llm-serving

Everything here is computed by the reference's OWN functions, imported from its tree:
``tests/reference/paged.py`` (``reference_paged_decode``, ``write_token_reference``,
``gather_pool``), the fp64 per-token ``_dense_oracle`` and input builder ``_build`` of
``tests/unit/test_triton_decode.py``, ``model/paged.py::PagedPool`` (CPU prefill writes),
``serve/block_manager.py::BlockManager`` and the seat path ``model/slab.py::KvSlab`` +
``model/attention/hand_baddbmm.py::HandBaddbmmBackend``. This repository's
``workloads.py`` (repository root) is loaded by file path so its seeded recipes run against the
reference's allocator. Outputs (small) go to ``tests/golden/``; large inputs are not stored:
the tests regenerate them from the recorded seeds and compare a SHA-256 of the bytes.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import math
import random
import sys
from pathlib import Path

import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent


def digest(*tensors) -> str:
    h = hashlib.sha256()
    for t in tensors:
        t = t.detach().cpu().contiguous()
        h.update(str(tuple(t.shape)).encode())
        h.update(str(t.dtype).encode())
        h.update(t.view(torch.uint8).numpy().tobytes() if t.numel() else b"")
    return h.hexdigest()


# The reference's own kernel test grid (tests/unit/test_triton_decode.py:115-125, 263-277)
# plus the extra shapes this repository's GPU tests use. (B, H, H_kv, D, block_size, lengths).
DECODE_CASES = [
    ("seqlen-1-gqa2-d8", 1, 2, 1, 8, 16, [1]),
    ("seqlen-15-16-gqa2-d8", 2, 4, 2, 8, 16, [15, 16]),
    ("seqlen-17-gqa2-d16", 1, 4, 2, 16, 16, [17]),
    ("seqlen-32-and-empty-gqa1", 2, 4, 4, 8, 16, [32, 0]),
    ("seqlen-100-bs32", 2, 4, 2, 16, 32, [100, 33]),
    ("gqa1-bs32-ragged", 3, 2, 2, 8, 32, [16, 17, 15]),
    ("b1-gqa1-d64-l1-bs16", 1, 2, 2, 64, 16, [1]),
    ("b3-gqa2-d128-l15-17-bs16", 3, 8, 4, 128, 16, [15, 16, 17]),
    ("b8-gqa4-d64-bs32", 8, 8, 2, 64, 32, [1, 15, 16, 17, 100, 1, 15, 16]),
    ("b1-gqa8-d256-l1664-bs16", 1, 8, 1, 256, 16, [1664]),
    ("b3-gqa8-d256-bs32", 3, 8, 1, 256, 32, [100, 1664, 1]),
    ("qwen3-b8-l1664", 8, 16, 8, 128, 16, [1664] * 8),
    ("qwen3-ragged-zero", 4, 16, 8, 128, 16, [0, 5, 3000, 129]),
]
SEEDS = {"cpu": 3, "cuda": 13}


def load_reference(root: Path):
    sys.path.insert(0, str(root))
    from model.attention.hand_baddbmm import HandBaddbmmBackend
    from model.layers import apply_rotary_emb_partial, rope_cos_sin
    from model.paged import PagedPool
    from model.slab import KvSlab
    from serve.block_manager import BlockManager
    from tests.reference import paged as ref_paged
    from tests.unit import test_triton_decode as ref_tests

    return {
        "HandBaddbmmBackend": HandBaddbmmBackend,
        "PagedPool": PagedPool,
        "KvSlab": KvSlab,
        "BlockManager": BlockManager,
        "paged": ref_paged,
        "tests": ref_tests,
        "apply_rotary_emb_partial": apply_rotary_emb_partial,
        "rope_cos_sin": rope_cos_sin,
    }


def load_workloads():
    spec = importlib.util.spec_from_file_location(
        "repo_workloads", REPO / "workloads.py"
    )
    module = importlib.util.module_from_spec(spec)
    sys.modules["repo_workloads"] = module  # dataclasses resolve their module by name
    spec.loader.exec_module(module)  # its ``serve.block_manager`` import is the reference's
    return module


def decode_goldens(ref):
    build = ref["tests"]._build
    dense = ref["tests"]._dense_oracle
    oracle = ref["paged"].reference_paged_decode
    records, tensors = [], {}
    for name, B, H, Hkv, D, bs, lengths in DECODE_CASES:
        for dtype in (torch.float32, torch.bfloat16, torch.float16):
            for seed in sorted(set(SEEDS.values())):
                q, k, v, table, seqlen = build(B, H, Hkv, D, bs, lengths, dtype=dtype, seed=seed)
                key = f"decode/{name}/{str(dtype)[6:]}/{seed}"
                out = oracle(q, k, v, table, seqlen)
                # fp32-upcast copy of the same values: the reference for the bf16 tolerance
                out32 = oracle(q.float(), k.float(), v.float(), table, seqlen)
                out64 = dense(q.double(), k.double(), v.double(), table, seqlen, 1.0 / math.sqrt(D))
                tensors[key + "/out"] = out
                tensors[key + "/out_f32"] = out32
                tensors[key + "/out_f64"] = out64
                records.append({"key": key, "case": name, "B": B, "H": H, "H_kv": Hkv, "D": D,
                                "block_size": bs, "lengths": lengths, "dtype": str(dtype)[6:],
                                "seed": seed, "inputs_sha256": digest(q, k, v, table, seqlen)})
    # Explicit scale and the duplicated / -999-tailed table (test_triton_decode.py:137-169).
    q, k, v, table, seqlen = build(2, 4, 2, 8, 16, [17, 5], seed=0)
    tensors["decode/explicit-scale/out"] = oracle(q, k, v, table, seqlen, scale=0.375)
    records.append({"key": "decode/explicit-scale", "B": 2, "H": 4, "H_kv": 2, "D": 8, "block_size": 16,
                    "lengths": [17, 5], "dtype": "float32", "seed": 0, "scale": 0.375,
                    "inputs_sha256": digest(q, k, v, table, seqlen)})
    q, k, v, _, _ = build(2, 4, 2, 8, 16, [50, 64], seed=7, n_blocks=6)
    table = torch.tensor([[3, 0, 3, 5, -999, -999], [5, 1, 4, 0, -999, -999]], dtype=torch.int32)
    seqlen = torch.tensor([50, 64], dtype=torch.int32)
    tensors["decode/duplicated-table/out"] = oracle(q, k, v, table, seqlen)
    tensors["decode/duplicated-table/table"] = table
    records.append({"key": "decode/duplicated-table", "B": 2, "H": 4, "H_kv": 2, "D": 8, "block_size": 16,
                    "lengths": [50, 64], "dtype": "float32", "seed": 7, "n_blocks": 6,
                    "inputs_sha256": digest(q, k, v)})
    return records, tensors


def append_goldens(ref):
    """Pools after the reference's writes (small CPU pools, fp32 and bf16)."""
    PagedPool = ref["PagedPool"]
    write_token = ref["paged"].write_token_reference
    records, tensors = [], {}
    for dtype in (torch.float32, torch.bfloat16):
        for bs in (16, 32):
            gen = torch.Generator().manual_seed(71 + bs)
            pool = PagedPool(2, 8, bs, 2, 8, dtype=dtype, n_head=4)
            table = [7, 0, 5, 3]
            length = bs + 5
            k = torch.randn(1, 2, length, 8, generator=gen)[0].permute(1, 0, 2)  # engine layout
            v = torch.randn(1, 2, length, 8, generator=gen)[0].permute(1, 0, 2)
            pool.write_prefill(0, table, 0, k, v)
            k2 = torch.randn(9, 2, 8, generator=gen)
            v2 = torch.randn(9, 2, 8, generator=gen)
            pool.write_prefill(1, [6, 2, 4], 21, k2, v2)  # starts mid-block
            key = f"append/prefill/{str(dtype)[6:]}/bs{bs}"
            tensors[key + "/k"] = k.contiguous()
            tensors[key + "/v"] = v.contiguous()
            tensors[key + "/k2"] = k2
            tensors[key + "/v2"] = v2
            for layer in range(2):
                tensors[f"{key}/keys{layer}"] = pool.keys[layer]
                tensors[f"{key}/values{layer}"] = pool.values[layer]
            records.append({"key": key, "dtype": str(dtype)[6:], "block_size": bs, "n_blocks": 8,
                            "table0": table, "start0": 0, "table1": [6, 2, 4], "start1": 21})
        # Decode token writes (write_token_reference) for two rows at block boundaries.
        gen = torch.Generator().manual_seed(11)
        pool = PagedPool(1, 8, 16, 2, 4, dtype=dtype, n_head=4)
        tables = [[5, 1, 7], [2, 0, 6]]
        positions = [20, 15]
        k = torch.randn(2, 2, 4, generator=gen)
        v = torch.randn(2, 2, 4, generator=gen)
        write_token(pool, 0, [0, 1], tables, positions, k, v)
        key = f"append/token/{str(dtype)[6:]}"
        tensors[key + "/k"] = k
        tensors[key + "/v"] = v
        tensors[key + "/keys"] = pool.keys[0]
        tensors[key + "/values"] = pool.values[0]
        records.append({"key": key, "dtype": str(dtype)[6:], "tables": tables, "positions": positions,
                        "n_blocks": 8, "block_size": 16})
    return records, tensors


def block_manager_goldens(ref, workloads):
    BlockManager = ref["BlockManager"]
    rng = random.Random(2024)
    bm = BlockManager(64, 16)
    live, trace = [], []
    for _ in range(200):
        if live and rng.random() < 0.45:
            ids = live.pop(rng.randrange(len(live)))
            bm.free(ids)
            trace.append({"op": "free", "ids": ids, "stats": bm.stats()})
        else:
            n = rng.randint(0, 12)
            ids = bm.reserve(n)
            if ids:
                live.append(ids)
            trace.append({"op": "reserve", "n": n, "ids": ids, "stats": bm.stats()})
    blocks_for = [[p, b, bm.blocks_for(p, b)] for p, b in [(0, 0), (1, 0), (16, 0), (17, 0), (2048, 64), (5, 11)]]
    cfg3 = []
    for seed in (0, 1):
        lengths = workloads.lognormal_lengths(64, seed)
        n_blocks = 2 * sum(-(-n // 16) for n in lengths) + 4096
        tables = workloads.fragmented_tables(lengths, n_blocks, 16, seed)
        cfg3.append({"seed": seed, "lengths": lengths, "n_blocks": n_blocks, "tables": tables})
    return {"trace": trace, "blocks_for": blocks_for, "config3": cfg3}


# Rotary cases: (key, n_kv_head, head_dim, rotary_dim, theta, dtype, positions). The K rows a
# decode step appends are rotated by the model just before the write; the fused append +
# decode must store exactly what this produces.
ROPE_CASES = [
    ("rope/qwen3-bf16", 8, 128, 128, 1e6, torch.bfloat16, [0, 1, 17, 2047, 5000, 40000]),
    ("rope/qwen3-f16", 8, 128, 128, 1e6, torch.float16, [3, 900, 31000]),
    ("rope/qwen3-f32", 8, 128, 128, 1e6, torch.float32, [2, 2048]),
    ("rope/qwen35-partial-bf16", 2, 256, 64, 1e7, torch.bfloat16, [0, 513, 4095, 100000]),
]


def rope_goldens(ref):
    """Per-row decode rotation: cos/sin of each row's position from the reference's
    rope_cos_sin (rows stacked as (B, 1, rotary_dim / 2)), K (B, 1, H_kv, D) rotated by the
    reference's apply_rotary_emb_partial."""
    gen = torch.Generator().manual_seed(41)
    records, tensors = [], {}
    for key, hkv, d, rot, theta, dtype, positions in ROPE_CASES:
        rows = [ref["rope_cos_sin"](d, theta, p, 1, dtype=dtype, rotary_dim=None if rot == d else rot)
                for p in positions]
        cos = torch.stack([c for c, _ in rows])  # (B, 1, rot / 2)
        sin = torch.stack([s for _, s in rows])
        k = torch.randn(len(positions), 1, hkv, d, generator=gen).to(dtype)
        out = ref["apply_rotary_emb_partial"](k, cos, sin, rot)
        tensors[key + "/k"] = k
        tensors[key + "/cos"] = cos
        tensors[key + "/sin"] = sin
        tensors[key + "/out"] = out
        records.append({"key": key, "n_kv_head": hkv, "head_dim": d, "rotary_dim": rot, "theta": theta,
                        "dtype": str(dtype), "positions": positions})
    return records, tensors


def seat_goldens(ref, workloads):
    """Config 1 through the reference's seat path and oracle (bf16 on CPU)."""
    wl = workloads.config1(device="cpu", seed=0)
    q, k, v = wl.q[0], wl.k_pools[0], wl.v_pools[0]
    B, H, D = q.shape
    Hkv = k.shape[2]
    lengths = wl.seqlen.tolist()
    lpad = -(-max(lengths) // 64) * 64
    pool_like = type("Pool", (), {})()
    pool_like.n_layer, pool_like.block_size, pool_like.n_kv_head, pool_like.head_dim = 1, 16, Hkv, D
    pool_like.keys, pool_like.values, pool_like.dtype, pool_like.device = [k], [v], k.dtype, k.device
    gk, gv = ref["paged"].gather_pool(pool_like, 0, wl.tables, lengths, lpad)
    slab = ref["KvSlab"](1, B, Hkv, D, lpad, dtype=torch.bfloat16, n_head=H)
    slab.keys[0].copy_(gk)
    slab.values[0].copy_(gv)
    for row, n in enumerate(lengths):
        slab.activate(row, n)
    slab.build_mask(next_token=False)
    seat = ref["HandBaddbmmBackend"]().decode(q.unsqueeze(2), slab.keys[0], slab.values[0], bias=slab.bias)[:, :, 0]
    out = ref["paged"].reference_paged_decode(q, k, v, wl.block_table, wl.seqlen)
    out32 = ref["paged"].reference_paged_decode(q.float(), k.float(), v.float(), wl.block_table, wl.seqlen)
    record = {"key": "seat/config1", "lengths": lengths, "lpad": lpad, "tables": wl.tables,
              "inputs_sha256": digest(q, k, v, wl.block_table, wl.seqlen),
              "gather_sha256": digest(gk, gv)}
    return record, {"seat/config1/seat": seat, "seat/config1/out": out, "seat/config1/out_f32": out32}


def main(argv=None) -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", required=True, type=Path)
    args = parser.parse_args(argv)
    ref = load_reference(args.reference)
    workloads = load_workloads()
    torch.manual_seed(0)
    dec_records, dec_tensors = decode_goldens(ref)
    app_records, app_tensors = append_goldens(ref)
    bm = block_manager_goldens(ref, workloads)
    seat_record, seat_tensors = seat_goldens(ref, workloads)
    rope_records, rope_tensors = rope_goldens(ref)
    tensors = {**dec_tensors, **app_tensors, **seat_tensors, **rope_tensors}
    torch.save(tensors, HERE / "golden_tensors.pt")
    meta = {"decode": dec_records, "append": app_records, "seat": seat_record, "rope": rope_records,
            "torch": torch.__version__, "generator": "tests/golden/make_golden.py"}
    (HERE / "golden_meta.json").write_text(json.dumps(meta, indent=1))
    (HERE / "block_manager.json").write_text(json.dumps(bm))
    size = (HERE / "golden_tensors.pt").stat().st_size
    print(f"wrote {len(tensors)} tensors ({size / 1e6:.2f} MB), {len(dec_records)} decode cases")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
