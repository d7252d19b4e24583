"""The drop-in boundary on a host without a GPU: the C-ABI library and the Python surface.

* ``libpaged_decode.so`` loads and exports every entry point ``include/paged_decode.h``
  declares (and the ctypes table binds exactly those);
* argument errors are reported by status code before any CUDA call;
* the Python modules keep the reference's error classes and message substrings
  (tests/unit/test_triton_decode.py:206-242, 405-459; tests/unit/test_paged_kv.py:222-242,
  522-542) -- RuntimeError for "no backend / not CUDA", ValueError for layout errors.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import pytest
import torch

from helpers import build_case
from model import _native

HEADER = Path(__file__).resolve().parent.parent / "include" / "paged_decode.h"


def _declared() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(pd_[a-z_0-9]+)\s*\(", text))


def test_library_loads_and_exports_every_declared_symbol():
    assert _native.AVAILABLE, _native.LOAD_ERROR
    declared = _declared()
    assert declared, "no declarations parsed"
    raw = ctypes.CDLL(str(_native.LIB_PATH))
    for name in sorted(declared):
        assert hasattr(raw, name), f"{name} declared in the header but not exported"
    assert declared == set(_native.EXPORTS), "ctypes table and header disagree"
    assert _native.lib.pd_abi_version() == 1


def test_status_strings():
    names = {s: _native.status_string(s) for s in range(5)}
    assert names[0] == "ok" and "invalid" in names[1] and "unsupported" in names[2]
    assert "CUDA" in names[3] and "workspace" in names[4]


def _pd_decode(**over):
    args = dict(q=None, q_sb=0, q_sh=0, k=None, v=None, n_blocks=8, bs=16, ks=None, vs=None,
                table=None, bt_stride=4, max_blocks=4, seqlen=None, out=None, o_sb=0, o_sh=0,
                B=1, H=4, Hkv=2, D=64, dtype=_native.PD_BF16, scale=1.0, ws=None, ws_bytes=0, stream=None)
    args.update(over)
    s3 = (ctypes.c_int64 * 3)(2048, 128, 64)
    return _native.lib.pd_decode(args["q"], args["q_sb"], args["q_sh"], args["k"], args["v"], args["n_blocks"],
                                 args["bs"], s3, s3, args["table"], args["bt_stride"], args["max_blocks"],
                                 args["seqlen"], args["out"], args["o_sb"], args["o_sh"], args["B"], args["H"],
                                 args["Hkv"], args["D"], args["dtype"], args["scale"], args["ws"],
                                 args["ws_bytes"], args["stream"])


@pytest.mark.parametrize("over,status", [
    (dict(D=12), _native.PD_ERR_INVALID),         # not a power of two
    (dict(D=512), _native.PD_ERR_UNSUPPORTED),    # beyond the kernel's 256
    (dict(H=3), _native.PD_ERR_INVALID),          # H not a multiple of H_kv
    (dict(bs=24), _native.PD_ERR_INVALID),        # block size not a power of two
    (dict(dtype=7), _native.PD_ERR_INVALID),
    (dict(B=-1), _native.PD_ERR_INVALID),
    (dict(n_blocks=0), _native.PD_ERR_INVALID),
])
def test_pd_decode_rejects_bad_arguments_before_touching_cuda(over, status):
    assert _pd_decode(**over) == status


def test_other_entry_points_reject_bad_arguments():
    lib = _native.lib
    s3 = (ctypes.c_int64 * 3)(1, 1, 1)
    assert lib.pd_lse_merge(None, None, None, 1, 1, 0, 1, 1, 8, None, 8, 8, 2, None) == _native.PD_ERR_INVALID
    assert lib.pd_lse_merge(None, None, None, 1, 1, 1, 1, 1, 6, None, 8, 8, 2, None) == _native.PD_ERR_UNSUPPORTED
    assert lib.pd_kv_append_slots(None, None, 8, 16, s3, s3, 2, None, 9, None, s3, None, s3, 2, 1, 2, 8, None) \
        == _native.PD_ERR_INVALID  # unknown slot dtype
    assert lib.pd_kv_append_table(None, None, 8, 16, s3, s3, 2, None, 4, 4, None, None, s3, None, s3, 2, 2, 2, 8,
                                  None) == _native.PD_ERR_INVALID  # no table / pos
    assert lib.pd_plan_create(None, 1, None, None, 8, 16, s3, s3, None, 4, 4, None, 1, 4, 2, 64, 2, 1.0, None,
                              0) == _native.PD_ERR_INVALID
    bits = ctypes.c_uint(0)
    assert lib.pd_device_error(None, 0) == _native.PD_ERR_INVALID
    del bits


def test_tuning_is_validated_and_restorable():
    before = _native.get_decode_tuning()
    with pytest.raises(ValueError):
        _native.set_decode_tuning(16, 3, 1, 4)   # more than 8 warps
    with pytest.raises(ValueError):
        _native.set_decode_tuning(8, 8, 1, 4)    # 8 x 8 x 8 KB of stages > 227 KB
    assert _native.get_decode_tuning() == before
    _native.set_decode_tuning(*before)


def test_decode_mode_is_validated_and_restorable():
    before = _native.get_decode_mode()
    with pytest.raises(ValueError):
        _native.set_decode_mode(3)
    with pytest.raises(ValueError):
        _native.set_decode_mode(-1)
    with pytest.raises(ValueError):
        _native.set_decode_mode(1, 9)
    assert _native.get_decode_mode() == before
    with pytest.raises(ValueError):
        _native.set_decode_mode(0, 0, 65)
    _native.set_decode_mode(1, 3, 5)
    assert _native.get_decode_mode() == (1, 3, 5)
    _native.set_decode_mode(0, 0, -1)
    assert _native.get_decode_mode() == (0, 0, 5)
    _native.set_decode_mode(2, 0, -1)
    assert _native.get_decode_mode() == (2, 0, 5)
    _native.set_decode_mode(*before)
    assert _native.get_decode_mode() == before


# ------------------------------------------------------------ Python surface (no GPU needed)


def test_paged_decode_rejects_cpu_tensors():
    from model.triton_decode import paged_decode

    q, k, v, table, seqlen = build_case(2, 4, 2, 8, 16, [17, 5])
    with pytest.raises(RuntimeError, match="Triton|CUDA"):
        paged_decode(q, k, v, table, seqlen)


def test_paged_decode_raises_when_the_library_is_unavailable(monkeypatch):
    import model.triton_decode as module

    q, k, v, table, seqlen = build_case(2, 4, 2, 8, 16, [17, 5])
    monkeypatch.setattr(module, "TRITON_AVAILABLE", False)
    with pytest.raises(RuntimeError, match="Triton"):
        module.paged_decode(q, k, v, table, seqlen)
    with pytest.raises(RuntimeError, match="Triton"):
        module.paged_decode_plan(q, [k], [v], table, seqlen)


@pytest.mark.parametrize("mutate,match", [
    (lambda a: a.update(q=a["q"][0]), "must be"),
    (lambda a: a.update(k=a["k"].bfloat16()), "share one dtype"),
    (lambda a: a.update(k=a["k"][..., :-1], v=a["v"][..., :-1]), "head_dim"),
    (lambda a: a.update(q=a["q"][:, :3]), "multiple of n_kv_head"),
    (lambda a: a.update(table=a["table"].long()), "int32"),
    (lambda a: a.update(seqlen=a["seqlen"] + 1000), "capacity"),
    (lambda a: a.update(seqlen=torch.tensor([-1, 3], dtype=torch.int32)), ">= 0"),
    (lambda a: a.update(seqlen=a["seqlen"].float()), "int32 or int64"),
])
def test_validation_messages_match_the_reference(mutate, match):
    from model import triton_decode

    q, k, v, table, seqlen = build_case(2, 4, 2, 16, 16, [17, 5])
    args = dict(q=q, k=k, v=v, table=table, seqlen=seqlen)
    mutate(args)
    triton_decode._SEQ_CHECK = None
    with pytest.raises(ValueError, match=match):
        triton_decode._validate(args["q"], args["k"], args["v"], args["table"], args["seqlen"])


def test_validation_accepts_int64_seqlen_and_caches_the_range_check():
    from model import triton_decode

    q, k, v, table, seqlen = build_case(2, 4, 2, 16, 16, [17, 5])
    triton_decode._SEQ_CHECK = None
    triton_decode._validate(q, k, v, table, seqlen.long())
    s32 = seqlen.clone()
    triton_decode._validate(q, k, v, table, s32)
    assert triton_decode._SEQ_CHECK[0] is s32
    s32[0] = 1000  # in-place change bumps the version: revalidated, not served from the cache
    with pytest.raises(ValueError, match="capacity"):
        triton_decode._validate(q, k, v, table, s32)


def test_head_dim_outside_the_kernel_range_is_a_value_error():
    from model import triton_decode

    q, k, v, table, seqlen = build_case(1, 2, 1, 4, 16, [3])
    triton_decode._SEQ_CHECK = None
    with pytest.raises(ValueError, match="head_dim"):
        triton_decode._validate(q, k, v, table, seqlen)


def test_pool_write_checks_run_before_the_cuda_requirement():
    from model.paged import PagedPool

    pool = PagedPool(2, 4, 16, 2, 4, n_head=4)  # CPU pool: host checks work, writes do not
    k = torch.randn(2, 2, 4)
    v = torch.randn(2, 2, 4)
    slots = torch.tensor([0, 1])
    with pytest.raises(ValueError, match="one entry per token"):
        pool.write_slots(0, slots[:1], k, v)
    with pytest.raises(ValueError, match="integer tensor"):
        pool.write_slots(0, slots.float(), k, v)
    with pytest.raises(ValueError, match="k/v shapes differ"):
        pool.write_slots(0, slots, k, v[:1])
    with pytest.raises(ValueError, match="head shape"):
        pool.write_slots(0, slots, k[:, :, :2], v[:, :, :2])
    with pytest.raises(IndexError, match="outside the pool's"):
        pool.write_slots(2, slots, k, v)
    with pytest.raises(RuntimeError, match="CUDA"):
        pool.write_slots(0, slots, k, v)
    with pytest.raises(IndexError):
        pool.write_prefill(0, [0], 0, torch.randn(17, 2, 4), torch.randn(17, 2, 4))  # table too short
    with pytest.raises(IndexError):
        pool.write_prefill(0, [4], 0, k, v)  # id outside the pool
    assert pool.bytes() == 2 * 2 * 4 * 16 * 2 * 4 * 4


def test_prefill_slot_map_is_cached_per_table_and_start():
    from model.paged import PagedPool

    pool = PagedPool(1, 8, 16, 2, 4)
    a = pool.slot_ids([7, 0, 5], 0, 21)
    assert a.tolist() == [7 * 16 + t for t in range(16)] + [0 * 16 + t for t in range(5)]
    assert pool.slot_ids([7, 0, 5], 0, 21) is a
    b = pool.slot_ids([6, 2, 4], 21, 14)
    assert b is not a and b.tolist()[:1] == [2 * 16 + 5]
    with pytest.raises(ValueError):
        pool.slot_ids([1], -1, 3)


def test_paged_kv_rejects_a_cpu_pool_with_a_clear_error():
    from model.paged import PagedKV, PagedPool

    pool = PagedPool(1, 4, 16, 2, 4)
    with pytest.raises(ValueError, match="CUDA") as info:
        PagedKV(pool, [[0]], [3], rope_len=16)
    assert "oracle" in str(info.value)
