"""CPU check of the decode kernel's split-item bookkeeping in unit mode.

``pd_decode_kernel`` (llm-serving_b200/csrc/pd_decode_kernel.cuh) cuts the units (row, item,
tile) into one contiguous range per worker warp. An item that several ranges overlap is
finished by the last of its pieces to arrive on the item's counter. This test restates, in
Python, which pieces arrive and which slots the merging warp reads, and checks on random
shapes that the two agree:

* a piece that ends inside its worker's range (the *mid* piece, only the item's last worker
  can have one) is written to slot 0 of that worker and arrives on its own;
* the pieces that end their ranges arrive one per CTA group when workers are numbered CTA by
  CTA (``grouped``: the group's last warp folds them in shared memory and writes the group's
  piece to slot 1 of the group's first worker, or writes the output itself when its group is
  the whole item), otherwise one each, in slot 1 of their worker;
* the merger expects ``global_reps + mid`` arrivals and reads the slots in that order.

It is a restatement of device code (``item_span``, ``global_reps``, ``merge_if_last``), so it
guards the arithmetic, not the kernel; the GPU parity tests cover the kernel itself.
"""

import random


def worker_of(u, units, workers):
    return ((u + 1) * workers - 1) // units


def _check(lens_tiles, items_per_row, workers, nwarps, grouped):
    pre = [0]
    for t in lens_tiles:
        pre.append(pre[-1] + t)
    units = items_per_row * pre[-1]
    written, arrivals = {}, {}

    def span(xs, xe):
        wa, wb = worker_of(xs, units, workers), worker_of(xe - 1, units, workers)
        mid = (wb + 1) * units // workers > xe
        return wa, wb, (wb - 1 if mid else wb), mid

    def reps(wa, wt):
        return (wt // nwarps - wa // nwarps + 1) if grouped else (wt - wa + 1)

    for w in range(workers):
        u0, u1 = w * units // workers, (w + 1) * units // workers
        assert u0 < u1, "every range is non-empty"
        segs, u = [], u0
        while u < u1:
            b = max(i for i in range(len(lens_tiles)) if items_per_row * pre[i] <= u and lens_tiles[i] > 0)
            nt = lens_tiles[b]
            item = (u - items_per_row * pre[b]) // nt
            xs = items_per_row * pre[b] + item * nt
            segs.append((b, item, u, min(xs + nt, u1), xs, xs + nt))
            u = min(xs + nt, u1)
        for k, (b, item, s0, s1, xs, xe) in enumerate(segs):
            if s0 == xs and s1 == xe:
                continue  # whole item in one range: written directly
            key = (b, item)
            if k != len(segs) - 1:  # mid piece
                written.setdefault(key, set()).add(w * 2)
                arrivals[key] = arrivals.get(key, 0) + 1
                continue
            wa, wb, wt, mid = span(xs, xe)
            assert wa <= w <= wt
            cta0 = (w // nwarps) * nwarps
            m0, m1 = max(wa, cta0) - cta0, min(wt, cta0 + nwarps - 1) - cta0
            if grouped and m1 > m0:
                if w - cta0 == m1 and not (reps(wa, wt) == 1 and not mid):
                    written.setdefault(key, set()).add((cta0 + m0) * 2 + 1)
                    arrivals[key] = arrivals.get(key, 0) + 1
            else:
                written.setdefault(key, set()).add(w * 2 + 1)
                arrivals[key] = arrivals.get(key, 0) + 1

    for (b, item), slots in written.items():
        xs = items_per_row * pre[b] + item * lens_tiles[b]
        wa, wb, wt, mid = span(xs, xs + lens_tiles[b])
        nreps = reps(wa, wt)
        assert arrivals[(b, item)] == nreps + mid
        expect = {wb * 2} if mid else set()
        for i in range(nreps):
            rep = (wa if i == 0 else (wa // nwarps + i) * nwarps) if grouped else wa + i
            expect.add(rep * 2 + 1)
        assert expect == slots


def test_every_split_item_gets_the_arrivals_and_slots_its_merger_expects():
    rng = random.Random(1)
    checked = 0
    for _ in range(2000):
        lens = [rng.choice([0, 1, 2, 3, 5, 8, 13, 40]) for _ in range(rng.randint(1, 6))]
        ipr = rng.choice([1, 2, 3, 4])
        units = ipr * sum(lens)
        if units == 0:
            continue
        workers = rng.randint(1, min(units, 64))
        nwarps = rng.choice([2, 4, 8])
        for grouped in (False, True):
            _check(lens, ipr, workers, nwarps, grouped)
            checked += 1
    assert checked > 3000


def test_qwen35_shape_folds_to_three_cta_pieces_per_item():
    # 32 rows x 256 tiles, 2 items per row, 1152 workers (18 per item) in CTAs of 8 warps:
    # every item's 18 range-ending pieces reach the global merge as 3 CTA-group pieces.
    _check([256] * 32, 2, 1152, 8, True)
    units, workers = 2 * 256 * 32, 1152
    for item in range(64):
        xs = item * 256
        wa, wb = worker_of(xs, units, workers), worker_of(xs + 255, units, workers)
        assert wb - wa + 1 == 18
        assert wb // 8 - wa // 8 + 1 == 3
