"""Invariants of the stream-K plan (higgs-audio.cpp_b200/csrc/hkv_plan.h), CPU.

Also walks the two-level merge: a segment with more than 16 partials is
merged in groups of max(8, ceil(sqrt(n))) by the last warp of each group,
and the last group merges the group partials; every segment must finish
exactly once.

Restates the plan's formulas -- W = min(U, grid warps) equal shares
floor(w U / W) .. floor((w + 1) U / W), warp_of(a) = ceil((a + 1) W / U) - 1,
part_off from the CTAs (WPC consecutive warps) a (slot, KV head) segment
touches, warp_entry -- and walks every warp the way attention_kernel does:
the warps of one CTA that share a segment leave their partials in shared
memory (slot 1 for the run's first warp, 0 for the others), the last of them
(run ticket) merges and publishes the CTA's partial.  Checks that every
shared-memory slot and run ticket is used by one run only, that each
segment's CTA partials are written exactly once and merged exactly once (or
the output written directly when one CTA holds the whole segment).  Empty
shares would break this (a segment would count a partial that never
arrives), which is why W is capped at U.
"""
from __future__ import annotations

import random

import pytest


WPC = 6  # warps per CTA (kAttnWarps)


def plan(npages, G, w_full, cta_merge=None):
    n = len(npages)
    unit_off = [0]
    for np_ in npages:
        unit_off.append(unit_off[-1] + np_ * G)
    U = unit_off[-1]
    W = min(U, w_full)
    if cta_merge is None:  # plan_cta_merge: two CTAs' worth of warps per segment
        cta_merge = W >= 2 * WPC * n * G
    span = WPC if cta_merge else 1
    warp_of = lambda a: ((a + 1) * W + U - 1) // U - 1  # noqa: E731
    part_off = [0]
    for e, np_ in enumerate(npages):
        for h in range(G):
            a = unit_off[e] + h * np_
            part_off.append(part_off[-1] + warp_of(a + np_ - 1) // span - warp_of(a) // span + 1)
    warp_entry, e = [], 0
    for k in range(W):
        ub = k * U // W
        while e + 1 < n and unit_off[e + 1] <= ub:
            e += 1
        warp_entry.append(e)
    return unit_off, part_off, warp_entry, U, W, warp_of, cta_merge


SINGLE_MAX = 16


def group_size(nparts):  # max(8, ceil(sqrt(nparts))), as merge_group_size
    g = 8
    while g * g < nparts:
        g += 1
    return g


def n_groups_of(nparts):
    return 0 if nparts <= SINGLE_MAX else -(-nparts // group_size(nparts))


def walk(npages, G=8, w_full=148 * 6, cta_merge=None):
    unit_off, part_off, warp_entry, U, W, warp_of, cta_merge = plan(npages, G, w_full, cta_merge)
    span = WPC if cta_merge else 1
    assert part_off[-1] <= W + len(npages) * G  # the engine's partial capacity
    n_groups = [n_groups_of(part_off[i + 1] - part_off[i]) for i in range(len(npages) * G)]
    assert sum(n_groups) <= (W + len(npages) * G) // 8 + len(npages) * G
    written, tickets, merges, direct = {}, {}, {}, {}
    group_tickets, group_merges = {}, {}
    slots_used, run_tickets, run_owner = {}, {}, {}
    for gw in range(W):
        ub, ue = gw * U // W, (gw + 1) * U // W
        assert ub < ue, "empty share"
        e = warp_entry[gw]
        np_ = npages[e]
        rem = ub - unit_off[e]
        h, i = rem // np_, rem % np_
        seg = None

        def flush(seg):
            e_, h_, part, nparts, run_lo, run_m = seg
            eh = e_ * G + h_
            if run_m > 1:
                slot = (gw, 1 if gw == run_lo else 0)
                assert slot not in slots_used, "shared-memory slot reused"
                slots_used[slot] = eh
                key = (gw // span, run_lo % span)
                assert run_owner.setdefault(key, eh) == eh, "run ticket shared by two runs"
                t = run_tickets.get(key, 0)
                run_tickets[key] = t + 1
                if t != run_m - 1:
                    return
            if nparts == 1:
                direct[eh] = direct.get(eh, 0) + 1
                return
            assert part_off[eh] <= part < part_off[eh + 1]
            written[part] = written.get(part, 0) + 1
            if nparts <= SINGLE_MAX:
                t = tickets.get(eh, 0)
                tickets[eh] = t + 1
                if t == nparts - 1:
                    merges[eh] = merges.get(eh, 0) + 1
                return
            gs = group_size(nparts)
            g = (part - part_off[eh]) // gs
            g_size = min(gs, nparts - g * gs)
            t = group_tickets.get((eh, g), 0)
            group_tickets[(eh, g)] = t + 1
            if t != g_size - 1:
                return
            group_merges[(eh, g)] = group_merges.get((eh, g), 0) + 1
            t = tickets.get(eh, 0)
            tickets[eh] = t + 1
            if t == n_groups_of(nparts) - 1:
                merges[eh] = merges.get(eh, 0) + 1

        for u in range(ub, ue):
            if u == ub or i == 0:
                if u != ub:
                    flush(seg)
                a = unit_off[e] + h * np_
                first, last = warp_of(a), warp_of(a + np_ - 1)
                cta = gw // span
                run_lo = max(first, cta * span)
                run_hi = min(last, cta * span + span - 1)
                seg = (e, h, part_off[e * G + h] + (cta - first // span),
                       last // span - first // span + 1, run_lo, run_hi - run_lo + 1)
            i += 1
            if i == np_:
                i, h = 0, h + 1
                if h == G:
                    h, e = 0, e + 1
                    if e < len(npages):
                        np_ = npages[e]
        flush(seg)
    for eh in range(len(npages) * G):
        if part_off[eh + 1] - part_off[eh] == 1:
            assert direct.get(eh) == 1
        else:
            assert merges.get(eh) == 1
            for p in range(part_off[eh], part_off[eh + 1]):
                assert written.get(p) == 1
            for g in range(n_groups[eh]):
                assert group_merges.get((eh, g)) == 1


@pytest.mark.parametrize("cta_merge", [None, False, True])
@pytest.mark.parametrize("npages", [[3, 1], [1] * 4, [1] * 300, [3, 19, 63], [2048],
                                    [1, 1000, 1, 1000], [40], [33, 2048]])
def test_plan_partitions_every_segment(npages, cta_merge):
    walk(npages, cta_merge=cta_merge)


@pytest.mark.parametrize("cta_merge", [None, False, True])
def test_plan_random_batches(cta_merge):
    rng = random.Random(0)
    for _ in range(30):
        walk([rng.randint(1, 1025) for _ in range(rng.randint(1, 64))],
             G=rng.choice([1, 2, 4, 8]), cta_merge=cta_merge)


def test_cta_merge_rule():
    # long segments (one request near the context limit) merge per CTA;
    # many short ones (16 slots) keep one partial per warp
    assert plan([2048], 8, 148 * 6)[-1]
    assert plan([2048], 1, 148 * 6)[-1]
    assert not plan([100] * 16, 8, 148 * 6)[-1]
    assert not plan([600] * 32, 8, 148 * 6)[-1]
