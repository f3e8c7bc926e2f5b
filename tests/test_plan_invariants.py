"""Invariants of the stream-K plan (higgs-audio.cpp_b200/csrc/hkv_plan.h), CPU.

The plan builder itself is compiled from its header (tests/cpp/plan_dump.cpp
prints its descriptor) and checked against a restatement here:
- shares: the unit range [0, U) is cut greedily into consecutive shares of
  cost at most B (a unit costs 16, leaving a segment inside a share costs 32
  when the share held it from its first page, 80 otherwise; a share never
  enters a segment it cannot take a unit of), and B is the smallest budget
  that needs at most W = min(U, grid warps) shares;
- segments: each (slot, KV head) segment records its first and last warp
  and its partial count (warps, or CTAs of WPC warps with the CTA merge).

The plan also chooses where the split partials are merged: by a combine
launch after the attention grid for CTA-merged segments of at most 32
partials, else inside the launch.  For one long request it may instead give
every KV head a thread-block cluster of C CTAs (plan_cluster), whose CTA
partials meet in the first CTA's shared memory: checked here are the choice
of C and that cluster h covers exactly head h's pages, evenly, one CTA
partial per cluster rank.

Then every warp is walked the way attention_kernel does, with the two-level
merge (a segment with more than 16 partials is merged in groups of
max(8, ceil(sqrt(n))) by the last warp of each group, and the last group
merges the group partials): the warps of one CTA that share a segment leave
their partials in shared memory (slot 1 for the run's first warp, 0 for the
others), the last of them (run ticket) merges and publishes the CTA's
partial.  Checks that every shared-memory slot and run ticket is used by one
run only, that each segment's partials are written exactly once and merged
exactly once (or the output written directly when one warp or CTA holds the
whole segment), and that no share past the last non-empty one is counted.
"""
from __future__ import annotations

import random
import shutil
import subprocess
from pathlib import Path

import pytest

REPO = Path(__file__).resolve().parents[1]
WPC = 8  # warps per CTA (kAttnWarps)
UNIT, LEAVE_WHOLE, LEAVE_SHARED = 16, 32, 80


@pytest.fixture(scope="module")
def plan_dump(tmp_path_factory):
    gxx = shutil.which("g++", path="/usr/bin:/bin")
    cuda_inc = Path("/usr/local/cuda/include")
    if gxx is None or not (cuda_inc / "cuda_runtime.h").exists():
        pytest.skip("no system g++ or CUDA headers")
    exe = tmp_path_factory.mktemp("plan") / "plan_dump"
    subprocess.run([gxx, "-std=c++17", "-O1", "-Wall", "-Werror",
                    f"-I{REPO / 'higgs-audio.cpp_b200' / 'csrc'}", f"-I{cuda_inc}",
                    str(REPO / "tests" / "cpp" / "plan_dump.cpp"), "-o", str(exe)], check=True)

    def run(batches):
        """batches: list of (G, W, positions); returns one parsed plan each."""
        text = "".join(f"{G} {W} " + " ".join(map(str, pos)) + "\n" for G, W, pos in batches)
        out = subprocess.run([str(exe)], input=text, capture_output=True, text=True, check=True,
                             timeout=120).stdout.splitlines()
        plans, i = [], 0
        for G, W, pos in batches:
            hdr = out[i].split()
            assert hdr[0] == "plan"
            shares, budget, cta, n_parts, n_groups, combine = map(int, hdr[1:])
            starts = list(map(int, out[i + 1].split()[1:]))
            n_seg = len(pos) * G
            segs = [tuple(map(int, out[i + 2 + j].split()[1:])) for j in range(n_seg)]
            part2 = list(map(int, out[i + 2 + n_seg].split()[1:]))
            warps = list(map(int, out[i + 3 + n_seg].split()[1:]))
            i += 4 + n_seg
            plans.append(dict(shares=shares, budget=budget, cta_merge=bool(cta), combine=bool(combine),
                              n_parts=n_parts,
                              n_groups=n_groups, starts=starts, segs=segs, part2=part2,
                              warps=[tuple(warps[k:k + 3]) for k in range(0, len(warps), 3)]))
        return plans
    run.exe = exe
    return run


def cut(npages, G, B, max_shares):
    """The greedy cut: share starts, or None when more than max_shares are needed."""
    seg_np = [np_ for np_ in npages for _ in range(G)]
    starts, s, i, u = [], 0, 0, 0
    while s < len(seg_np):
        if len(starts) == max_shares:
            return None
        starts.append(u)
        budget, from_first = B, i == 0
        while True:
            take = min(seg_np[s] - i, budget // UNIT)
            assert take >= 1
            i, u, budget = i + take, u + take, budget - take * UNIT
            if i < seg_np[s]:
                break
            s, i = s + 1, 0
            if s == len(seg_np):
                break
            leave = LEAVE_WHOLE if from_first else LEAVE_SHARED
            if budget - leave < UNIT:
                break
            budget -= leave
            from_first = True
    return starts


def restate(npages, G, w_full, cta_merge=None):
    U = sum(npages) * G
    W = min(U, w_full)
    if cta_merge is None:  # plan_cta_merge: two CTAs' worth of warps per segment
        cta_merge = W >= 2 * WPC * len(npages) * G
    B = UNIT  # smallest feasible budget, by a plain upward search from the bound
    B = max(B, UNIT * -(-U // W))
    while cut(npages, G, B, W) is None:
        B += 1
    starts = cut(npages, G, B, W)
    shares = len(starts)
    starts = starts + [U] * (W - shares) + [U]
    span = WPC if cta_merge else 1
    segs, parts, k = [], 0, 0
    a = 0
    for np_ in npages:
        for _ in range(G):
            while starts[k + 1] <= a:
                k += 1
            last = k
            while starts[last + 1] <= a + np_ - 1:
                last += 1
            n_p = last // span - k // span + 1
            segs.append((parts, n_p, k, last))
            parts += n_p
            a += np_
    return dict(U=U, W=W, B=B, shares=shares, starts=starts, segs=segs, cta_merge=cta_merge)


SINGLE_MAX = 16


def group_size(nparts):  # max(8, ceil(sqrt(nparts))), as merge_group_size
    g = 8
    while g * g < nparts:
        g += 1
    return g


def n_groups_of(nparts):
    return 0 if nparts <= SINGLE_MAX else -(-nparts // group_size(nparts))


def walk(plan_dump, npages, G=8, w_full=148 * WPC):
    pos = [16 * np_ - 1 - (j % 16) for j, np_ in enumerate(npages)]  # np_ pages each
    got = plan_dump([(G, min(sum(npages) * G, w_full), pos)])[0]
    ref = restate(npages, G, w_full)
    U, W = ref["U"], ref["W"]
    assert got["budget"] == ref["B"] and got["shares"] == ref["shares"]
    assert got["starts"] == ref["starts"]
    assert got["segs"] == ref["segs"] and got["cta_merge"] == ref["cta_merge"]
    assert got["n_parts"] == sum(n for _, n, _, _ in ref["segs"])
    # merged by the combine launch: CTA-merged segments of at most 32 partials
    max_parts = max(n for _, n, _, _ in ref["segs"])
    assert got["combine"] == (ref["cta_merge"] and 1 < max_parts <= 32)
    n_seg = len(npages) * G
    n_groups = [n_groups_of(sg[1]) for sg in ref["segs"]]
    assert got["part2"] == [sum(n_groups[:i]) for i in range(n_seg + 1)]
    assert got["n_parts"] <= W + n_seg  # the engine's partial capacity
    assert sum(n_groups) <= (W + n_seg) // 8 + n_seg
    # the tighter bound the no-allocation entry point sizes its scratch by
    parts_bound = W + n_seg
    assert sum(n_groups) <= parts_bound // 8 + parts_bound // 17 + 1
    # the cost bound: no share costs more than B, and B is not loose
    span = WPC if ref["cta_merge"] else 1
    starts, segs = ref["starts"], ref["segs"]
    seg_start = []
    a = 0
    for np_ in npages:
        for _ in range(G):
            seg_start.append(a)
            a += np_
    seg_start.append(U)
    for k in range(ref["shares"]):
        ub, ue = starts[k], starts[k + 1]
        assert ub < ue, "empty share inside the range"
        crossed = [s for s in range(n_seg) if ub < seg_start[s + 1] < ue]
        cost = UNIT * (ue - ub)
        for j, s in enumerate(crossed):
            held_from_first = (seg_start[s] >= ub) if j == 0 else True
            cost += LEAVE_WHOLE if held_from_first else LEAVE_SHARED
        assert cost <= ref["B"]
    assert ref["B"] == UNIT or cut(npages, G, ref["B"] - 1, W) is None

    written, tickets, merges, direct = {}, {}, {}, {}
    group_tickets, group_merges = {}, {}
    slots_used, run_tickets, run_owner = {}, {}, {}
    warp_records = iter(got["warps"])
    seg_of = []
    for s in range(n_seg):
        seg_of.extend([s] * (seg_start[s + 1] - seg_start[s]))
    for gw in range(W):
        ub, ue = starts[gw], starts[gw + 1]
        if ub >= ue:
            assert gw >= ref["shares"]
            assert all(not (f <= gw <= l) for _, _, f, l in segs), "idle warp counted"
            continue
        s0 = seg_of[ub]
        e0, h0, i0 = s0 // G, s0 % G, ub - seg_start[s0]
        assert next(warp_records) == (e0, h0, i0)
        seg = None

        def flush(seg):
            eh, part, nparts, run_lo, run_m = seg
            p_first = segs[eh][0]
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
            assert p_first <= part < p_first + nparts
            written[part] = written.get(part, 0) + 1
            if nparts <= SINGLE_MAX:
                t = tickets.get(eh, 0)
                tickets[eh] = t + 1
                if t == nparts - 1:
                    merges[eh] = merges.get(eh, 0) + 1
                return
            gs = group_size(nparts)
            g = (part - p_first) // gs
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
            s = seg_of[u]
            if u == ub or u == seg_start[s]:
                if u != ub:
                    flush(seg)
                p0, n_p, first, last = segs[s]
                assert first <= gw <= last
                cta = gw // span
                run_lo = max(first, cta * span)
                run_hi = min(last, cta * span + span - 1)
                seg = (s, p0 + (cta - first // span), n_p, run_lo, run_hi - run_lo + 1)
        flush(seg)
    for eh in range(n_seg):
        p0, n_p = segs[eh][0], segs[eh][1]
        if n_p == 1 and segs[eh][2] // span == segs[eh][3] // span:
            assert direct.get(eh) == 1
        else:
            assert merges.get(eh) == 1
            for p in range(p0, p0 + n_p):
                assert written.get(p) == 1
            for g in range(n_groups[eh]):
                assert group_merges.get((eh, g)) == 1


@pytest.mark.parametrize("npages", [[3, 1], [1] * 4, [1] * 300, [3, 19, 63], [2048],
                                    [1, 1000, 1, 1000], [40], [33, 2048], [17] * 16,
                                    [1] * 2000])
def test_plan_partitions_every_segment(plan_dump, npages):
    walk(plan_dump, npages)


def test_plan_random_batches(plan_dump):
    rng = random.Random(0)
    for _ in range(40):
        walk(plan_dump, [rng.randint(1, 1025) for _ in range(rng.randint(1, 64))],
             G=rng.choice([1, 2, 4, 8]), w_full=rng.choice([148 * WPC, 37, 6]))


def test_shares_balance_segment_switches():
    # 16 slots of 256-4096 positions: the shares that move between
    # segments hold fewer units, and every share costs about the same
    rng = random.Random(2000)
    npages = [rng.randint(256, 4096) // 16 + 1 for _ in range(16)]
    ref = restate(npages, 8, 148 * WPC)
    starts, U = ref["starts"], ref["U"]
    sizes = [starts[k + 1] - starts[k] for k in range(ref["shares"])]
    assert ref["shares"] <= 148 * WPC
    assert max(sizes) == ref["B"] // UNIT
    assert min(sizes[:-1]) >= max(sizes) - LEAVE_SHARED // UNIT - 1
    assert sum(sizes) == U


def test_cta_merge_rule():
    # long segments (one request near the context limit) merge per CTA;
    # many short ones (16 slots) keep one partial per warp
    assert restate([2048], 8, 148 * WPC)["cta_merge"]
    assert restate([2048], 1, 148 * WPC)["cta_merge"]
    assert not restate([100] * 16, 8, 148 * WPC)["cta_merge"]
    assert not restate([600] * 32, 8, 148 * WPC)["cta_merge"]


def raw_lines(plan_dump, text):
    return subprocess.run([str(plan_dump.exe)], input=text, capture_output=True, text=True,
                          check=True, timeout=60).stdout.splitlines()


@pytest.mark.parametrize("C,G,pos", [(16, 8, 32760), (8, 8, 1040), (8, 8, 1023), (2, 8, 300),
                                     (16, 1, 5000), (4, 2, 16 * 32 - 1)])
def test_cluster_plan_covers_each_head_with_one_cluster(plan_dump, C, G, pos):
    out = raw_lines(plan_dump, f"cluster {C} {G} {pos}\n")
    P = pos // 16 + 1
    W = G * C * WPC
    shares, budget, cta, n_parts, n_groups, combine = map(int, out[0].split()[1:])
    assert (cta, combine, n_groups, n_parts, shares) == (1, 0, 0, G * C, W)
    starts = list(map(int, out[1].split()[1:]))
    assert len(starts) == W + 1 and starts[-1] == P * G
    segs = [tuple(map(int, out[2 + h].split()[1:])) for h in range(G)]
    for h in range(G):
        # cluster h = CTAs [h C, (h + 1) C): its warps hold head h's pages, in order
        assert segs[h] == (h * C, C, h * C * WPC, (h + 1) * C * WPC - 1)
        sizes = [starts[k + 1] - starts[k] for k in range(h * C * WPC, (h + 1) * C * WPC)]
        assert starts[h * C * WPC] == h * P and sum(sizes) == P
        assert min(sizes) >= 1 and max(sizes) - min(sizes) <= 1
    warps = list(map(int, out[3 + G].split()[1:]))
    triples = [tuple(warps[k:k + 3]) for k in range(0, len(warps), 3)]
    assert len(triples) == W
    for k, (e, h, i) in enumerate(triples):
        assert (e, h, i) == (0, k // (C * WPC), starts[k] - (k // (C * WPC)) * P)


def test_cluster_choice(plan_dump):
    # fit = clusters of 2, 4, 8, 16 CTAs resident at once (B200: one CTA per SM)
    cases = [
        ((1, 8, 2048, 1184, 74, 37, 18, 8), 16),  # one request near 32k: 8 x 16 CTAs
        ((1, 8, 2048, 1184, 74, 37, 18, 7), 0),   # 16-CTA clusters in two waves: stream-K plan
        ((1, 8, 66, 1184, 74, 37, 18, 8), 8),     # the batch-1 step at 1,040 positions: 8 x 8
        ((1, 8, 63, 1184, 74, 37, 18, 8), 0),     # 63 pages: 4-CTA clusters would use 256 of
                                                  # the 504 warps the stream-K plan uses
        ((1, 4, 2048, 1184, 74, 37, 18, 8), 0),   # 64 CTAs for 4 heads: under 3/4 of the grid
        ((2, 8, 2048, 1184, 74, 37, 18, 8), 0),   # two requests: stream-K plan
        ((1, 8, 10, 1184, 74, 37, 18, 8), 0),     # short: one partial per warp, no CTA merge
    ]
    text = "".join("choose " + " ".join(map(str, a)) + "\n" for a, _ in cases)
    got = [int(line.split()[1]) for line in raw_lines(plan_dump, text)]
    assert got == [want for _, want in cases]
