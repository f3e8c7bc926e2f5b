// hkv_plan.h -- host-side plan of one decode-attention launch (header only).
//
// A batch of n slots attending pos[e] + 1 rows each is cut into units (one
// unit = one 16-row page of one KV head, 8 KiB of K and V).  Units are
// ordered (entry, KV head, page) and the range [0, U) is cut into at most W
// consecutive shares, one per warp, W = min(U, warps of a full grid).
// Shares are balanced by cost, not by unit count: a unit costs kCostUnit,
// and a warp that moves on to another (entry, KV head) segment inside its
// share pays for publishing the segment it leaves and staging the next
// one's queries (kCostLeaveWhole when it held that segment from its first
// page, kCostLeaveShared when an earlier warp holds part of it, since then
// a partial result is published and a merge ticket taken).  The smallest
// per-share budget B for which a greedy cut needs no more than W shares is
// found by bisection; warps past the last share have empty shares and no
// segment counts them.
// Each (entry, KV head) segment is covered by warps first .. last, one
// partial result each -- or, when segments are long (plan_cta_merge: at
// least two CTAs' worth of warps per segment on average), the warps of one
// CTA (kAttnWarps consecutive warps) merge theirs in shared memory first and
// the segment has one partial per CTA it spans.
//
// One long request (plan_cluster): each KV head's segment gets a cluster of C
// thread-block CTAs (8C warps, the pages split evenly), the warps of a CTA
// merge in shared memory, and the C CTA partials meet in the first CTA's
// shared memory (distributed shared memory), which writes the output: no
// combine launch and no global ticket.
//
// A segment with more than kMergeSingleMax partials is merged in two levels:
// groups of merge_group_size() partials are merged by the last warp of each
// group into one "group partial", and the last group merges those.
// part2_off gives each such segment's first group partial (stored after the
// n_parts partials) and its first group counter (after the n*G segment
// counters).
//
// Device descriptor (int32 words, uploaded in one copy; the 16-byte records
// first, so each stays aligned):
//   warp_start[W][12] per warp {entry, kv head, page index, pages of the entry}
//                     {page_off[entry], physical pages of its first 3 units}
//                     {first unit, end unit, 0, 0}
//   seg[n*G][4]       per segment {first partial, partials, first warp, last warp}
//   pos[n] ntok[n] npages[n] page_off[n+1] unit_off[n+1] part2_off[n*G+1]
//   pages[total_pages]
#pragma once

#include <stdint.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "hkv_internal.h"

namespace hkv {

// Warps to share U units among (at most one per unit).
inline int32_t plan_warps(int64_t total_units, int64_t max_warps) {
    return static_cast<int32_t>(total_units < max_warps ? total_units : max_warps);
}

// CTA-level pre-merge pays when a segment spans many warps (a few long
// requests); with many short segments it only adds shared-memory traffic
// and footprint.
inline bool plan_cta_merge(int64_t n_segments, int64_t W) { return W >= 2 * kAttnWarps * n_segments; }

// Where the split partials are merged.  Inside the attention launch, by the
// last warp (or CTA) of each segment to finish, behind a fence and an atomic
// ticket -- best when segments are short (many segments, a few warp partials
// each: the merges of early segments overlap the other warps' work), and for
// one segment over the whole grid (its groups merge as they complete).  Or
// by a combine launch after the attention grid, one CTA per (segment, query
// head) -- best for CTA-merged segments of at most kCombineMaxParts partials
// (a few long requests: one request near 32k positions +11%, the batch-1
// backbone step +7%, measured against the in-launch merge), whose in-launch
// merge would sit in the tail behind fences, tickets and a second level.
// The combine launch for warp-partial plans too lost: 16 slots of 256-4096
// positions -8%, 32 slots of 2k-16k -2.5%.  So did the combine launch for
// segments of up to 256 CTA partials (one request near 32k positions split
// by KV head, one or two KV heads per GPU: -22% / -12%), whose four or eight
// combine CTAs read every partial with little parallelism, and plans of at
// least 4 units per warp (-1.5% on one KV head of that request, -6% on the
// batch-1 backbone step).
constexpr int32_t kCombineMaxParts = 32;
inline bool plan_combine(bool cta_merge, int32_t max_parts) {
    return cta_merge && max_parts > 1 && max_parts <= kCombineMaxParts;
}

// Share costs in sixteenths of a unit, from per-warp timestamps of the
// attention kernel on B200 (16 slots of 256-4096 positions): a unit takes
// about 0.95 us of a warp's time, leaving a segment held whole about 1 us
// (output stores, next queries), leaving a shared one about 3.3 us (partial
// stores, fence, ticket round trip, next queries).
// Raised from 16 / 56 after a same-box sweep (16/40, 16/56, 16/80, 16/104, 32/80):
// 32/80 was best on batched and churn by 0.2-0.4% and equal on the scale-out shard.
constexpr int64_t kCostUnit = 16;
constexpr int64_t kCostLeaveWhole = 32;
constexpr int64_t kCostLeaveShared = 80;

// Greedy cut of the segments (segment s has npg[s / G] units) into shares of
// cost at most B (B >= kCostUnit, so every share holds a unit).  Returns the
// number of shares, or max_shares + 1 as soon as more are needed; writes each
// share's first unit to starts[] when starts is not null.
inline int64_t plan_cut(const int32_t *npg, int32_t G, int64_t S, int64_t B, int64_t max_shares,
                        int32_t *starts) {
    int64_t k = 0, s = 0, i = 0, u = 0;  // shares, segment, unit within it, flat unit
    while (s < S) {
        if (k == max_shares) {
            return max_shares + 1;
        }
        if (starts != nullptr) {
            starts[k] = static_cast<int32_t>(u);
        }
        ++k;
        int64_t budget = B;
        bool from_first_page = i == 0;
        for (;;) {
            const int64_t np = npg[s / G];
            const int64_t take = std::min(np - i, budget / kCostUnit);
            i += take;
            u += take;
            budget -= take * kCostUnit;
            if (i < np) {
                break;  // the share ends inside this segment
            }
            ++s;
            i = 0;
            if (s == S) {
                break;
            }
            const int64_t leave = from_first_page ? kCostLeaveWhole : kCostLeaveShared;
            if (budget - leave < kCostUnit) {
                break;  // the next segment opens the next share
            }
            budget -= leave;
            from_first_page = true;
        }
    }
    return k;
}

constexpr int kWarpStartWords = 12;
constexpr int kSegWords = 4;

inline size_t plan_words(int64_t n, int64_t G, int64_t total_pages, int64_t W) {
    return static_cast<size_t>(kWarpStartWords * W + kSegWords * n * G + 3 * n + 2 * (n + 1) +
                               (n * G + 1) + total_pages);
}

// Thread-block clusters for a batch of one entry (one long request, or the
// batch-1 decode step): the largest C of 16, 8, 4, 2 CTAs per cluster such
// that every KV head's cluster runs at once (fit[i] = clusters of 2^i CTAs
// that can be resident together), every warp gets at least one page, and the
// cluster plan's G * C * kAttnWarps warps are at least 3/4 of the warps the
// stream-K plan would use (fewer SMs would cost bandwidth); and only where
// that plan would pre-merge per CTA (long segments).  0: no clusters (the
// stream-K plan).
inline int32_t plan_cluster(int32_t n, int32_t G, int64_t npages, int64_t max_warps,
                            const int32_t (&fit)[5]) {
    if (n != 1 || G <= 0) {
        return 0;
    }
    const int64_t w_default = plan_warps(npages * G, max_warps);
    if (!plan_cta_merge(G, w_default)) {
        return 0;
    }
    for (int i = 4; i >= 1; --i) {
        const int64_t C = int64_t{1} << i;
        const int64_t warps = G * C * kAttnWarps;
        if (warps <= max_warps && fit[i] >= G && npages >= C * kAttnWarps && 4 * warps >= 3 * w_default) {
            return static_cast<int32_t>(C);
        }
    }
    return 0;
}

struct PlanSummary {
    int64_t total_pages = 0;
    int64_t total_units = 0;
    int32_t n_parts = 0;   // level-1 partials
    int32_t n_groups = 0;  // group partials (and group counters)
    int32_t shares = 0;    // non-empty shares (<= W)
    int32_t split_segments = 0;  // segments with more than one partial
    int32_t max_parts = 0;       // most partials of one segment
    bool combine = false;        // split partials merged by the combine launch (plan_combine)
    int64_t budget = 0;    // the cost bound B of every share
    bool cta_merge = false;
    int32_t cluster = 0;   // CTAs per cluster (plan_cluster), 0: none
};


// Descriptor arrays inside `w` (the layout at the top of this file).
struct PlanArrays {
    int32_t *warp_start, *seg, *pos, *ntok, *npg, *page_off, *unit_off, *part2_off, *pages;
};

// Lays the arrays out in `w` and fills the per-entry ones (positions, page
// counts, prefix sums, page lists).
inline PlanArrays plan_arrays(int32_t *w, int32_t n, int32_t G, const int32_t *pos_in,
                              const int32_t *const *page_lists, int32_t W) {
    const int64_t S = static_cast<int64_t>(n) * G;
    PlanArrays a;
    a.warp_start = w;
    a.seg = a.warp_start + kWarpStartWords * W;
    a.pos = a.seg + kSegWords * S;
    a.ntok = a.pos + n;
    a.npg = a.ntok + n;
    a.page_off = a.npg + n;
    a.unit_off = a.page_off + (n + 1);
    a.part2_off = a.unit_off + (n + 1);
    a.pages = a.part2_off + (S + 1);
    a.page_off[0] = a.unit_off[0] = a.part2_off[0] = 0;
    for (int32_t e = 0; e < n; ++e) {
        const int32_t np = pos_in[e] / kPageTokens + 1;
        a.pos[e] = pos_in[e];
        a.ntok[e] = pos_in[e] + 1;
        a.npg[e] = np;
        std::memcpy(a.pages + a.page_off[e], page_lists[e], static_cast<size_t>(np) * sizeof(int32_t));
        a.page_off[e + 1] = a.page_off[e] + np;
        a.unit_off[e + 1] = a.unit_off[e] + np * G;
    }
    return a;
}

// The segment and per-warp records of a plan whose shares are known:
// warp k holds units [starts[k], starts[k + 1]), starts[W] = U; span warps
// share one partial.
inline void fill_records(const PlanArrays &a, int32_t n, int32_t G, int32_t W,
                         const int32_t *starts, int64_t span, PlanSummary &s) {
    const int64_t S = static_cast<int64_t>(n) * G;
    // ---- segments: warps first .. last, partials
    int32_t parts = 0;
    int32_t k = 0;  // the share holding unit u
    for (int64_t sg = 0; sg < S; ++sg) {
        const int32_t e = static_cast<int32_t>(sg / G);
        const int64_t u = a.unit_off[e] + (sg % G) * a.npg[e];
        while (starts[k + 1] <= u) {
            ++k;
        }
        int32_t last = k;
        while (starts[last + 1] <= u + a.npg[e] - 1) {
            ++last;
        }
        const int32_t np_parts = static_cast<int32_t>(last / span - k / span + 1);
        int32_t *rec = a.seg + kSegWords * sg;
        rec[0] = parts;
        rec[1] = np_parts;
        rec[2] = k;
        rec[3] = last;
        parts += np_parts;
        s.split_segments += np_parts > 1 ? 1 : 0;
        s.max_parts = std::max(s.max_parts, np_parts);
        a.part2_off[sg + 1] = a.part2_off[sg] + merge_groups(np_parts);
    }

    // ---- per-warp records
    int32_t e = 0;
    for (int32_t kw = 0; kw < W; ++kw) {
        const int64_t ub = starts[kw];
        const int64_t ue = starts[kw + 1];
        int32_t *ws = a.warp_start + kWarpStartWords * kw;
        ws[8] = static_cast<int32_t>(ub);
        ws[9] = static_cast<int32_t>(ue);
        ws[10] = ws[11] = 0;
        if (ub >= ue) {
            for (int j = 0; j < 8; ++j) {
                ws[j] = 0;
            }
            continue;
        }
        while (e + 1 < n && a.unit_off[e + 1] <= ub) {
            ++e;
        }
        const int32_t np = a.npg[e];
        const int32_t rem = static_cast<int32_t>(ub - a.unit_off[e]);
        ws[0] = e;
        ws[1] = rem / np;
        ws[2] = rem % np;
        ws[3] = np;
        ws[4] = a.page_off[e];
        // physical pages of the share's first three units
        int32_t ce = e, ch = ws[1], ci = ws[2];
        for (int j = 0; j < 3; ++j) {
            if (ub + j < ue) {
                ws[5 + j] = a.pages[a.page_off[ce] + ci];
                if (++ci == a.npg[ce]) {
                    ci = 0;
                    if (++ch == G) {
                        ch = 0;
                        ++ce;
                    }
                }
            } else {
                ws[5 + j] = -1;
            }
        }
    }
    s.n_parts = parts;
    s.n_groups = a.part2_off[S];
}

// Fills `w` (plan_words(...) words, 16-byte aligned).  page_lists[e] points
// at slot e's page ids, at least pos[e] / 16 + 1 of them.
inline PlanSummary build_plan(int32_t *w, int32_t n, int32_t G, const int32_t *pos_in,
                              const int32_t *const *page_lists, int64_t total_pages, int32_t W) {
    PlanSummary s;
    s.total_pages = total_pages;
    s.total_units = total_pages * G;
    s.cta_merge = plan_cta_merge(static_cast<int64_t>(n) * G, W);
    const int64_t U = s.total_units;
    const int64_t S = static_cast<int64_t>(n) * G;
    const PlanArrays a = plan_arrays(w, n, G, pos_in, page_lists, W);

    // ---- shares: the smallest budget that fits W warps (bisection)
    const int64_t per = (U + W - 1) / W;
    int64_t bad = kCostUnit * per - 1;  // W shares of fewer than per units cannot hold U
    int64_t good = kCostUnit * per + kCostLeaveShared * (S + 1);
    while (plan_cut(a.npg, G, S, good, W, nullptr) > W) {
        good *= 2;
    }
    while (good - bad > 1) {
        const int64_t mid = bad + (good - bad) / 2;
        if (plan_cut(a.npg, G, S, mid, W, nullptr) > W) {
            bad = mid;
        } else {
            good = mid;
        }
    }
    s.budget = good;
    std::vector<int32_t> starts(static_cast<size_t>(W) + 1);
    s.shares = static_cast<int32_t>(plan_cut(a.npg, G, S, good, W, starts.data()));
    for (int64_t k = s.shares; k <= W; ++k) {
        starts[k] = static_cast<int32_t>(U);
    }
    fill_records(a, n, G, W, starts.data(), s.cta_merge ? kAttnWarps : 1, s);
    s.combine = plan_combine(s.cta_merge, s.max_parts);
    return s;
}

// The cluster plan of a one-entry batch (plan_cluster returned C): KV head h
// is segment h and cluster h, CTAs [h C, (h + 1) C), warps [8 h C, 8 (h + 1) C);
// warp j of a segment of P pages holds pages [j P / 8C, (j + 1) P / 8C)
// (at least one, as P >= 8C).  `w` holds plan_words(1, G, P, 8 G C) words.
inline PlanSummary build_cluster_plan(int32_t *w, int32_t G, int32_t pos0,
                                      const int32_t *page_list, int32_t C) {
    const int32_t P = pos0 / kPageTokens + 1;
    const int32_t per_seg = C * kAttnWarps;
    const int32_t W = G * per_seg;
    PlanSummary s;
    s.total_pages = P;
    s.total_units = static_cast<int64_t>(P) * G;
    s.cta_merge = true;
    s.cluster = C;
    const PlanArrays a = plan_arrays(w, 1, G, &pos0, &page_list, W);
    std::vector<int32_t> starts(static_cast<size_t>(W) + 1);
    for (int32_t h = 0; h < G; ++h) {
        for (int32_t j = 0; j < per_seg; ++j) {
            starts[h * per_seg + j] = static_cast<int32_t>(static_cast<int64_t>(h) * P +
                                                           static_cast<int64_t>(j) * P / per_seg);
        }
    }
    starts[W] = static_cast<int32_t>(s.total_units);
    s.shares = W;
    fill_records(a, 1, G, W, starts.data(), kAttnWarps, s);
    s.combine = false;
    return s;
}

// Device view of an uploaded plan.
inline BatchView bind_plan(const int32_t *d, int32_t n, int32_t G, const PlanSummary &s,
                           int32_t W) {
    BatchView b;
    b.warp_start = reinterpret_cast<const int4 *>(d);
    b.seg = reinterpret_cast<const int4 *>(d + kWarpStartWords * W);
    b.pos = d + kWarpStartWords * W + kSegWords * n * G;
    b.ntok = b.pos + n;
    b.npages = b.ntok + n;
    b.page_off = b.npages + n;
    b.unit_off = b.page_off + (n + 1);
    b.part2_off = b.unit_off + (n + 1);
    b.pages = b.part2_off + (n * G + 1);
    b.n = n;
    b.total_units = static_cast<int32_t>(s.total_units);
    b.n_warps = W;
    b.n_parts = s.n_parts;
    b.cta_merge = s.cta_merge ? 1 : 0;
    b.split_segments = s.split_segments;
    b.combine = s.combine ? 1 : 0;
    b.cluster = s.cluster;
    return b;
}

}  // namespace hkv
