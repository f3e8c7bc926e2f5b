// hkv_plan.h -- host-side plan of one decode-attention launch (header only).
//
// A batch of n slots attending pos[e] + 1 rows each is cut into units (one
// unit = one 16-row page of one KV head, 8 KiB of K and V).  Units are
// ordered (entry, KV head, page); the range [0, U) is split into W equal
// shares, one per warp, W = min(U, warps of a full grid) so that no share is
// empty:
//     share(w) = [floor(w U / W), floor((w + 1) U / W))
// and the warp holding unit a is warp_of(a) = ceil((a + 1) W / U) - 1.
// Each (entry, KV head) segment [a, a + np) is covered by warps
// warp_of(a) .. warp_of(a + np - 1), one partial result each -- or, when
// segments are long (plan_cta_merge: at least two CTAs' worth of warps per
// segment on average), the warps of one CTA (kAttnWarps consecutive warps)
// merge theirs in shared memory first and the segment has one partial per CTA
// it spans.
//
// A segment with more than kMergeSingleMax partials is merged in two levels:
// groups of merge_group_size() partials are merged by the last warp of each
// group into one "group partial", and the last group merges those.
// part2_off gives each such segment's first group partial (stored after the
// n_parts partials) and its first group counter (after the n*G segment
// counters).
//
// Device descriptor (int32 words, uploaded in one copy):
//   warp_start[W][8]  per warp {entry, kv head, page index, pages of the entry}
//                     {page_off[entry], physical pages of its first 3 units}
//                     (first, so each record is 16-byte aligned)
//   pos[n] ntok[n] npages[n] page_off[n+1] unit_off[n+1] part_off[n*G+1]
//   part2_off[n*G+1] pages[total_pages]
#pragma once

#include <stdint.h>

#include <cstring>

#include "hkv_internal.h"

namespace hkv {

inline int64_t plan_warp_of(int64_t a, int64_t U, int64_t W) { return ((a + 1) * W + U - 1) / U - 1; }

// Warps to share U units among: every share must hold at least one unit (a
// segment's partial count is the number of warps its range touches, so an
// empty share in the middle would be counted but never arrive).
inline int32_t plan_warps(int64_t total_units, int64_t max_warps) {
    return static_cast<int32_t>(total_units < max_warps ? total_units : max_warps);
}

// CTA-level pre-merge pays when a segment spans many warps (a few long
// requests); with many short segments it only adds shared-memory traffic
// and footprint.
inline bool plan_cta_merge(int64_t n_segments, int64_t W) { return W >= 2 * kAttnWarps * n_segments; }

constexpr int kWarpStartWords = 8;

inline size_t plan_words(int64_t n, int64_t G, int64_t total_pages, int64_t W) {
    return static_cast<size_t>(kWarpStartWords * W + 3 * n + 2 * (n + 1) + 2 * (n * G + 1) +
                               total_pages);
}

struct PlanSummary {
    int64_t total_pages = 0;
    int64_t total_units = 0;
    int32_t n_parts = 0;   // level-1 partials
    int32_t n_groups = 0;  // group partials (and group counters)
    bool cta_merge = false;
};

// Fills `w` (plan_words(...) words, 16-byte aligned).  page_lists[e] points
// at slot e's page ids, at least pos[e] / 16 + 1 of them.
inline PlanSummary build_plan(int32_t *w, int32_t n, int32_t G, const int32_t *pos_in,
                              const int32_t *const *page_lists, int64_t total_pages, int32_t W) {
    PlanSummary s;
    s.total_pages = total_pages;
    s.total_units = total_pages * G;
    s.cta_merge = plan_cta_merge(static_cast<int64_t>(n) * G, W);
    const int64_t U = s.total_units;
    const int64_t span = s.cta_merge ? kAttnWarps : 1;  // warps per partial
    int32_t *warp_start = w;
    int32_t *pos = warp_start + kWarpStartWords * W;
    int32_t *ntok = pos + n;
    int32_t *npg = ntok + n;
    int32_t *page_off = npg + n;
    int32_t *unit_off = page_off + (n + 1);
    int32_t *part_off = unit_off + (n + 1);
    int32_t *part2_off = part_off + (n * G + 1);
    int32_t *pages = part2_off + (n * G + 1);
    page_off[0] = unit_off[0] = part_off[0] = part2_off[0] = 0;
    for (int32_t e = 0; e < n; ++e) {
        const int32_t np = pos_in[e] / kPageTokens + 1;
        pos[e] = pos_in[e];
        ntok[e] = pos_in[e] + 1;
        npg[e] = np;
        std::memcpy(pages + page_off[e], page_lists[e], static_cast<size_t>(np) * sizeof(int32_t));
        page_off[e + 1] = page_off[e] + np;
        unit_off[e + 1] = unit_off[e] + np * G;
        for (int32_t h = 0; h < G; ++h) {
            const int64_t a = unit_off[e] + static_cast<int64_t>(h) * np;
            const int64_t parts = plan_warp_of(a + np - 1, U, W) / span - plan_warp_of(a, U, W) / span + 1;
            part_off[e * G + h + 1] = part_off[e * G + h] + static_cast<int32_t>(parts);
            part2_off[e * G + h + 1] =
                part2_off[e * G + h] + merge_groups(static_cast<int32_t>(parts));
        }
    }
    int32_t e = 0;
    for (int32_t k = 0; k < W; ++k) {
        const int64_t ub = static_cast<int64_t>(k) * U / W;
        const int64_t ue = static_cast<int64_t>(k + 1) * U / W;
        while (e + 1 < n && unit_off[e + 1] <= ub) {
            ++e;
        }
        int32_t *ws = warp_start + kWarpStartWords * k;
        const int32_t np = npg[e];
        const int32_t rem = static_cast<int32_t>(ub - unit_off[e]);
        ws[0] = e;
        ws[1] = rem / np;
        ws[2] = rem % np;
        ws[3] = np;
        ws[4] = page_off[e];
        // physical pages of the share's first three units
        int32_t ce = e, ch = ws[1], ci = ws[2];
        for (int j = 0; j < 3; ++j) {
            if (ub + j < ue) {
                ws[5 + j] = pages[page_off[ce] + ci];
                if (++ci == npg[ce]) {
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
    s.n_parts = part_off[n * G];
    s.n_groups = part2_off[n * G];
    return s;
}

// Device view of an uploaded plan.
inline BatchView bind_plan(const int32_t *d, int32_t n, int32_t G, const PlanSummary &s,
                           int32_t W) {
    BatchView b;
    b.warp_start = reinterpret_cast<const int4 *>(d);
    b.pos = d + kWarpStartWords * W;
    b.ntok = b.pos + n;
    b.npages = b.ntok + n;
    b.page_off = b.npages + n;
    b.unit_off = b.page_off + (n + 1);
    b.part_off = b.unit_off + (n + 1);
    b.part2_off = b.part_off + (n * G + 1);
    b.pages = b.part2_off + (n * G + 1);
    b.n = n;
    b.total_units = static_cast<int32_t>(s.total_units);
    b.n_warps = W;
    b.n_parts = s.n_parts;
    b.cta_merge = s.cta_merge ? 1 : 0;
    return b;
}

}  // namespace hkv
