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
// warp_of(a) .. warp_of(a + np - 1), one partial result each.
//
// Device descriptor (int32 words, uploaded in one copy):
//   pos[n] ntok[n] npages[n] page_off[n+1] unit_off[n+1] part_off[n*G+1]
//   warp_entry[W] pages[total_pages]
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

inline size_t plan_words(int64_t n, int64_t G, int64_t total_pages, int64_t W) {
    return static_cast<size_t>(3 * n + 2 * (n + 1) + (n * G + 1) + W + total_pages);
}

struct PlanSummary {
    int64_t total_pages = 0;
    int64_t total_units = 0;
    int32_t n_parts = 0;
};

// Fills `w` (plan_words(...) words).  page_lists[e] points at slot e's page
// ids, at least pos[e] / 16 + 1 of them.
inline PlanSummary build_plan(int32_t *w, int32_t n, int32_t G, const int32_t *pos_in,
                              const int32_t *const *page_lists, int64_t total_pages, int32_t W) {
    PlanSummary s;
    s.total_pages = total_pages;
    s.total_units = total_pages * G;
    const int64_t U = s.total_units;
    int32_t *pos = w;
    int32_t *ntok = pos + n;
    int32_t *npg = ntok + n;
    int32_t *page_off = npg + n;
    int32_t *unit_off = page_off + (n + 1);
    int32_t *part_off = unit_off + (n + 1);
    int32_t *warp_entry = part_off + (n * G + 1);
    int32_t *pages = warp_entry + W;
    page_off[0] = unit_off[0] = part_off[0] = 0;
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
            const int64_t parts = plan_warp_of(a + np - 1, U, W) - plan_warp_of(a, U, W) + 1;
            part_off[e * G + h + 1] = part_off[e * G + h] + static_cast<int32_t>(parts);
        }
    }
    int32_t e = 0;
    for (int32_t k = 0; k < W; ++k) {
        const int64_t ub = static_cast<int64_t>(k) * U / W;
        while (e + 1 < n && unit_off[e + 1] <= ub) {
            ++e;
        }
        warp_entry[k] = e;
    }
    s.n_parts = part_off[n * G];
    return s;
}

// Device view of an uploaded plan.
inline BatchView bind_plan(const int32_t *d, int32_t n, int32_t G, const PlanSummary &s,
                           int32_t W) {
    BatchView b;
    b.pos = d;
    b.ntok = d + n;
    b.npages = d + 2 * n;
    b.page_off = d + 3 * n;
    b.unit_off = b.page_off + (n + 1);
    b.part_off = b.unit_off + (n + 1);
    b.warp_entry = b.part_off + (n * G + 1);
    b.pages = b.warp_entry + W;
    b.n = n;
    b.total_units = static_cast<int32_t>(s.total_units);
    b.n_warps = W;
    b.n_parts = s.n_parts;
    return b;
}

}  // namespace hkv
