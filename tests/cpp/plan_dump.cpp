// plan_dump.cpp -- prints the decode-attention plan (hkv_plan.h) of batches
// read from stdin, for tests/test_plan_invariants.py.
//
// Input, one batch per line:  G W pos_0 pos_1 ... pos_{n-1}
//   or  cluster C G pos          (the cluster plan of one request, W = 8 G C)
//   or  choose n G pages max_warps fit_2 fit_4 fit_8 fit_16
//                                (prints "cluster <plan_cluster(...)>")
// Output, per batch:
//   plan <shares> <budget> <cta_merge> <n_parts> <n_groups> <combine>
//   starts <u_begin of warp 0 .. W-1> <U>
//   seg <first partial> <partials> <first warp> <last warp>   (one line per segment)
//   part2 <part2_off[0 .. n*G]>
//   warps <entry> <kv head> <page index> per warp with a non-empty share
#include <cstdio>
#include <iostream>
#include <sstream>
#include <string>
#include <vector>

#include "hkv_plan.h"

int main() {
    std::string line;
    while (std::getline(std::cin, line)) {
        std::istringstream in(line);
        int32_t G = 0, W = 0, C = 0;
        if (line.rfind("choose", 0) == 0) {
            std::string word;
            int32_t n = 0;
            long long pages = 0, max_warps = 0;
            int32_t fit[5] = {0, 0, 0, 0, 0};
            in >> word >> n >> G >> pages >> max_warps >> fit[1] >> fit[2] >> fit[3] >> fit[4];
            std::printf("cluster %d\n", hkv::plan_cluster(n, G, pages, max_warps, fit));
            continue;
        }
        if (line.rfind("cluster", 0) == 0) {
            std::string word;
            in >> word >> C >> G;
            W = G * C * hkv::kAttnWarps;
        } else if (!(in >> G >> W)) {
            continue;
        }
        std::vector<int32_t> pos;
        int32_t p = 0;
        while (in >> p) {
            pos.push_back(p);
        }
        const int32_t n = static_cast<int32_t>(pos.size());
        std::vector<std::vector<int32_t>> lists(static_cast<size_t>(n));
        std::vector<const int32_t *> ptrs(static_cast<size_t>(n));
        int64_t total_pages = 0;
        for (int32_t e = 0; e < n; ++e) {
            const int32_t np = pos[e] / hkv::kPageTokens + 1;
            for (int32_t i = 0; i < np; ++i) {
                lists[e].push_back(static_cast<int32_t>(total_pages + i));
            }
            ptrs[e] = lists[e].data();
            total_pages += np;
        }
        std::vector<int32_t> w(hkv::plan_words(n, G, total_pages, W));
        const hkv::PlanSummary s =
            C > 0 ? hkv::build_cluster_plan(w.data(), G, pos[0], ptrs[0], C)
                  : hkv::build_plan(w.data(), n, G, pos.data(), ptrs.data(), total_pages, W);
        std::printf("plan %d %lld %d %d %d %d\n", s.shares, static_cast<long long>(s.budget),
                    s.cta_merge ? 1 : 0, s.n_parts, s.n_groups, s.combine ? 1 : 0);
        std::printf("starts");
        for (int32_t k = 0; k < W; ++k) {
            std::printf(" %d", w[hkv::kWarpStartWords * k + 8]);
        }
        std::printf(" %lld\n", static_cast<long long>(s.total_units));
        const int32_t *seg = w.data() + hkv::kWarpStartWords * W;
        for (int64_t sg = 0; sg < static_cast<int64_t>(n) * G; ++sg) {
            std::printf("seg %d %d %d %d\n", seg[4 * sg], seg[4 * sg + 1], seg[4 * sg + 2], seg[4 * sg + 3]);
        }
        const int32_t *part2 = seg + hkv::kSegWords * n * G + 3 * n + 2 * (n + 1);
        std::printf("part2");
        for (int64_t i = 0; i <= static_cast<int64_t>(n) * G; ++i) {
            std::printf(" %d", part2[i]);
        }
        std::printf("\nwarps");
        for (int32_t k = 0; k < W; ++k) {
            const int32_t *ws = w.data() + hkv::kWarpStartWords * k;
            if (ws[8] < ws[9]) {
                std::printf(" %d %d %d", ws[0], ws[1], ws[2]);
            }
        }
        std::printf("\n");
    }
    return 0;
}
