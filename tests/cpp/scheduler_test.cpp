// Exercises include/hkv_scheduler.hpp on a GPU with a 2-layer Q4_K backbone:
//  * requests of different prompt lengths and frame counts are admitted (one
//    waits in the queue), batched per step and retired; every request gets
//    exactly its frames, all slots are released, and the frames equal those
//    of running the requests one at a time; some prompt steps mix requests
//    at their last prompt token with requests inside their prompts;
//  * cancellation (the reference's throw_if_cancelled): a request whose flag
//    is set mid-run ends between steps with its frames so far, its pages go
//    back to the pool at once, and the other requests' frames are unchanged;
//    a request whose deadline has passed never starts;
//  * the low-margin window refresh: forced on every frame (a margin no
//    logits reach), the slot is truncated by its last two generated rows and
//    they are decoded again; run alone, the request's frames and its whole
//    cache (every layer, gathered before release) equal bit for bit those of
//    the same request without refresh, and in a batch the other requests'
//    frames and caches are unchanged.
#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <functional>
#include <map>
#include <vector>

#include "backbone_fixture.hpp"
#include "hkv_scheduler.hpp"

#define EXPECT(c)                                                                \
    do {                                                                         \
        if (!(c)) {                                                              \
            std::fprintf(stderr, "FAILED %s:%d: %s\n", __FILE__, __LINE__, #c);  \
            return 1;                                                            \
        }                                                                        \
    } while (0)

namespace {

using fixture::dmalloc;
using fixture::norm;
using fixture::q4k;

using Sched = hkv_pipeline::StepScheduler;
using Frames = std::vector<Sched::Frame>;
using Cache = std::vector<uint16_t>;  // every layer's K then V rows [0, used)

struct RunResult {
    std::vector<Frames> frames;
    std::vector<hkv_pipeline::RequestStatus> status;
    std::vector<int32_t> refreshes;
    std::map<int64_t, Cache> caches;  // per request, gathered at retirement
    size_t max_live = 0;
    int64_t mixed_prompt_steps = 0;
};

// Runs `reqs` through a scheduler of max_batch places; `between(step, sched,
// engine)` is called after every step.
RunResult run(const hkv_backbone_weights &w, const std::vector<hkv_pipeline::GenerateRequest> &reqs,
              int32_t max_batch, const std::function<void(int, Sched &, hkv_engine *)> &between = {}) {
    hkv_config cfg;
    hkv_config_default(&cfg);
    cfg.n_layers = 2;
    cfg.n_pages = 64;
    cfg.max_slots = 4;
    cfg.device = 0;
    hkv_pipeline::PagedKvRuntime rt(cfg);
    hkv_backbone *bb = nullptr;
    hkv_pipeline::check(nullptr, hkv_backbone_create(rt.engine(), &w, 4, &bb), "hkv_backbone_create");
    RunResult out;
    {
        Sched sched(rt, bb, max_batch, nullptr);
        sched.on_retire = [&](int64_t id, int32_t slot) {
            int64_t used = 0;
            hkv_slot_len(rt.engine(), slot, &used);
            const size_t row = 8 * 128;
            Cache c;
            if (used > 0) {
                uint16_t *dk = static_cast<uint16_t *>(dmalloc(used * row * 2));
                uint16_t *dv = static_cast<uint16_t *>(dmalloc(used * row * 2));
                for (int layer = 0; layer < cfg.n_layers; ++layer) {
                    hkv_pipeline::check(rt.engine(), hkv_gather(rt.engine(), slot, layer, 0, used, dk, dv, nullptr),
                                        "hkv_gather");
                    const size_t at = c.size();
                    c.resize(at + 2 * used * row);
                    cudaMemcpy(c.data() + at, dk, used * row * 2, cudaMemcpyDeviceToHost);
                    cudaMemcpy(c.data() + at + used * row, dv, used * row * 2, cudaMemcpyDeviceToHost);
                }
            }
            out.caches[id] = std::move(c);
        };
        std::vector<int64_t> ids;
        for (const auto &r : reqs) ids.push_back(sched.submit(r));
        for (int it = 0; it < 1000 && sched.step() > 0; ++it) {
            if (sched.live() > out.max_live) out.max_live = sched.live();
            if (between) between(it, sched, rt.engine());
        }
        for (int64_t id : ids) {
            if (!sched.finished(id)) throw std::runtime_error("request did not end");
            out.frames.push_back(sched.frames(id));
            out.status.push_back(sched.status(id));
            out.refreshes.push_back(sched.refreshes(id));
        }
        out.mixed_prompt_steps = sched.mixed_prompt_steps();
        hkv_pool_stats st{};
        hkv_pool_stats_get(rt.engine(), &st);
        if (st.live_slots != 0 || st.reserved != 0 || st.free_pages != cfg.n_pages) {
            throw std::runtime_error("slots not released");
        }
    }
    hkv_backbone_destroy(bb);
    return out;
}

int count_differences(const Frames &a, const Frames &b) {
    if (a.size() != b.size()) return 1 << 20;
    int d = 0;
    for (size_t f = 0; f < a.size(); ++f) {
        for (int c = 0; c < 8; ++c) d += a[f][c] != b[f][c];
    }
    return d;
}

}  // namespace

int main() {
    using hkv_pipeline::RequestStatus;
    const int L = 2, vocab = 512;
    std::vector<hkv_backbone_layer> layers(L);
    for (int l = 0; l < L; ++l) {
        layers[l] = {q4k(4096, 2560), q4k(1024, 2560), q4k(1024, 2560), q4k(2560, 4096),
                     q4k(9728, 2560), q4k(9728, 2560), q4k(2560, 9728),
                     norm(2560), norm(2560), norm(128), norm(128)};
    }
    const hkv_backbone_weights w = {2560, 9728, vocab, 8, 1026, 1e-6f, layers.data(),
                                    q4k(vocab, 2560), q4k(8 * 1026, 2560), norm(2560), q4k(8 * 1026, 2560)};
    std::vector<hkv_pipeline::GenerateRequest> reqs(4);
    const int prompt_len[4] = {5, 9, 3, 6};
    const int frames[4] = {4, 2, 6, 3};
    for (int r = 0; r < 4; ++r) {
        for (int t = 0; t < prompt_len[r]; ++t) reqs[r].prompt_ids.push_back((37 * r + 11 * t) % vocab);
        reqs[r].max_frames = frames[r];
    }

    // ---- batching against one-at-a-time
    const RunResult batched = run(w, reqs, 3);  // the 4th request queues
    const RunResult solo = run(w, reqs, 1);
    EXPECT(batched.max_live == 3 && solo.max_live == 1);
    EXPECT(batched.mixed_prompt_steps > 0);
    for (int r = 0; r < 4; ++r) {
        EXPECT(batched.status[r] == RequestStatus::kDone);
        EXPECT(static_cast<int>(batched.frames[r].size()) == frames[r]);
        EXPECT(static_cast<int>(solo.frames[r].size()) == frames[r]);
        for (const auto &f : batched.frames[r]) {
            for (int c = 0; c < 8; ++c) EXPECT(f[c] >= 0 && f[c] < 1026);
        }
        // batched and one-at-a-time runs differ only in float summation order
        EXPECT(count_differences(batched.frames[r], solo.frames[r]) == 0);
    }

    // ---- cancellation mid-run and a deadline already passed
    {
        std::vector<hkv_pipeline::GenerateRequest> rq = reqs;
        volatile int cancel_flag = 0;
        rq[2].cancel = &cancel_flag;  // 3-token prompt, 6 frames: cancelled after its 2nd frame
        rq[3].deadline = std::chrono::steady_clock::now() - std::chrono::seconds(1);
        int64_t free_before = -1;
        bool cancelled_seen = false, freed_at_cancel = false;
        const RunResult res = run(w, rq, 3, [&](int step, Sched &sched, hkv_engine *eng) {
            hkv_pool_stats st{};
            hkv_pool_stats_get(eng, &st);
            if (cancel_flag != 0 && !cancelled_seen && sched.status(2) == RequestStatus::kCancelled) {
                cancelled_seen = true;
                freed_at_cancel = st.free_pages > free_before;
            }
            if (step == 4) {  // prompt (3 steps) + 2 frames
                cancel_flag = 1;
                free_before = st.free_pages;
            }
        });
        EXPECT(cancelled_seen && freed_at_cancel);
        EXPECT(res.status[2] == RequestStatus::kCancelled);
        EXPECT(res.frames[2].size() == 2);
        EXPECT(res.status[3] == RequestStatus::kTimedOut && res.frames[3].empty());
        EXPECT(res.status[0] == RequestStatus::kDone && res.status[1] == RequestStatus::kDone);
        // the others' frames do not change (greedy codes)
        EXPECT(count_differences(res.frames[0], batched.frames[0]) == 0);
        EXPECT(count_differences(res.frames[1], batched.frames[1]) == 0);
        for (int f = 0; f < 2; ++f) {
            for (int c = 0; c < 8; ++c) EXPECT(res.frames[2][f][c] == batched.frames[2][f][c]);
        }
    }

    // ---- low-margin window refresh, forced on every frame
    {
        std::vector<hkv_pipeline::GenerateRequest> rq = {reqs[2]};
        rq[0].refresh_margin = 1e30f;
        rq[0].refresh_window = 2;
        const RunResult plain = run(w, {reqs[2]}, 1);
        const RunResult refreshed = run(w, rq, 1);
        EXPECT(refreshed.refreshes[0] == frames[2] && plain.refreshes[0] == 0);
        EXPECT(count_differences(refreshed.frames[0], plain.frames[0]) == 0);
        const Cache &a = refreshed.caches.at(0), &b = plain.caches.at(0);
        EXPECT(!a.empty() && a.size() == b.size());
        EXPECT(std::equal(a.begin(), a.end(), b.begin()));
        // in a batch: the refreshed request's neighbours are untouched
        std::vector<hkv_pipeline::GenerateRequest> rb = reqs;
        rb[0].refresh_margin = 1e30f;
        rb[0].refresh_window = 2;
        const RunResult br = run(w, rb, 3);
        EXPECT(br.refreshes[0] == frames[0]);
        for (int r = 0; r < 4; ++r) {
            EXPECT(br.status[r] == RequestStatus::kDone);
            EXPECT(count_differences(br.frames[r], batched.frames[r]) == 0);
            if (r != 0) EXPECT(br.caches.at(r) == batched.caches.at(r));
        }
    }
    fixture::free_all();
    std::printf("scheduler ok\n");
    return 0;
}
