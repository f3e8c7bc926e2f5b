// Exercises include/hkv_scheduler.hpp on a GPU: requests of different prompt
// lengths and frame counts are admitted (one waits in the queue), batched
// per step through a 2-layer Q4_K backbone and retired.  Every request must
// get exactly its frames, codes in range, all slots released, and the same
// frames as when the requests run one at a time.
#include <cmath>
#include <cstdio>
#include <vector>

#include "hkv_scheduler.hpp"

#define EXPECT(c)                                                                \
    do {                                                                         \
        if (!(c)) {                                                              \
            std::fprintf(stderr, "FAILED %s:%d: %s\n", __FILE__, __LINE__, #c);  \
            return 1;                                                            \
        }                                                                        \
    } while (0)

namespace {

uint64_t g_rng = 0x9E3779B97F4A7C15ull;
float next_normal() {  // sum of four uniforms, unit variance (test data only)
    float s = 0.f;
    for (int i = 0; i < 4; ++i) {
        g_rng = g_rng * 6364136223846793005ull + 1442695040888963407ull;
        s += static_cast<float>((g_rng >> 40) & 0xFFFFFF) / 16777216.0f - 0.5f;
    }
    return s * 1.7320508f;
}

std::vector<void *> g_allocs;
void *dmalloc(size_t bytes) {
    void *p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) throw std::runtime_error("cudaMalloc");
    g_allocs.push_back(p);
    return p;
}

const void *q4k(int64_t rows, int64_t cols) {
    std::vector<float> h(static_cast<size_t>(rows * cols));
    for (float &x : h) x = 0.02f * next_normal();
    float *f = static_cast<float *>(dmalloc(h.size() * 4));
    cudaMemcpy(f, h.data(), h.size() * 4, cudaMemcpyHostToDevice);
    void *b = dmalloc(static_cast<size_t>(rows * cols / 256 * 144));
    char msg[256];
    if (hkv_q4k_quantize(f, rows, cols, b, nullptr, msg, sizeof msg) != HKV_OK) throw std::runtime_error(msg);
    return b;
}

const float *norm(int64_t n) {
    std::vector<float> h(static_cast<size_t>(n));
    for (float &x : h) x = 1.0f + 0.1f * next_normal();
    float *d = static_cast<float *>(dmalloc(h.size() * 4));
    cudaMemcpy(d, h.data(), h.size() * 4, cudaMemcpyHostToDevice);
    return d;
}

using Frames = std::vector<hkv_pipeline::StepScheduler::Frame>;

std::vector<Frames> run(const hkv_backbone_weights &w, const std::vector<hkv_pipeline::GenerateRequest> &reqs,
                        int32_t max_batch, size_t *max_live_seen) {
    hkv_config cfg;
    hkv_config_default(&cfg);
    cfg.n_layers = 2;
    cfg.n_pages = 64;
    cfg.max_slots = 4;
    cfg.device = 0;
    hkv_pipeline::PagedKvRuntime rt(cfg);
    hkv_backbone *bb = nullptr;
    hkv_pipeline::check(nullptr, hkv_backbone_create(rt.engine(), &w, 4, &bb), "hkv_backbone_create");
    std::vector<Frames> out;
    {
        hkv_pipeline::StepScheduler sched(rt, bb, max_batch, nullptr);
        std::vector<int64_t> ids;
        for (const auto &r : reqs) ids.push_back(sched.submit(r));
        *max_live_seen = 0;
        for (int it = 0; it < 1000 && sched.step() > 0; ++it) {
            if (sched.live() > *max_live_seen) *max_live_seen = sched.live();
        }
        for (int64_t id : ids) {
            if (!sched.finished(id)) throw std::runtime_error("request did not finish");
            out.push_back(sched.frames(id));
        }
        hkv_pool_stats st{};
        hkv_pool_stats_get(rt.engine(), &st);
        if (st.live_slots != 0 || st.reserved != 0) throw std::runtime_error("slots not released");
    }
    hkv_backbone_destroy(bb);
    return out;
}

}  // namespace

int main() {
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
    size_t live_batched = 0, live_solo = 0;
    const std::vector<Frames> batched = run(w, reqs, 3, &live_batched);  // the 4th request queues
    const std::vector<Frames> solo = run(w, reqs, 1, &live_solo);
    EXPECT(live_batched == 3 && live_solo == 1);
    int differ = 0;
    for (int r = 0; r < 4; ++r) {
        EXPECT(static_cast<int>(batched[r].size()) == frames[r]);
        EXPECT(static_cast<int>(solo[r].size()) == frames[r]);
        for (int f = 0; f < frames[r]; ++f) {
            for (int c = 0; c < 8; ++c) {
                EXPECT(batched[r][f][c] >= 0 && batched[r][f][c] < 1026);
                differ += batched[r][f][c] != solo[r][f][c];
            }
        }
    }
    // batched and one-at-a-time runs differ only in float summation order
    EXPECT(differ == 0);
    for (void *p : g_allocs) cudaFree(p);
    std::printf("scheduler ok\n");
    return 0;
}
