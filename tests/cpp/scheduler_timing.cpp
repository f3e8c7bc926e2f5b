// scheduler_timing.cpp -- host cost of hkv_pipeline::StepScheduler, the C++
// serving loop, on the Q4_K backbone (hidden 2560, FFN 9728, GQA 32/8,
// random weights, distinct buffers per layer so no layer reads another's
// bytes from L2).
//
// For each batch size B: B requests with 32-token prompts run through the
// scheduler on their own stream; after the prompts and 8 warm-up frames the
// scheduler's counters are reset and `steps` generation steps are timed on
// the host clock.  A generation step is one hkv_backbone_embed_codes +
// hkv_backbone_decode for the batch and the read-back of its greedy codes
// (one stream synchronisation).  The same decode is then launched back to
// back on B fresh slots at the same contexts, without host reads, and timed
// with CUDA events: the device time of a step.  One JSON line per B:
//   device_ms_per_step      back-to-back decode, CUDA events
//   wall_ms_per_step        scheduler step() on the host clock
//   host_us_per_step        step() time outside the synchronisations
//   wait_us_per_step        step() time blocked in the synchronisations
//
// usage: scheduler_timing [layers=36] [steps=64] [batch ...=1 4 16]
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "backbone_fixture.hpp"
#include "hkv_scheduler.hpp"

namespace {

constexpr int kPrompt = 32;
constexpr int kWarm = 8;
constexpr int kHidden = 2560, kFfn = 9728, kTextVocab = 4096, kCodes = 8 * 1026;

struct Sources {  // one F32 matrix per projection shape
    const float *q, *kv, *o, *gate, *up, *down;
};

hkv_backbone_weights make_weights(int layers, std::vector<hkv_backbone_layer> &out) {
    using fixture::normal_f32;
    using fixture::q4k_from;
    using fixture::norm;
    const Sources s = {normal_f32(4096, kHidden), normal_f32(1024, kHidden), normal_f32(kHidden, 4096),
                       normal_f32(kFfn, kHidden), normal_f32(kFfn, kHidden), normal_f32(kHidden, kFfn)};
    out.resize(static_cast<size_t>(layers));
    for (auto &l : out) {
        l = {q4k_from(s.q, 4096, kHidden), q4k_from(s.kv, 1024, kHidden), q4k_from(s.kv, 1024, kHidden),
             q4k_from(s.o, kHidden, 4096), q4k_from(s.gate, kFfn, kHidden), q4k_from(s.up, kFfn, kHidden),
             q4k_from(s.down, kHidden, kFfn), norm(kHidden), norm(kHidden), norm(128), norm(128)};
    }
    return {kHidden, kFfn, kTextVocab, 8, 1026, 1e-6f, out.data(), fixture::q4k(kTextVocab, kHidden),
            fixture::q4k(kCodes, kHidden), norm(kHidden), fixture::q4k(kCodes, kHidden)};
}

void check(hkv_backbone *bb, int st, const char *what) {
    if (st != HKV_OK) {
        std::fprintf(stderr, "%s: %s\n", what, bb != nullptr ? hkv_backbone_last_error(bb) : "error");
        std::exit(1);
    }
}

void run(const hkv_backbone_weights &w, int layers, int steps, int batch, cudaStream_t stream) {
    hkv_config cfg;
    hkv_config_default(&cfg);
    cfg.n_layers = layers;
    cfg.max_slots = 2 * batch;
    const int capacity = kPrompt + kWarm + steps + 1;
    cfg.n_pages = 2 * batch * (capacity / 16 + 2);
    cfg.device = 0;
    cfg.shuffle_seed = 7;
    hkv_pipeline::PagedKvRuntime rt(cfg);
    hkv_backbone *bb = nullptr;
    check(nullptr, hkv_backbone_create(rt.engine(), &w, batch, &bb), "hkv_backbone_create");
    hkv_stream hs = stream;

    // ---- through the scheduler
    double wall_us = 0.0;
    hkv_pipeline::StepScheduler::StepTimes t;
    {
        hkv_pipeline::StepScheduler sched(rt, bb, batch, hs);
        for (int r = 0; r < batch; ++r) {
            hkv_pipeline::GenerateRequest req;
            for (int i = 0; i < kPrompt; ++i) req.prompt_ids.push_back((131 * r + 17 * i) % kTextVocab);
            req.max_frames = kWarm + steps;
            sched.submit(std::move(req));
        }
        for (int i = 0; i < kPrompt + kWarm; ++i) sched.step();
        sched.reset_times();
        const auto t0 = std::chrono::steady_clock::now();
        for (int i = 0; i < steps; ++i) sched.step();
        wall_us = std::chrono::duration<double, std::micro>(std::chrono::steady_clock::now() - t0).count();
        t = sched.times();
        if (sched.live() != 0 || sched.queued() != 0) {
            std::fprintf(stderr, "requests did not finish in the timed steps\n");
            std::exit(1);
        }
    }

    // ---- the same decode back to back, device time
    std::vector<int32_t> slots(static_cast<size_t>(batch));
    for (auto &s : slots) check(nullptr, hkv_slot_acquire(rt.engine(), capacity, nullptr, &s), "hkv_slot_acquire");
    std::vector<int32_t> ids(static_cast<size_t>(batch));
    for (int i = 0; i < kPrompt; ++i) {
        for (int r = 0; r < batch; ++r) ids[static_cast<size_t>(r)] = (131 * r + 17 * i) % kTextVocab;
        check(bb, hkv_backbone_embed_text(bb, batch, ids.data(), hs), "embed text");
        check(bb, hkv_backbone_decode(bb, batch, slots.data(), i == kPrompt - 1, hs), "prompt decode");
    }
    auto frame = [&] {
        check(bb, hkv_backbone_embed_codes(bb, batch, nullptr, hs), "embed codes");
        check(bb, hkv_backbone_decode(bb, batch, slots.data(), 1, hs), "frame decode");
    };
    for (int i = 0; i < kWarm; ++i) frame();
    cudaEvent_t e0, e1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    cudaEventRecord(e0, stream);
    for (int i = 0; i < steps; ++i) frame();
    cudaEventRecord(e1, stream);
    check(bb, hkv_backbone_sync_check(bb, hs), "device check");
    float dev_ms = 0.f;
    cudaEventElapsedTime(&dev_ms, e0, e1);
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    for (int32_t s : slots) hkv_slot_release(rt.engine(), s);
    hkv_backbone_destroy(bb);

    const double n = static_cast<double>(steps);
    std::printf("{\"batch\": %d, \"layers\": %d, \"steps\": %d, \"contexts\": [%d, %d], "
                "\"device_ms_per_step\": %.4f, \"wall_ms_per_step\": %.4f, \"host_us_per_step\": %.1f, "
                "\"wait_us_per_step\": %.1f, \"counted_steps\": %lld, \"host_frac_of_device\": %.3f, "
                "\"wall_over_device\": %.3f}\n",
                batch, layers, steps, kPrompt + kWarm + 1, kPrompt + kWarm + steps, dev_ms / n, wall_us / n / 1e3,
                t.host_us / n, t.wait_us / n, static_cast<long long>(t.steps), t.host_us / n / (dev_ms / n * 1e3),
                wall_us / n / 1e3 / (dev_ms / n));
    std::fflush(stdout);
}

}  // namespace

int main(int argc, char **argv) {
    const int layers = argc > 1 ? std::atoi(argv[1]) : 36;
    const int steps = argc > 2 ? std::atoi(argv[2]) : 64;
    std::vector<int> batches;
    for (int i = 3; i < argc; ++i) batches.push_back(std::atoi(argv[i]));
    if (batches.empty()) batches = {1, 4, 16};
    if (layers <= 0 || steps <= 0) {
        std::fprintf(stderr, "usage: scheduler_timing [layers] [steps] [batch ...]\n");
        return 2;
    }
    for (int b : batches) {
        if (b <= 0) {
            std::fprintf(stderr, "batch sizes must be positive\n");
            return 2;
        }
    }
    cudaStream_t stream;
    cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
    std::vector<hkv_backbone_layer> layer_weights;
    const hkv_backbone_weights w = make_weights(layers, layer_weights);
    cudaDeviceSynchronize();  // quantised on the legacy stream; used on `stream`
    for (int b : batches) run(w, layers, steps, b, stream);
    cudaStreamDestroy(stream);
    fixture::free_all();
    return 0;
}
