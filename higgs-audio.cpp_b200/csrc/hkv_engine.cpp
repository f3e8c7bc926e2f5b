// hkv_engine.cpp -- host side of the paged KV decode engine behind include/hkv.h.
//
// Host-authoritative bookkeeping (slots, page lists, refcounts, reservations,
// prefix registry) under one mutex; the GPU sees only a per-batch descriptor
// (positions, page lists, stream-K split plan) uploaded in one copy when the
// batch changes, so the 36 per-layer launches of a decode step reuse it.
//
// Reference counterparts (bluryar/higgs-audio.cpp, src/higgs_pipeline.cpp):
//   BackendRuntime slot arena + acquire/release      :357-403, :1191-1220
//   backend_kv_cache_offset_bytes (range checks)      :1137-1142
//   make_backend_kv_cache / capacity growth            :1144-1175, :1197-1199
//   make_bf16_rope_table / ensure_backend_kv_rope_tables :475-487, :1606-1622
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <string>
#include <utility>
#include <vector>

#include "../../include/hkv.h"
#include "hkv_internal.h"
#include "hkv_plan.h"

namespace hkv {
namespace {

// ------------------------------------------------------------ status text
const char *status_name(int s) {
    switch (s) {
    case HKV_OK: return "ok";
    case HKV_ERR_INVALID: return "invalid argument";
    case HKV_ERR_OOM: return "out of pages or slots";
    case HKV_ERR_BAD_SLOT: return "bad slot";
    case HKV_ERR_RANGE: return "position out of range";
    case HKV_ERR_CUDA: return "CUDA error";
    case HKV_ERR_TIMEOUT: return "device wait timed out";
    case HKV_ERR_NO_DEVICE: return "host-only engine";
    case HKV_ERR_NOT_FOUND: return "not found";
    case HKV_ERR_DEVICE: return "device bounds check failed";
    default: return "unknown status";
    }
}

// BF16 round trip of the reference's table entries: round to nearest even
// on the upper 16 bits, NaN kept quiet (ggml_fp32_to_bf16 semantics, used by
// bf16_rne_to_f32 at src/higgs_pipeline.cpp:471-473).
float bf16_round(float x) {
    uint32_t u;
    std::memcpy(&u, &x, 4);
    uint32_t b;
    if ((u & 0x7fffffffu) > 0x7f800000u) {
        b = (u >> 16) | 64u;
    } else {
        b = (u + (0x7fffu + ((u >> 16) & 1u))) >> 16;
    }
    b <<= 16;
    float out;
    std::memcpy(&out, &b, 4);
    return out;
}

// The reference's table expression, evaluated the same way on the host
// (float pow / cos / sin overloads, then BF16 rounding).
void build_rope_tables(int64_t context_length, int64_t key_length, float base,
                       std::vector<float> &cos_tab, std::vector<float> &sin_tab) {
    const int64_t half = key_length / 2;
    cos_tab.assign(static_cast<size_t>(half * context_length), 0.f);
    sin_tab.assign(static_cast<size_t>(half * context_length), 0.f);
    for (int64_t pos = 0; pos < context_length; ++pos) {
        for (int64_t i = 0; i < half; ++i) {
            const float dim = static_cast<float>(i * 2);
            const float freq = 1.0f / std::pow(base, dim / static_cast<float>(key_length));
            const float angle = static_cast<float>(pos) * freq;
            cos_tab[static_cast<size_t>(pos * half + i)] = bf16_round(std::cos(angle));
            sin_tab[static_cast<size_t>(pos * half + i)] = bf16_round(std::sin(angle));
        }
    }
}

// Restores the caller's current device when a call leaves.
class DeviceGuard {
  public:
    explicit DeviceGuard(int device) {
        if (device >= 0 && cudaGetDevice(&prev_) == cudaSuccess && prev_ != device) {
            cudaSetDevice(device);
            restore_ = true;
        }
    }
    ~DeviceGuard() {
        if (restore_) {
            cudaSetDevice(prev_);
        }
    }

  private:
    int prev_ = -1;
    bool restore_ = false;
};

// Double-buffered host->device staging for small metadata.  A buffer is
// rewritten on the host only after its previous copy ran, and on the device
// only after the kernels that read it (events), so one call's upload never
// races the previous one's readers.
class Staging {
  public:
    ~Staging() { release(); }

    void release() {
        for (Buf &b : buf_) {
            if (b.host != nullptr) {
                cudaEventSynchronize(b.used);
                cudaFreeHost(b.host);
                cudaFree(b.dev);
            }
            if (b.copied != nullptr) {
                cudaEventDestroy(b.copied);
                cudaEventDestroy(b.used);
            }
            b = Buf{};
        }
    }

    // Host memory for the next upload of `bytes`.
    cudaError_t begin(size_t bytes, void **host_out) {
        cur_ ^= 1;
        Buf &b = buf_[cur_];
        if (b.copied == nullptr) {
            cudaError_t e = cudaEventCreateWithFlags(&b.copied, cudaEventDisableTiming);
            if (e == cudaSuccess) e = cudaEventCreateWithFlags(&b.used, cudaEventDisableTiming);
            if (e != cudaSuccess) return e;
        }
        if (b.copy_pending) {
            const auto t0 = std::chrono::steady_clock::now();
            cudaError_t e = cudaEventSynchronize(b.copied);
            wait_ns_ += std::chrono::duration_cast<std::chrono::nanoseconds>(
                            std::chrono::steady_clock::now() - t0)
                            .count();
            if (e != cudaSuccess) return e;
            b.copy_pending = false;
        }
        if (bytes > b.cap) {
            if (b.host != nullptr) {
                cudaEventSynchronize(b.used);
                cudaFreeHost(b.host);
                cudaFree(b.dev);
                b.host = nullptr;
                b.dev = nullptr;
                b.cap = 0;
            }
            size_t cap = 4096;
            while (cap < bytes) cap *= 2;
            cudaError_t e = cudaHostAlloc(&b.host, cap, cudaHostAllocDefault);
            if (e != cudaSuccess) return e;
            e = cudaMalloc(&b.dev, cap);
            if (e != cudaSuccess) return e;
            b.cap = cap;
            b.used_recorded = false;
        }
        *host_out = b.host;
        return cudaSuccess;
    }

    // Copies the staged bytes to the device, ordered on `stream`.
    cudaError_t commit(size_t bytes, cudaStream_t stream, void **dev_out) {
        Buf &b = buf_[cur_];
        if (b.used_recorded) {
            cudaError_t e = cudaStreamWaitEvent(stream, b.used, 0);
            if (e != cudaSuccess) return e;
        }
        cudaError_t e = cudaMemcpyAsync(b.dev, b.host, bytes, cudaMemcpyHostToDevice, stream);
        if (e != cudaSuccess) return e;
        e = cudaEventRecord(b.copied, stream);
        if (e != cudaSuccess) return e;
        b.copy_pending = true;
        *dev_out = b.dev;
        return cudaSuccess;
    }

    // Host time spent waiting for an earlier upload from the buffer now reused.
    int64_t take_wait_ns() {
        const int64_t w = wait_ns_;
        wait_ns_ = 0;
        return w;
    }

    // Marks the current buffer as read by work queued on `stream` so far.
    cudaError_t mark_used(cudaStream_t stream) {
        Buf &b = buf_[cur_];
        b.used_recorded = true;
        return cudaEventRecord(b.used, stream);
    }

  private:
    struct Buf {
        void *host = nullptr;
        void *dev = nullptr;
        size_t cap = 0;
        cudaEvent_t copied = nullptr;
        cudaEvent_t used = nullptr;
        bool copy_pending = false;
        bool used_recorded = false;
    };
    Buf buf_[2];
    int cur_ = 1;
    int64_t wait_ns_ = 0;
};

struct Slot {
    bool live = false;
    int64_t used = 0;
    int64_t reserved = 0;          // pages this slot may still allocate without failing
    std::vector<int32_t> pages;    // physical page of positions [16 i, 16 i + 16)
};

struct Prefix {
    int64_t n_tokens = 0;
    std::vector<int32_t> pages;
};

struct BatchCache {
    bool valid = false;
    uint64_t epoch = 0;
    std::vector<int32_t> slots;
    std::vector<int64_t> used;
    BatchView view{};
    // Kernels read the descriptor until the batch changes; its staging buffer
    // is marked used (event on the consumers' stream) only then, so no event
    // sits between the consecutive launches of a step.
    bool consumed = false;
    cudaStream_t consumer_stream = nullptr;
};

struct ProfileRecord {
    cudaEvent_t start;
    cudaEvent_t stop;
};

}  // namespace
}  // namespace hkv

struct hkv_engine {
    hkv_config cfg{};
    mutable std::mutex mu;
    mutable std::string last_error;
    bool device_mode = false;

    // host bookkeeping
    std::vector<int32_t> refcnt;
    std::vector<int32_t> free_pages;  // stack
    int64_t reserved_total = 0;
    int64_t shared_pages = 0;
    int64_t cow_copies = 0;
    int64_t kernel_launches = 0;  // every kernel this engine enqueued
    std::vector<hkv::Slot> slots;
    std::vector<int32_t> free_slots;  // stack
    std::map<std::pair<uint64_t, int64_t>, hkv::Prefix> prefixes;
    uint64_t epoch = 1;
    int64_t page_bytes = 0;
    std::vector<float> rope_cos, rope_sin;

    // device state
    uint8_t *pool = nullptr;
    float *d_cos = nullptr;
    float *d_sin = nullptr;
    hkv::DeviceError *d_err = nullptr;
    float *part_o = nullptr;
    float *part_ml = nullptr;
    int32_t *counters = nullptr;  // one per (batch entry, KV head), zero between launches
    int64_t part_cap = 0;
    int num_sms = 0;
    float scale_log2 = 0.f;
    hkv::Staging batch_stage, range_stage, gather_stage, cow_stage;
    // Copy-on-write copies decided on the host and not yet enqueued:
    // {source page, destination page} pairs, flushed as one kernel launch.
    std::vector<int32_t> cow_pending;
    hkv::BatchCache batch;

    // Launch overlap bookkeeping: a decode launch may start while the previous
    // kernel in the stream finishes (programmatic dependent launch) only if
    // that kernel was this engine's decode launch of another layer on the same
    // stream with nothing else enqueued by the engine in between.
    uint64_t enqueue_seq = 0;       // bumped by every non-decode enqueue
    uint64_t last_decode_seq = ~0ull;
    int32_t last_decode_layer = -1;
    cudaStream_t last_decode_stream = nullptr;

    // KV-head split exchange (hkv_split_*): this rank's region holds the
    // per-layer arrival counters, then the head-major output rows of all ranks.
    int32_t split_world = 0;
    int32_t split_rank = -1;
    uint8_t *xchg = nullptr;
    size_t xchg_flags_bytes = 0;
    int32_t xchg_row_floats = 0;
    std::vector<void *> peer_bases;          // opened IPC mappings (nullptr for self)
    float **d_outs = nullptr;                // [world] device array
    uint32_t **d_flags = nullptr;            // [world] device array
    std::vector<uint32_t> split_target;      // expected arrivals per layer
    bool split_connected = false;

    // host time spent inside the compute entry points (hkv_host_stats)
    mutable std::mutex host_mu;
    int64_t host_calls = 0;
    int64_t host_ns = 0;
    int64_t launch_ns = 0;  // of host_ns: inside the kernel launch calls
    int64_t staging_wait_ns = 0;  // of host_ns: waiting to reuse a plan upload buffer

    // profiling
    bool profiling = false;
    std::vector<hkv::ProfileRecord> prof[HKV_KERNEL_COUNT];
    std::vector<cudaEvent_t> event_pool;
};

namespace hkv {
namespace {

int fail(const hkv_engine *eng, int status, const char *fmt, ...) {
    if (eng != nullptr) {
        char buf[512];
        va_list ap;
        va_start(ap, fmt);
        std::vsnprintf(buf, sizeof(buf), fmt, ap);
        va_end(ap);
        eng->last_error = std::string(status_name(status)) + ": " + buf;
    }
    return status;
}

int cuda_fail(const hkv_engine *eng, cudaError_t e, const char *what) {
    return fail(eng, HKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

#define HKV_CUDA_TRY(eng, expr)                              \
    do {                                                     \
        cudaError_t hkv_e_ = (expr);                         \
        if (hkv_e_ != cudaSuccess) {                         \
            return cuda_fail((eng), hkv_e_, #expr);          \
        }                                                    \
    } while (0)

int64_t pages_for(int64_t tokens) { return (tokens + kPageTokens - 1) / kPageTokens; }

bool slot_ok(const hkv_engine *eng, int32_t slot) {
    return slot >= 0 && slot < static_cast<int32_t>(eng->slots.size()) && eng->slots[slot].live;
}

int64_t unreserved_free(const hkv_engine *eng) {
    return static_cast<int64_t>(eng->free_pages.size()) - eng->reserved_total;
}

void incref(hkv_engine *eng, int32_t page) {
    if (++eng->refcnt[page] == 2) {
        ++eng->shared_pages;
    }
}

void decref(hkv_engine *eng, int32_t page) {
    const int32_t r = --eng->refcnt[page];
    if (r == 1) {
        --eng->shared_pages;
    } else if (r == 0) {
        eng->free_pages.push_back(page);
    }
}

// Takes one free page for `slot`, from its reservation first.  The caller has
// checked availability.
int32_t take_page(hkv_engine *eng, Slot &slot) {
    if (slot.reserved > 0) {
        --slot.reserved;
        --eng->reserved_total;
    }
    const int32_t page = eng->free_pages.back();
    eng->free_pages.pop_back();
    eng->refcnt[page] = 1;
    return page;
}

// Bytes of one page within one layer's slab (K and V of every KV head).
int64_t layer_page_bytes(const hkv_engine *eng) {
    return 2ll * eng->cfg.n_head_kv * kHeadBlockBytes;
}

uint8_t *page_ptr(const hkv_engine *eng, int32_t layer, int32_t page) {
    return eng->pool +
           (static_cast<int64_t>(layer) * eng->cfg.n_pages + page) * layer_page_bytes(eng);
}

// Pages `slot` must newly take to own every page touched by rows
// [begin, end): fresh pages past its list plus copies of shared ones.
int64_t pages_needed(const hkv_engine *eng, const Slot &s, int64_t begin, int64_t end) {
    if (end <= begin) {
        return 0;
    }
    int64_t need = 0;
    const int64_t first = begin / kPageTokens;
    const int64_t last = (end - 1) / kPageTokens;
    for (int64_t p = first; p <= last; ++p) {
        if (p >= static_cast<int64_t>(s.pages.size())) {
            ++need;
        } else if (eng->refcnt[s.pages[p]] > 1) {
            ++need;
        }
    }
    return need;
}

int64_t pages_beyond_reservation(const Slot &s, int64_t need) {
    return std::max<int64_t>(0, need - s.reserved);
}

// References held on copy-on-write sources until their copies are enqueued
// (a page another slot of the same call left can be owned outright).
int32_t pending_cow_sources(const hkv_engine *eng, int32_t page) {
    int32_t n = 0;
    for (size_t i = 0; i < eng->cow_pending.size(); i += 2) {
        n += eng->cow_pending[i] == page ? 1 : 0;
    }
    return n;
}

// Makes `slot` the only owner of every page touched by rows [begin, end),
// appending fresh pages and copying shared ones (copy-on-write) on `stream`.
// Availability has been checked by the caller.
int own_rows(hkv_engine *eng, Slot &s, int64_t begin, int64_t end, cudaStream_t stream) {
    if (end <= begin) {
        return HKV_OK;
    }
    const int64_t first = begin / kPageTokens;
    const int64_t last = (end - 1) / kPageTokens;
    bool changed = false;
    for (int64_t p = first; p <= last; ++p) {
        if (p >= static_cast<int64_t>(s.pages.size())) {
            s.pages.push_back(take_page(eng, s));
            changed = true;
        } else if (eng->refcnt[s.pages[p]] - pending_cow_sources(eng, s.pages[p]) > 1) {
            const int32_t old = s.pages[p];
            const int32_t fresh = take_page(eng, s);
            if (eng->device_mode) {
                // The page lives in every layer's slab; flush_cow copies all
                // layers of all pending pages in one launch.  Until then the
                // old page keeps a reference, so it cannot be reused.
                incref(eng, old);
                eng->cow_pending.push_back(old);
                eng->cow_pending.push_back(fresh);
            }
            decref(eng, old);
            s.pages[p] = fresh;
            ++eng->cow_copies;
            changed = true;
        }
    }
    if (changed) {
        ++eng->epoch;
    }
    return HKV_OK;
}

PoolView pool_view(const hkv_engine *eng);

// Enqueues the pending copy-on-write copies (one kernel launch for all pages
// and layers) and drops the references that kept their source pages alive.
int flush_cow(hkv_engine *eng, cudaStream_t stream) {
    if (eng->cow_pending.empty()) {
        return HKV_OK;
    }
    const int32_t n_pairs = static_cast<int32_t>(eng->cow_pending.size() / 2);
    const size_t bytes = eng->cow_pending.size() * sizeof(int32_t);
    void *host = nullptr;
    int st = HKV_OK;
    cudaError_t e = eng->cow_stage.begin(bytes, &host);
    void *dev = nullptr;
    if (e == cudaSuccess) {
        std::memcpy(host, eng->cow_pending.data(), bytes);
        ++eng->enqueue_seq;
        e = eng->cow_stage.commit(bytes, stream, &dev);
    }
    if (e == cudaSuccess) {
        launch_cow_copy(pool_view(eng), static_cast<const int32_t *>(dev), n_pairs, eng->d_err,
                        stream);
        ++eng->kernel_launches;
        e = cudaGetLastError();
        if (e == cudaSuccess) {
            e = eng->cow_stage.mark_used(stream);
        }
    }
    if (e != cudaSuccess) {
        st = cuda_fail(eng, e, "copy-on-write launch");
    }
    for (size_t i = 0; i < eng->cow_pending.size(); i += 2) {
        decref(eng, eng->cow_pending[i]);
    }
    eng->cow_pending.clear();
    return st;
}

PoolView pool_view(const hkv_engine *eng) {
    PoolView v;
    v.base = eng->pool;
    v.n_pages = eng->cfg.n_pages;
    v.n_layers = eng->cfg.n_layers;
    v.n_head_kv = eng->cfg.n_head_kv;
    return v;
}

RopeView rope_view(const hkv_engine *eng) {
    RopeView v;
    v.cos_tab = eng->d_cos;
    v.sin_tab = eng->d_sin;
    v.context_length = eng->cfg.context_length;
    return v;
}

cudaEvent_t pooled_event(hkv_engine *eng) {
    if (!eng->event_pool.empty()) {
        cudaEvent_t e = eng->event_pool.back();
        eng->event_pool.pop_back();
        return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
}

// Brackets one kernel launch with events when profiling is on.
class ProfileScope {
  public:
    ProfileScope(hkv_engine *eng, int kernel, cudaStream_t stream)
        : eng_(eng), kernel_(kernel), stream_(stream) {
        if (eng_->profiling) {
            rec_.start = pooled_event(eng_);
            rec_.stop = pooled_event(eng_);
            cudaEventRecord(rec_.start, stream_);
        }
    }
    ~ProfileScope() {
        if (eng_->profiling) {
            cudaEventRecord(rec_.stop, stream_);
            eng_->prof[kernel_].push_back(rec_);
        }
    }

  private:
    hkv_engine *eng_;
    int kernel_;
    cudaStream_t stream_;
    ProfileRecord rec_{};
};

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Adds the host time of one compute call (entry to return, lock included)
// to the engine's counters.
class HostTimer {
  public:
    explicit HostTimer(hkv_engine *eng) : eng_(eng), t0_(std::chrono::steady_clock::now()) {}
    ~HostTimer() {
        const auto dt = std::chrono::steady_clock::now() - t0_;
        const int64_t waited = eng_->batch_stage.take_wait_ns();
        std::lock_guard<std::mutex> lock(eng_->host_mu);
        ++eng_->host_calls;
        eng_->host_ns += std::chrono::duration_cast<std::chrono::nanoseconds>(dt).count();
        eng_->staging_wait_ns += waited;
    }

  private:
    hkv_engine *eng_;
    std::chrono::steady_clock::time_point t0_;
};

int check_compute(hkv_engine *eng, int32_t layer) {
    if (!eng->device_mode) {
        return fail(eng, HKV_ERR_NO_DEVICE, "engine was created without a device");
    }
    if (layer < 0 || layer >= eng->cfg.n_layers) {
        return fail(eng, HKV_ERR_RANGE, "layer %d outside [0, %d)", layer, eng->cfg.n_layers);
    }
    return HKV_OK;
}

// Builds (or reuses) the device descriptor of a decode batch: every slot gets
// its row `used` owned (fresh page or copy-on-write), then positions, page
// lists and the stream-K split are uploaded in one copy.
int ensure_batch(hkv_engine *eng, int32_t n, const int32_t *slots, cudaStream_t stream) {
    BatchCache &bc = eng->batch;
    if (n <= 0 || slots == nullptr) {
        return fail(eng, HKV_ERR_INVALID, "empty slot list");
    }
    if (bc.valid && bc.epoch == eng->epoch && static_cast<int32_t>(bc.slots.size()) == n) {
        bool same = true;
        for (int32_t e = 0; e < n && same; ++e) {
            same = bc.slots[e] == slots[e] && slot_ok(eng, slots[e]) &&
                   bc.used[e] == eng->slots[slots[e]].used;
        }
        if (same) {
            return HKV_OK;
        }
    }
    // Phase 1: validate and count, changing nothing.
    int64_t extra = 0;
    for (int32_t e = 0; e < n; ++e) {
        const int32_t s = slots[e];
        if (!slot_ok(eng, s)) {
            return fail(eng, HKV_ERR_BAD_SLOT, "slot %d is not live (batch entry %d)", s, e);
        }
        for (int32_t f = 0; f < e; ++f) {
            if (slots[f] == s) {
                return fail(eng, HKV_ERR_INVALID, "slot %d appears twice in one batch", s);
            }
        }
        const Slot &sl = eng->slots[s];
        if (sl.used >= eng->cfg.context_length) {
            return fail(eng, HKV_ERR_RANGE, "slot %d: position %lld reaches context length %d", s,
                        static_cast<long long>(sl.used), eng->cfg.context_length);
        }
        extra += pages_beyond_reservation(sl, pages_needed(eng, sl, sl.used, sl.used + 1));
    }
    if (extra > unreserved_free(eng)) {
        return fail(eng, HKV_ERR_OOM, "batch needs %lld unreserved pages, %lld free",
                    static_cast<long long>(extra), static_cast<long long>(unreserved_free(eng)));
    }
    // Phase 2: own the rows being written.
    for (int32_t e = 0; e < n; ++e) {
        Slot &sl = eng->slots[slots[e]];
        const int st = own_rows(eng, sl, sl.used, sl.used + 1, stream);
        if (st != HKV_OK) {
            return st;
        }
    }
    {
        const int st = flush_cow(eng, stream);
        if (st != HKV_OK) {
            return st;
        }
    }
    // Descriptor: positions, page lists and the stream-K split (hkv_plan.h).
    const int32_t G = eng->cfg.n_head_kv;
    int64_t total_pages = 0;
    std::vector<int32_t> pos(static_cast<size_t>(n));
    std::vector<const int32_t *> lists(static_cast<size_t>(n));
    for (int32_t e = 0; e < n; ++e) {
        const Slot &sl = eng->slots[slots[e]];
        pos[e] = static_cast<int32_t>(sl.used);
        lists[e] = sl.pages.data();
        total_pages += sl.used / kPageTokens + 1;
    }
    if (total_pages * G > INT32_MAX / 2) {
        return fail(eng, HKV_ERR_RANGE, "batch too large (%lld units)",
                    static_cast<long long>(total_pages * G));
    }
    const int64_t max_warps = static_cast<int64_t>(eng->num_sms) * kAttnWarps;
    // One long request: one thread-block cluster per KV head (plan_cluster).
    int32_t C = 0;
    if (n == 1) {
        int32_t fit[5] = {0, 0, 0, 0, 0};
        for (int i = 1; i < 5; ++i) {
            fit[i] = attention_cluster_fit(1 << i);
        }
        C = plan_cluster(n, G, total_pages, max_warps, fit);
    }
    const int32_t W = C > 0 ? G * C * kAttnWarps : plan_warps(total_pages * G, max_warps);
    const size_t words = plan_words(n, G, total_pages, W);
    if (bc.consumed) {
        HKV_CUDA_TRY(eng, eng->batch_stage.mark_used(bc.consumer_stream));
        bc.consumed = false;
    }
    void *host = nullptr;
    HKV_CUDA_TRY(eng, eng->batch_stage.begin(words * sizeof(int32_t), &host));
    const PlanSummary plan =
        C > 0 ? build_cluster_plan(static_cast<int32_t *>(host), G, pos[0], lists[0], C)
              : build_plan(static_cast<int32_t *>(host), n, G, pos.data(), lists.data(), total_pages, W);
    if (static_cast<int64_t>(plan.n_parts) + plan.n_groups > eng->part_cap) {
        return fail(eng, HKV_ERR_OOM, "split plan needs %d partials, capacity %lld",
                    plan.n_parts + plan.n_groups, static_cast<long long>(eng->part_cap));
    }
    void *dev = nullptr;
    ++eng->enqueue_seq;
    HKV_CUDA_TRY(eng, eng->batch_stage.commit(words * sizeof(int32_t), stream, &dev));
    bc.view = bind_plan(static_cast<const int32_t *>(dev), n, G, plan, W);
    bc.slots.assign(slots, slots + n);
    bc.used.resize(static_cast<size_t>(n));
    for (int32_t e = 0; e < n; ++e) {
        bc.used[e] = eng->slots[slots[e]].used;
    }
    bc.epoch = eng->epoch;
    bc.valid = true;
    return HKV_OK;
}

int launch_status(hkv_engine *eng, const char *what) {
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        return cuda_fail(eng, e, what);
    }
    return HKV_OK;
}

int do_append(hkv_engine *eng, int32_t layer, int32_t n, const int32_t *slots, const float *k,
              const float *v, bool rope, cudaStream_t stream) {
    int st = check_compute(eng, layer);
    if (st != HKV_OK) return st;
    if (k == nullptr || v == nullptr || !aligned16(k) || !aligned16(v)) {
        return fail(eng, HKV_ERR_INVALID, "k and v must be non-null 16-byte aligned device pointers");
    }
    st = ensure_batch(eng, n, slots, stream);
    if (st != HKV_OK) return st;
    ++eng->enqueue_seq;
    {
        ProfileScope ps(eng, HKV_KERNEL_APPEND, stream);
        launch_append(pool_view(eng), rope_view(eng), eng->batch.view, layer, k, v, rope,
                      eng->d_err, stream);
        ++eng->kernel_launches;
    }
    eng->batch.consumed = true;
    eng->batch.consumer_stream = stream;
    return launch_status(eng, "append kernel launch");
}

// One attention launch over the current batch; with k_new / v_new it is the
// fused decode step (append + attention).
int do_attention(hkv_engine *eng, int32_t layer, const float *q, const float *k_new,
                 const float *v_new, float *out, cudaStream_t stream,
                 const Exchange &xchg = Exchange{nullptr, nullptr, 0, 0, 0, 0}) {
    // Profiling brackets each launch with events, which would sit between the
    // kernels, so overlap is only used when profiling is off.
    const bool overlap = !eng->profiling && eng->last_decode_seq == eng->enqueue_seq &&
                         eng->last_decode_stream == stream && eng->last_decode_layer != layer;
    {
        ProfileScope ps(eng, k_new != nullptr ? HKV_KERNEL_STEP : HKV_KERNEL_ATTN, stream);
        const auto t0 = std::chrono::steady_clock::now();
        launch_attention(pool_view(eng), rope_view(eng), eng->batch.view, layer, q, k_new, v_new,
                         eng->part_o, eng->part_ml, eng->counters, out, xchg,
                         eng->scale_log2, eng->d_err, overlap, stream);
        eng->kernel_launches +=
            (eng->batch.view.combine && eng->batch.view.split_segments > 0) ? 2 : 1;
        const auto dt = std::chrono::steady_clock::now() - t0;
        std::lock_guard<std::mutex> lock(eng->host_mu);
        eng->launch_ns += std::chrono::duration_cast<std::chrono::nanoseconds>(dt).count();
    }
    eng->last_decode_seq = eng->enqueue_seq;
    eng->last_decode_layer = layer;
    eng->last_decode_stream = stream;
    eng->batch.consumed = true;
    eng->batch.consumer_stream = stream;
    return launch_status(eng, "attention kernel launch");
}

void free_split(hkv_engine *eng) {
    for (void *p : eng->peer_bases) {
        if (p != nullptr) {
            cudaIpcCloseMemHandle(p);
        }
    }
    eng->peer_bases.clear();
    cudaFree(eng->d_outs);
    cudaFree(eng->d_flags);
    cudaFree(eng->xchg);
    eng->d_outs = nullptr;
    eng->d_flags = nullptr;
    eng->xchg = nullptr;
    eng->split_world = 0;
    eng->split_rank = -1;
    eng->split_connected = false;
}

void free_device(hkv_engine *eng) {
    free_split(eng);
    eng->batch_stage.release();
    eng->range_stage.release();
    eng->gather_stage.release();
    eng->cow_stage.release();
    for (auto &list : eng->prof) {
        for (auto &r : list) {
            cudaEventDestroy(r.start);
            cudaEventDestroy(r.stop);
        }
        list.clear();
    }
    for (cudaEvent_t e : eng->event_pool) {
        cudaEventDestroy(e);
    }
    eng->event_pool.clear();
    cudaFree(eng->pool);
    cudaFree(eng->d_cos);
    cudaFree(eng->d_sin);
    cudaFree(eng->d_err);
    cudaFree(eng->part_o);
    cudaFree(eng->part_ml);
    cudaFree(eng->counters);
    eng->pool = nullptr;
    eng->d_cos = eng->d_sin = nullptr;
    eng->d_err = nullptr;
    eng->part_o = eng->part_ml = nullptr;
    eng->counters = nullptr;
}

}  // namespace
}  // namespace hkv

using namespace hkv;

extern "C" {

int hkv_abi_version(void) { return HKV_ABI_VERSION; }

const char *hkv_status_string(int status) { return status_name(status); }

const char *hkv_last_error(const hkv_engine *eng) {
    if (eng == nullptr) {
        return "null engine";
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    return eng->last_error.c_str();
}

int hkv_config_default(hkv_config *cfg) {
    if (cfg == nullptr) {
        return HKV_ERR_INVALID;
    }
    std::memset(cfg, 0, sizeof(*cfg));
    cfg->n_layers = 36;
    cfg->n_head = 32;
    cfg->n_head_kv = 8;
    cfg->head_dim = 128;
    cfg->page_tokens = 16;
    cfg->context_length = 32768;
    cfg->rope_freq_base = 1e6f;
    cfg->max_slots = 256;
    cfg->n_pages = 4096;
    cfg->device = 0;
    cfg->shuffle_seed = 0;
    return HKV_OK;
}

int hkv_engine_create(const hkv_config *cfg, hkv_engine **out) {
    if (cfg == nullptr || out == nullptr) {
        return HKV_ERR_INVALID;
    }
    *out = nullptr;
    if (cfg->head_dim != kHeadDim || cfg->page_tokens != kPageTokens || cfg->n_head_kv <= 0 ||
        cfg->n_head != kGqa * cfg->n_head_kv || cfg->n_layers <= 0 || cfg->context_length <= 0 ||
        cfg->max_slots <= 0 || cfg->n_pages <= 0 || cfg->n_pages > INT32_MAX ||
        !(cfg->rope_freq_base > 0.f)) {
        return HKV_ERR_INVALID;
    }
    hkv_engine *eng = new (std::nothrow) hkv_engine();
    if (eng == nullptr) {
        return HKV_ERR_OOM;
    }
    eng->cfg = *cfg;
    eng->page_bytes = static_cast<int64_t>(cfg->n_layers) * 2 * cfg->n_head_kv * kHeadBlockBytes;
    eng->refcnt.assign(static_cast<size_t>(cfg->n_pages), 0);
    eng->free_pages.resize(static_cast<size_t>(cfg->n_pages));
    for (int64_t i = 0; i < cfg->n_pages; ++i) {
        // Stack: page 0 is handed out first.
        eng->free_pages[static_cast<size_t>(i)] = static_cast<int32_t>(cfg->n_pages - 1 - i);
    }
    if (cfg->shuffle_seed != 0) {
        // Fisher-Yates with splitmix64, so the order is reproducible anywhere.
        uint64_t state = cfg->shuffle_seed;
        auto next = [&state]() {
            uint64_t z = (state += 0x9E3779B97F4A7C15ull);
            z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
            z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
            return z ^ (z >> 31);
        };
        for (size_t i = eng->free_pages.size() - 1; i > 0; --i) {
            const size_t j = static_cast<size_t>(next() % (i + 1));
            std::swap(eng->free_pages[i], eng->free_pages[j]);
        }
    }
    eng->slots.resize(static_cast<size_t>(cfg->max_slots));
    for (int32_t i = cfg->max_slots - 1; i >= 0; --i) {
        eng->free_slots.push_back(i);
    }
    build_rope_tables(cfg->context_length, cfg->head_dim, cfg->rope_freq_base, eng->rope_cos,
                      eng->rope_sin);
    // 1/sqrt(head_dim) as the reference computes it (:5767), times log2(e)
    // because the kernels exponentiate in base 2.
    const float scale = 1.0f / std::sqrt(static_cast<float>(cfg->head_dim));
    eng->scale_log2 = scale * 1.4426950408889634f;

    if (cfg->device >= 0) {
        eng->device_mode = true;
        DeviceGuard guard(cfg->device);
        auto fail_create = [&](cudaError_t e, const char *what) {
            std::fprintf(stderr, "hkv_engine_create: %s: %s\n", what, cudaGetErrorString(e));
            free_device(eng);
            delete eng;
            return HKV_ERR_CUDA;
        };
        cudaError_t e = cudaSetDevice(cfg->device);
        if (e != cudaSuccess) return fail_create(e, "cudaSetDevice");
        int major = 0;
        e = cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, cfg->device);
        if (e != cudaSuccess) return fail_create(e, "compute capability");
        if (major != 10) {
            std::fprintf(stderr, "hkv_engine_create: device %d is sm_%d0, kernels are sm_100a\n",
                         cfg->device, major);
            free_device(eng);
            delete eng;
            return HKV_ERR_INVALID;
        }
        e = cudaDeviceGetAttribute(&eng->num_sms, cudaDevAttrMultiProcessorCount, cfg->device);
        if (e != cudaSuccess) return fail_create(e, "SM count");
        const size_t pool_bytes = static_cast<size_t>(cfg->n_pages) * eng->page_bytes;
        e = cudaMalloc(&eng->pool, pool_bytes);
        if (e != cudaSuccess) return fail_create(e, "page pool");
        e = cudaMemset(eng->pool, 0, pool_bytes);
        if (e != cudaSuccess) return fail_create(e, "page pool zero fill");
        const size_t tab_bytes = eng->rope_cos.size() * sizeof(float);
        e = cudaMalloc(&eng->d_cos, tab_bytes);
        if (e == cudaSuccess) e = cudaMalloc(&eng->d_sin, tab_bytes);
        if (e == cudaSuccess)
            e = cudaMemcpy(eng->d_cos, eng->rope_cos.data(), tab_bytes, cudaMemcpyHostToDevice);
        if (e == cudaSuccess)
            e = cudaMemcpy(eng->d_sin, eng->rope_sin.data(), tab_bytes, cudaMemcpyHostToDevice);
        if (e != cudaSuccess) return fail_create(e, "rope tables");
        e = cudaMalloc(&eng->d_err, sizeof(DeviceError));
        if (e == cudaSuccess) e = cudaMemset(eng->d_err, 0, sizeof(DeviceError));
        if (e != cudaSuccess) return fail_create(e, "error word");
        // Worst case partial count: one per active warp plus one extra per
        // (entry, KV head) share boundary, then the group partials of the
        // two-level merge (at most one per 8 partials, rounded up).
        const int64_t segs = static_cast<int64_t>(cfg->max_slots) * cfg->n_head_kv;
        const int64_t level1 = static_cast<int64_t>(eng->num_sms) * kAttnWarps + segs;
        const int64_t groups = level1 / 8 + segs;
        eng->part_cap = level1 + groups;
        e = cudaMalloc(&eng->part_o, static_cast<size_t>(eng->part_cap) * kGqa * kHeadDim * 4);
        if (e == cudaSuccess)
            e = cudaMalloc(&eng->part_ml, static_cast<size_t>(eng->part_cap) * 2 * kGqa * 4);
        if (e != cudaSuccess) return fail_create(e, "split partials");
        // segment counters, then group counters
        const size_t counter_bytes = static_cast<size_t>(segs + groups) * 4;
        e = cudaMalloc(&eng->counters, counter_bytes);
        if (e == cudaSuccess) e = cudaMemset(eng->counters, 0, counter_bytes);
        if (e != cudaSuccess) return fail_create(e, "merge counters");
        e = cudaDeviceSynchronize();
        if (e != cudaSuccess) return fail_create(e, "create sync");
    }
    *out = eng;
    return HKV_OK;
}

int hkv_engine_destroy(hkv_engine *eng) {
    if (eng == nullptr) {
        return HKV_ERR_INVALID;
    }
    if (eng->device_mode) {
        DeviceGuard guard(eng->cfg.device);
        cudaDeviceSynchronize();
        free_device(eng);
    }
    delete eng;
    return HKV_OK;
}

// ------------------------------------------------------------------ slots

int hkv_slot_acquire(hkv_engine *eng, int64_t capacity_hint, const hkv_prefix_key *share,
                     int32_t *slot_out) {
    if (eng == nullptr || slot_out == nullptr) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    if (capacity_hint < 0 || capacity_hint > eng->cfg.context_length) {
        return fail(eng, HKV_ERR_RANGE, "capacity %lld outside [0, %d]",
                    static_cast<long long>(capacity_hint), eng->cfg.context_length);
    }
    if (eng->free_slots.empty()) {
        return fail(eng, HKV_ERR_OOM, "all %d slots are live", eng->cfg.max_slots);
    }
    const Prefix *prefix = nullptr;
    if (share != nullptr) {
        auto it = eng->prefixes.find({share->hash, share->n_tokens});
        if (it != eng->prefixes.end()) {
            prefix = &it->second;
        }
    }
    const int64_t mapped_tokens = prefix != nullptr ? prefix->n_tokens : 0;
    int64_t reserve = 0;
    if (capacity_hint > mapped_tokens) {
        reserve = pages_for(capacity_hint) - pages_for(mapped_tokens);
        if (mapped_tokens % kPageTokens != 0) {
            ++reserve;  // the shared partial page is copied on the first append
        }
    }
    if (reserve > unreserved_free(eng)) {
        return fail(eng, HKV_ERR_OOM, "capacity %lld needs %lld pages, %lld unreserved free",
                    static_cast<long long>(capacity_hint), static_cast<long long>(reserve),
                    static_cast<long long>(unreserved_free(eng)));
    }
    const int32_t id = eng->free_slots.back();
    eng->free_slots.pop_back();
    Slot &s = eng->slots[id];
    s = Slot{};
    s.live = true;
    s.reserved = reserve;
    eng->reserved_total += reserve;
    if (prefix != nullptr) {
        s.pages = prefix->pages;
        for (int32_t p : s.pages) {
            incref(eng, p);
        }
        s.used = prefix->n_tokens;
    }
    ++eng->epoch;
    *slot_out = id;
    return HKV_OK;
}

int hkv_slot_release(hkv_engine *eng, int32_t slot) {
    if (eng == nullptr) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    if (!slot_ok(eng, slot)) {
        return fail(eng, HKV_ERR_BAD_SLOT, "release of slot %d that is not live", slot);
    }
    Slot &s = eng->slots[slot];
    for (int32_t p : s.pages) {
        decref(eng, p);
    }
    eng->reserved_total -= s.reserved;
    s = Slot{};
    eng->free_slots.push_back(slot);
    ++eng->epoch;
    return HKV_OK;
}

int hkv_slot_fork(hkv_engine *eng, int32_t src, int64_t n_tokens, int32_t *dst_out) {
    if (eng == nullptr || dst_out == nullptr) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    if (!slot_ok(eng, src)) {
        return fail(eng, HKV_ERR_BAD_SLOT, "fork of slot %d that is not live", src);
    }
    if (n_tokens < 0 || n_tokens > eng->slots[src].used) {
        return fail(eng, HKV_ERR_RANGE, "fork of %lld tokens from a slot holding %lld",
                    static_cast<long long>(n_tokens),
                    static_cast<long long>(eng->slots[src].used));
    }
    if (eng->free_slots.empty()) {
        return fail(eng, HKV_ERR_OOM, "all %d slots are live", eng->cfg.max_slots);
    }
    const int32_t id = eng->free_slots.back();
    eng->free_slots.pop_back();
    Slot &d = eng->slots[id];
    d = Slot{};
    d.live = true;
    const Slot &s = eng->slots[src];
    d.pages.assign(s.pages.begin(), s.pages.begin() + pages_for(n_tokens));
    for (int32_t p : d.pages) {
        incref(eng, p);
    }
    d.used = n_tokens;
    ++eng->epoch;
    *dst_out = id;
    return HKV_OK;
}

int hkv_slot_len(const hkv_engine *eng, int32_t slot, int64_t *used_out) {
    if (eng == nullptr || used_out == nullptr) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    if (!slot_ok(eng, slot)) {
        return fail(eng, HKV_ERR_BAD_SLOT, "slot %d is not live", slot);
    }
    *used_out = eng->slots[slot].used;
    return HKV_OK;
}

int hkv_slot_set_len(hkv_engine *eng, int32_t slot, int64_t used) {
    if (eng == nullptr) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    if (!slot_ok(eng, slot)) {
        return fail(eng, HKV_ERR_BAD_SLOT, "slot %d is not live", slot);
    }
    Slot &s = eng->slots[slot];
    if (used < 0 || used > s.used) {
        return fail(eng, HKV_ERR_RANGE, "length %lld outside [0, %lld]",
                    static_cast<long long>(used), static_cast<long long>(s.used));
    }
    const int64_t keep = pages_for(used);
    while (static_cast<int64_t>(s.pages.size()) > keep) {
        decref(eng, s.pages.back());
        s.pages.pop_back();
    }
    s.used = used;
    ++eng->epoch;
    return HKV_OK;
}

int hkv_slot_advance(hkv_engine *eng, int32_t n, const int32_t *slots, int64_t n_tokens) {
    if (eng == nullptr || (n > 0 && slots == nullptr) || n < 0) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    if (n_tokens < 0) {
        return fail(eng, HKV_ERR_RANGE, "negative advance");
    }
    for (int32_t e = 0; e < n; ++e) {
        if (!slot_ok(eng, slots[e])) {
            return fail(eng, HKV_ERR_BAD_SLOT, "slot %d is not live", slots[e]);
        }
        const Slot &s = eng->slots[slots[e]];
        if (pages_for(s.used + n_tokens) > static_cast<int64_t>(s.pages.size()) ||
            s.used + n_tokens > eng->cfg.context_length) {
            return fail(eng, HKV_ERR_RANGE,
                        "slot %d: advance to %lld past the rows written (%lld pages)", slots[e],
                        static_cast<long long>(s.used + n_tokens),
                        static_cast<long long>(s.pages.size()));
        }
    }
    for (int32_t e = 0; e < n; ++e) {
        eng->slots[slots[e]].used += n_tokens;
    }
    return HKV_OK;
}

int hkv_prefix_publish(hkv_engine *eng, const hkv_prefix_key *key, int32_t slot) {
    if (eng == nullptr || key == nullptr) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    if (!slot_ok(eng, slot)) {
        return fail(eng, HKV_ERR_BAD_SLOT, "slot %d is not live", slot);
    }
    const Slot &s = eng->slots[slot];
    if (key->n_tokens <= 0 || key->n_tokens > s.used) {
        return fail(eng, HKV_ERR_RANGE, "prefix of %lld tokens from a slot holding %lld",
                    static_cast<long long>(key->n_tokens), static_cast<long long>(s.used));
    }
    const auto k = std::make_pair(key->hash, key->n_tokens);
    if (eng->prefixes.count(k) != 0) {
        return fail(eng, HKV_ERR_INVALID, "prefix key already published");
    }
    Prefix p;
    p.n_tokens = key->n_tokens;
    p.pages.assign(s.pages.begin(), s.pages.begin() + pages_for(key->n_tokens));
    for (int32_t page : p.pages) {
        incref(eng, page);
    }
    eng->prefixes.emplace(k, std::move(p));
    ++eng->epoch;
    return HKV_OK;
}

int hkv_prefix_drop(hkv_engine *eng, const hkv_prefix_key *key) {
    if (eng == nullptr || key == nullptr) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    auto it = eng->prefixes.find({key->hash, key->n_tokens});
    if (it == eng->prefixes.end()) {
        return fail(eng, HKV_ERR_NOT_FOUND, "prefix key not published");
    }
    for (int32_t page : it->second.pages) {
        decref(eng, page);
    }
    eng->prefixes.erase(it);
    ++eng->epoch;
    return HKV_OK;
}

int hkv_slot_pages(const hkv_engine *eng, int32_t slot, int32_t *pages_out, int64_t cap,
                   int64_t *n_out) {
    if (eng == nullptr || n_out == nullptr || (cap > 0 && pages_out == nullptr)) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    if (!slot_ok(eng, slot)) {
        return fail(eng, HKV_ERR_BAD_SLOT, "slot %d is not live", slot);
    }
    const Slot &s = eng->slots[slot];
    *n_out = static_cast<int64_t>(s.pages.size());
    const int64_t m = std::min<int64_t>(cap, *n_out);
    if (m > 0) {
        std::memcpy(pages_out, s.pages.data(), static_cast<size_t>(m) * sizeof(int32_t));
    }
    return HKV_OK;
}

int hkv_engine_config(const hkv_engine *eng, hkv_config *out) {
    if (eng == nullptr || out == nullptr) {
        return HKV_ERR_INVALID;
    }
    *out = eng->cfg;
    return HKV_OK;
}

int hkv_pool_stats_get(const hkv_engine *eng, hkv_pool_stats *out) {
    if (eng == nullptr || out == nullptr) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    out->n_pages = eng->cfg.n_pages;
    out->free_pages = static_cast<int64_t>(eng->free_pages.size());
    out->reserved = eng->reserved_total;
    out->shared_pages = eng->shared_pages;
    out->live_slots = eng->cfg.max_slots - static_cast<int32_t>(eng->free_slots.size());
    out->prefixes = static_cast<int32_t>(eng->prefixes.size());
    out->page_bytes = eng->page_bytes;
    out->cow_copies = eng->cow_copies;
    out->kernel_launches = eng->kernel_launches;
    return HKV_OK;
}

// ---------------------------------------------------------------- compute

int hkv_append(hkv_engine *eng, int32_t layer, int32_t n, const int32_t *slots, const float *k,
               const float *v, hkv_stream stream) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    DeviceGuard guard(eng->cfg.device);
    return do_append(eng, layer, n, slots, k, v, false, static_cast<cudaStream_t>(stream));
}

int hkv_rope_append(hkv_engine *eng, int32_t layer, int32_t n, const int32_t *slots,
                    const float *k_prerope, const float *v, hkv_stream stream) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    DeviceGuard guard(eng->cfg.device);
    return do_append(eng, layer, n, slots, k_prerope, v, true, static_cast<cudaStream_t>(stream));
}

int hkv_rope_append_range(hkv_engine *eng, int32_t layer, int32_t slot, int64_t n_tokens,
                          const float *k_prerope, const float *v, hkv_stream stream_h) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    DeviceGuard guard(eng->cfg.device);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_h);
    int st = check_compute(eng, layer);
    if (st != HKV_OK) return st;
    if (!slot_ok(eng, slot)) {
        return fail(eng, HKV_ERR_BAD_SLOT, "slot %d is not live", slot);
    }
    if (k_prerope == nullptr || v == nullptr || !aligned16(k_prerope) || !aligned16(v)) {
        return fail(eng, HKV_ERR_INVALID, "k and v must be non-null 16-byte aligned device pointers");
    }
    Slot &s = eng->slots[slot];
    if (n_tokens <= 0 || s.used + n_tokens > eng->cfg.context_length) {
        return fail(eng, HKV_ERR_RANGE, "range [%lld, %lld) outside the context of %d",
                    static_cast<long long>(s.used), static_cast<long long>(s.used + n_tokens),
                    eng->cfg.context_length);
    }
    const int64_t begin = s.used;
    const int64_t end = s.used + n_tokens;
    const int64_t extra = pages_beyond_reservation(s, pages_needed(eng, s, begin, end));
    if (extra > unreserved_free(eng)) {
        return fail(eng, HKV_ERR_OOM, "range needs %lld unreserved pages, %lld free",
                    static_cast<long long>(extra), static_cast<long long>(unreserved_free(eng)));
    }
    st = own_rows(eng, s, begin, end, stream);
    if (st != HKV_OK) return st;
    st = flush_cow(eng, stream);
    if (st != HKV_OK) return st;
    const int64_t p0 = begin / kPageTokens;
    const int64_t p1 = (end - 1) / kPageTokens + 1;
    void *host = nullptr;
    const size_t bytes = static_cast<size_t>(p1 - p0) * sizeof(int32_t);
    HKV_CUDA_TRY(eng, eng->range_stage.begin(bytes, &host));
    std::memcpy(host, s.pages.data() + p0, bytes);
    void *dev = nullptr;
    ++eng->enqueue_seq;
    HKV_CUDA_TRY(eng, eng->range_stage.commit(bytes, stream, &dev));
    {
        ProfileScope ps(eng, HKV_KERNEL_APPEND, stream);
        launch_append_range(pool_view(eng), rope_view(eng), static_cast<const int32_t *>(dev),
                            begin, n_tokens, layer, k_prerope, v, true, eng->d_err, stream);
        ++eng->kernel_launches;
    }
    HKV_CUDA_TRY(eng, eng->range_stage.mark_used(stream));
    return launch_status(eng, "range append kernel launch");
}

int hkv_decode_attn(hkv_engine *eng, int32_t layer, int32_t n, const int32_t *slots,
                    const float *q_prerope, float *out, hkv_stream stream_h) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    HostTimer host_timer(eng);
    std::lock_guard<std::mutex> lock(eng->mu);
    DeviceGuard guard(eng->cfg.device);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_h);
    int st = check_compute(eng, layer);
    if (st != HKV_OK) return st;
    if (q_prerope == nullptr || out == nullptr || !aligned16(q_prerope) || !aligned16(out)) {
        return fail(eng, HKV_ERR_INVALID, "q and out must be non-null 16-byte aligned device pointers");
    }
    st = ensure_batch(eng, n, slots, stream);
    if (st != HKV_OK) return st;
    return do_attention(eng, layer, q_prerope, nullptr, nullptr, out, stream);
}

int hkv_decode_step(hkv_engine *eng, int32_t layer, int32_t n, const int32_t *slots,
                    const float *q_prerope, const float *k_prerope, const float *v, float *out,
                    hkv_stream stream_h) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    HostTimer host_timer(eng);
    std::lock_guard<std::mutex> lock(eng->mu);
    DeviceGuard guard(eng->cfg.device);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_h);
    if (q_prerope == nullptr || out == nullptr || !aligned16(q_prerope) || !aligned16(out)) {
        return fail(eng, HKV_ERR_INVALID, "q and out must be non-null 16-byte aligned device pointers");
    }
    int st = check_compute(eng, layer);
    if (st != HKV_OK) return st;
    if (k_prerope == nullptr || v == nullptr || !aligned16(k_prerope) || !aligned16(v)) {
        return fail(eng, HKV_ERR_INVALID, "k and v must be non-null 16-byte aligned device pointers");
    }
    st = ensure_batch(eng, n, slots, stream);
    if (st != HKV_OK) return st;
    return do_attention(eng, layer, q_prerope, k_prerope, v, out, stream);
}

int hkv_gather(hkv_engine *eng, int32_t slot, int32_t layer, int64_t pos0, int64_t n,
               uint16_t *k_out, uint16_t *v_out, hkv_stream stream_h) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    DeviceGuard guard(eng->cfg.device);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_h);
    int st = check_compute(eng, layer);
    if (st != HKV_OK) return st;
    if (!slot_ok(eng, slot)) {
        return fail(eng, HKV_ERR_BAD_SLOT, "slot %d is not live", slot);
    }
    if (k_out == nullptr || v_out == nullptr || !aligned16(k_out) || !aligned16(v_out)) {
        return fail(eng, HKV_ERR_INVALID, "outputs must be non-null 16-byte aligned device pointers");
    }
    const Slot &s = eng->slots[slot];
    const int64_t covered = static_cast<int64_t>(s.pages.size()) * kPageTokens;
    if (pos0 < 0 || n <= 0 || pos0 + n > covered) {
        return fail(eng, HKV_ERR_RANGE, "gather [%lld, %lld) outside the %lld mapped rows",
                    static_cast<long long>(pos0), static_cast<long long>(pos0 + n),
                    static_cast<long long>(covered));
    }
    void *host = nullptr;
    const size_t bytes = s.pages.size() * sizeof(int32_t);
    HKV_CUDA_TRY(eng, eng->gather_stage.begin(bytes, &host));
    std::memcpy(host, s.pages.data(), bytes);
    void *dev = nullptr;
    ++eng->enqueue_seq;
    HKV_CUDA_TRY(eng, eng->gather_stage.commit(bytes, stream, &dev));
    {
        ProfileScope ps(eng, HKV_KERNEL_GATHER, stream);
        launch_gather(pool_view(eng), static_cast<const int32_t *>(dev), pos0, n, layer, k_out,
                      v_out, eng->d_err, stream);
        ++eng->kernel_launches;
    }
    HKV_CUDA_TRY(eng, eng->gather_stage.mark_used(stream));
    return launch_status(eng, "gather kernel launch");
}

int hkv_sync_check(hkv_engine *eng, hkv_stream stream) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    if (!eng->device_mode) {
        return fail(eng, HKV_ERR_NO_DEVICE, "engine was created without a device");
    }
    DeviceGuard guard(eng->cfg.device);
    HKV_CUDA_TRY(eng, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    DeviceError err{};
    HKV_CUDA_TRY(eng, cudaMemcpy(&err, eng->d_err, sizeof(err), cudaMemcpyDeviceToHost));
    if (err.code != 0) {
        HKV_CUDA_TRY(eng, cudaMemset(eng->d_err, 0, sizeof(DeviceError)));
        if (err.code == kErrTimeout) {
            return fail(eng, HKV_ERR_TIMEOUT, "kernel %d gave up waiting (unit %d, block %d)",
                        err.where, err.a, err.b);
        }
        return fail(eng, HKV_ERR_DEVICE, "kernel %d bounds check: values %d, %d", err.where,
                    err.a, err.b);
    }
    return HKV_OK;
}

int hkv_rope_tables(const hkv_engine *eng, float *cos_out, float *sin_out) {
    if (eng == nullptr || cos_out == nullptr || sin_out == nullptr) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    std::memcpy(cos_out, eng->rope_cos.data(), eng->rope_cos.size() * sizeof(float));
    std::memcpy(sin_out, eng->rope_sin.data(), eng->rope_sin.size() * sizeof(float));
    return HKV_OK;
}

// ---------------------------------------------------------- KV-head split

int hkv_split_export(hkv_engine *eng, int32_t world, int32_t rank, void *handle_out) {
    if (eng == nullptr || handle_out == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    if (!eng->device_mode) {
        return fail(eng, HKV_ERR_NO_DEVICE, "engine was created without a device");
    }
    if (world < 1 || rank < 0 || rank >= world) {
        return fail(eng, HKV_ERR_INVALID, "rank %d outside a world of %d", rank, world);
    }
    DeviceGuard guard(eng->cfg.device);
    free_split(eng);
    eng->xchg_flags_bytes = (static_cast<size_t>(eng->cfg.n_layers) * sizeof(uint32_t) + 255) & ~size_t(255);
    eng->xchg_row_floats = world * kGqa * eng->cfg.n_head_kv * kHeadDim;
    const size_t bytes = eng->xchg_flags_bytes + static_cast<size_t>(eng->cfg.n_layers) *
                                                     eng->cfg.max_slots * eng->xchg_row_floats *
                                                     sizeof(float);
    HKV_CUDA_TRY(eng, cudaMalloc(&eng->xchg, bytes));
    HKV_CUDA_TRY(eng, cudaMemset(eng->xchg, 0, bytes));
    cudaIpcMemHandle_t h;
    HKV_CUDA_TRY(eng, cudaIpcGetMemHandle(&h, eng->xchg));
    std::memcpy(handle_out, &h, sizeof(h));
    eng->split_world = world;
    eng->split_rank = rank;
    eng->split_target.assign(static_cast<size_t>(eng->cfg.n_layers), 0u);
    HKV_CUDA_TRY(eng, cudaDeviceSynchronize());
    return HKV_OK;
}

int hkv_split_connect(hkv_engine *eng, const void *handles) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    if (eng->xchg == nullptr) {
        return fail(eng, HKV_ERR_INVALID, "hkv_split_export first");
    }
    DeviceGuard guard(eng->cfg.device);
    if (handles == nullptr) {
        // Disconnect: close the peers' mappings, keep this rank's region.
        HKV_CUDA_TRY(eng, cudaDeviceSynchronize());
        for (void *p : eng->peer_bases) {
            if (p != nullptr) {
                HKV_CUDA_TRY(eng, cudaIpcCloseMemHandle(p));
            }
        }
        eng->peer_bases.clear();
        cudaFree(eng->d_outs);
        cudaFree(eng->d_flags);
        eng->d_outs = nullptr;
        eng->d_flags = nullptr;
        eng->split_connected = false;
        return HKV_OK;
    }
    const int32_t world = eng->split_world;
    eng->peer_bases.assign(static_cast<size_t>(world), nullptr);
    std::vector<float *> outs(static_cast<size_t>(world));
    std::vector<uint32_t *> flags(static_cast<size_t>(world));
    for (int32_t r = 0; r < world; ++r) {
        uint8_t *base = eng->xchg;
        if (r != eng->split_rank) {
            cudaIpcMemHandle_t h;
            std::memcpy(&h, static_cast<const uint8_t *>(handles) + r * sizeof(h), sizeof(h));
            void *p = nullptr;
            const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
            if (e != cudaSuccess) {
                return cuda_fail(eng, e, "cudaIpcOpenMemHandle of a peer's exchange region");
            }
            eng->peer_bases[r] = p;
            base = static_cast<uint8_t *>(p);
        }
        flags[r] = reinterpret_cast<uint32_t *>(base);
        outs[r] = reinterpret_cast<float *>(base + eng->xchg_flags_bytes);  // layer 0 block
    }
    HKV_CUDA_TRY(eng, cudaMalloc(&eng->d_outs, world * sizeof(float *)));
    HKV_CUDA_TRY(eng, cudaMalloc(&eng->d_flags, world * sizeof(uint32_t *)));
    HKV_CUDA_TRY(eng, cudaMemcpy(eng->d_outs, outs.data(), world * sizeof(float *),
                                 cudaMemcpyHostToDevice));
    HKV_CUDA_TRY(eng, cudaMemcpy(eng->d_flags, flags.data(), world * sizeof(uint32_t *),
                                 cudaMemcpyHostToDevice));
    eng->split_connected = true;
    return HKV_OK;
}

int hkv_split_step(hkv_engine *eng, int32_t layer, int32_t n, const int32_t *slots,
                   const float *q_prerope, const float *k_prerope, const float *v,
                   hkv_stream stream_h) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    DeviceGuard guard(eng->cfg.device);
    cudaStream_t stream = static_cast<cudaStream_t>(stream_h);
    int st = check_compute(eng, layer);
    if (st != HKV_OK) return st;
    if (!eng->split_connected) {
        return fail(eng, HKV_ERR_INVALID, "hkv_split_connect first");
    }
    if (q_prerope == nullptr || k_prerope == nullptr || v == nullptr || !aligned16(q_prerope) ||
        !aligned16(k_prerope) || !aligned16(v)) {
        return fail(eng, HKV_ERR_INVALID, "q, k and v must be non-null 16-byte aligned device pointers");
    }
    st = ensure_batch(eng, n, slots, stream);
    if (st != HKV_OK) return st;
    Exchange x;
    x.outs = eng->d_outs;
    x.flags = eng->d_flags;
    x.n_ranks = eng->split_world;
    x.row_floats = eng->xchg_row_floats;
    x.col_off = eng->split_rank * kGqa * eng->cfg.n_head_kv * kHeadDim;
    x.layer_floats = static_cast<int64_t>(eng->cfg.max_slots) * eng->xchg_row_floats;
    st = do_attention(eng, layer, q_prerope, k_prerope, v, nullptr, stream, x);
    if (st != HKV_OK) return st;
    // every rank signals once per (entry, KV head) its attention launch
    // finishes, and -- when split partials go through the combine launch --
    // once per query head of every segment that launch finishes
    const uint32_t whole = static_cast<uint32_t>(n) * eng->cfg.n_head_kv - eng->batch.view.split_segments;
    const uint32_t per_split = eng->batch.view.combine ? kGqa : 1;
    eng->split_target[layer] +=
        (whole + per_split * static_cast<uint32_t>(eng->batch.view.split_segments)) * eng->split_world;
    return HKV_OK;
}

int hkv_split_wait(hkv_engine *eng, int32_t layer, hkv_stream stream_h) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    DeviceGuard guard(eng->cfg.device);
    int st = check_compute(eng, layer);
    if (st != HKV_OK) return st;
    if (!eng->split_connected) {
        return fail(eng, HKV_ERR_INVALID, "hkv_split_connect first");
    }
    // The wait writes neither the pool nor a plan, so the next decode launch
    // may still overlap it (enqueue_seq stays).
    launch_split_wait(reinterpret_cast<const uint32_t *>(eng->xchg) + layer,
                      eng->split_target[layer], eng->d_err, static_cast<cudaStream_t>(stream_h));
    ++eng->kernel_launches;
    return launch_status(eng, "split wait launch");
}

int hkv_split_output(const hkv_engine *eng, int32_t layer, float **out_dev, int64_t *row_floats) {
    if (eng == nullptr || out_dev == nullptr || row_floats == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    if (eng->xchg == nullptr) {
        return fail(eng, HKV_ERR_INVALID, "hkv_split_export first");
    }
    if (layer < 0 || layer >= eng->cfg.n_layers) {
        return fail(eng, HKV_ERR_RANGE, "layer %d outside [0, %d)", layer, eng->cfg.n_layers);
    }
    *out_dev = reinterpret_cast<float *>(eng->xchg + eng->xchg_flags_bytes) +
               static_cast<int64_t>(layer) * eng->cfg.max_slots * eng->xchg_row_floats;
    *row_floats = eng->xchg_row_floats;
    return HKV_OK;
}

// -------------------------------------------------------------- profiling

int hkv_profile_enable(hkv_engine *eng, int on) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    if (!eng->device_mode) {
        return fail(eng, HKV_ERR_NO_DEVICE, "engine was created without a device");
    }
    eng->profiling = on != 0;
    return HKV_OK;
}

int hkv_profile_reset(hkv_engine *eng) {
    if (eng == nullptr) return HKV_ERR_INVALID;
    std::lock_guard<std::mutex> lock(eng->mu);
    if (!eng->device_mode) {
        return fail(eng, HKV_ERR_NO_DEVICE, "engine was created without a device");
    }
    DeviceGuard guard(eng->cfg.device);
    for (auto &list : eng->prof) {
        for (auto &r : list) {
            cudaEventSynchronize(r.stop);
            eng->event_pool.push_back(r.start);
            eng->event_pool.push_back(r.stop);
        }
        list.clear();
    }
    return HKV_OK;
}

int hkv_host_stats(hkv_engine *eng, int64_t *calls, double *host_us, double *blocked_us,
                   int reset) {
    if (eng == nullptr || calls == nullptr || host_us == nullptr || blocked_us == nullptr) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->host_mu);
    *calls = eng->host_calls;
    *host_us = static_cast<double>(eng->host_ns) * 1e-3;
    *blocked_us = static_cast<double>(eng->launch_ns + eng->staging_wait_ns) * 1e-3;
    if (reset) {
        eng->host_calls = 0;
        eng->host_ns = 0;
        eng->launch_ns = 0;
        eng->staging_wait_ns = 0;
    }
    return HKV_OK;
}

int hkv_profile_read(hkv_engine *eng, int kernel_id, int64_t *launches, double *total_ms) {
    if (eng == nullptr || launches == nullptr || total_ms == nullptr || kernel_id < 0 ||
        kernel_id >= HKV_KERNEL_COUNT) {
        return HKV_ERR_INVALID;
    }
    std::lock_guard<std::mutex> lock(eng->mu);
    if (!eng->device_mode) {
        return fail(eng, HKV_ERR_NO_DEVICE, "engine was created without a device");
    }
    DeviceGuard guard(eng->cfg.device);
    double total = 0.0;
    for (auto &r : eng->prof[kernel_id]) {
        HKV_CUDA_TRY(eng, cudaEventSynchronize(r.stop));
        float ms = 0.f;
        HKV_CUDA_TRY(eng, cudaEventElapsedTime(&ms, r.start, r.stop));
        total += ms;
    }
    *launches = static_cast<int64_t>(eng->prof[kernel_id].size());
    *total_ms = total;
    return HKV_OK;
}

}  // extern "C"
