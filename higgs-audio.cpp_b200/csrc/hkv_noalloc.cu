// hkv_noalloc.cu -- decode attention for callers that cannot allocate GPU memory.
//
// Some callers of this library may not call cudaMalloc at all: code that runs
// inside another framework's memory pool (the pipeline's ggml backend buffers
// hold every tensor, and a second allocator on the same device would fragment
// or exceed its budget), or code on a hot path where an allocation could
// block or fail.  hkv_decode_attn_noalloc serves them: it takes device memory
// the caller already owns (a page pool in the engine's layout, the RoPE
// tables, q, out) and keeps its own working memory -- the batch descriptor,
// the split-K partials, the merge counters and the device error word -- in one file-scope
// __device__ array of fixed size, so no call allocates device memory.
//
// The array is kNoAllocScratchBytes (8 MiB) on every GPU that loads the
// library, held until the process exits.  All calls share it: calls that
// overlap on the GPU (different streams, or several host threads) race on it,
// so order them.  Each call rewrites the plan and clears the merge counters it
// uses.  The error word is not cleared by a call: a kernel that gives up on a
// bounded wait or meets a bad page id records the first such error there, and
// it stays until hkv_decode_attn_noalloc_sync_check reads and clears it.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "../../include/hkv.h"
#include "hkv_internal.h"
#include "hkv_plan.h"

namespace hkv {
namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;
constexpr int kMaxDevices = 64;

// Device code could name this array directly; host code may not: on the host
// `g_noalloc_scratch` is only a stand-in symbol, so its address is looked up
// with cudaGetSymbolAddress (once per device, that device current).
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mu;
unsigned char *g_scratch_ptr[kMaxDevices] = {};
int g_num_sms[kMaxDevices] = {};

void set_msg(char *buf, size_t len, const char *fmt, ...) __attribute__((format(printf, 3, 4)));
void set_msg(char *buf, size_t len, const char *fmt, ...) {
    if (buf == nullptr || len == 0) return;
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, len, fmt, ap);
    va_end(ap);
}

size_t align256(size_t x) { return (x + 255) & ~size_t(255); }

}  // namespace
}  // namespace hkv

using namespace hkv;

namespace hkv {
namespace {

// Device address of the static array for the current device, looked up once
// per device (with that device current); HKV_OK or HKV_ERR_CUDA.
int scratch_for_current_device(unsigned char **scratch, int *num_sms, char *err_msg,
                               size_t err_len) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        set_msg(err_msg, err_len, "no current CUDA device");
        return HKV_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (g_scratch_ptr[dev] == nullptr) {
        void *ptr = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
        if (e != cudaSuccess || ptr == nullptr) {
            set_msg(err_msg, err_len, "cudaGetSymbolAddress of the static scratch: %s",
                    cudaGetErrorString(e));
            return HKV_ERR_CUDA;
        }
        int sms = 0;
        e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
        if (e != cudaSuccess || sms <= 0) {
            set_msg(err_msg, err_len, "SM count: %s", cudaGetErrorString(e));
            return HKV_ERR_CUDA;
        }
        g_num_sms[dev] = sms;
        g_scratch_ptr[dev] = static_cast<unsigned char *>(ptr);
    }
    *scratch = g_scratch_ptr[dev];
    if (num_sms != nullptr) {
        *num_sms = g_num_sms[dev];
    }
    return HKV_OK;
}

// Scratch layout of one call:
//   [error word][merge counters][descriptor][partials o][partials m, l]
// (segment counters then group counters; level-1 then group partials).
struct ScratchLayout {
    size_t cnt_off, desc_off, po_off, pml_off, need;
};
ScratchLayout scratch_layout(size_t n_counters, size_t words, size_t n_partials) {
    ScratchLayout l;
    l.cnt_off = align256(sizeof(DeviceError));
    l.desc_off = align256(l.cnt_off + n_counters * sizeof(int32_t));
    l.po_off = align256(l.desc_off + words * sizeof(int32_t));
    l.pml_off = align256(l.po_off + n_partials * kGqa * kHeadDim * sizeof(float));
    l.need = l.pml_off + n_partials * 2 * kGqa * sizeof(float);
    return l;
}

}  // namespace
}  // namespace hkv

extern "C" int hkv_decode_attn_noalloc(const hkv_paged_view *view, int32_t layer, int32_t n,
                                       const int32_t *pos, const int32_t *page_off,
                                       const int32_t *pages, const float *q_prerope, float *out,
                                       hkv_stream stream_h, char *err_msg, size_t err_len) {
    set_msg(err_msg, err_len, "%s", "");
    cudaStream_t stream = static_cast<cudaStream_t>(stream_h);
    if (view == nullptr || pos == nullptr || page_off == nullptr || pages == nullptr ||
        q_prerope == nullptr || out == nullptr || view->pool == nullptr ||
        view->rope_cos == nullptr || view->rope_sin == nullptr) {
        set_msg(err_msg, err_len, "null argument");
        return HKV_ERR_INVALID;
    }
    const uintptr_t mis = reinterpret_cast<uintptr_t>(q_prerope) | reinterpret_cast<uintptr_t>(out) |
                          reinterpret_cast<uintptr_t>(view->pool);
    if ((mis & 15u) != 0) {
        set_msg(err_msg, err_len, "q, out and the pool must be 16-byte aligned");
        return HKV_ERR_INVALID;
    }
    const int32_t G = view->n_head_kv;
    if (n <= 0 || G <= 0 || view->n_layers <= 0 || view->n_pages <= 0 ||
        view->n_pages > INT32_MAX || view->context_length <= 0) {
        set_msg(err_msg, err_len, "bad shape: n=%d n_head_kv=%d n_layers=%d", n, G,
                view->n_layers);
        return HKV_ERR_INVALID;
    }
    if (layer < 0 || layer >= view->n_layers) {
        set_msg(err_msg, err_len, "layer %d outside [0, %d)", layer, view->n_layers);
        return HKV_ERR_RANGE;
    }

    // ---- per-device set-up (first call on each device)
    unsigned char *scratch = nullptr;
    int num_sms = 0;
    const int st = scratch_for_current_device(&scratch, &num_sms, err_msg, err_len);
    if (st != HKV_OK) {
        return st;
    }

    // ---- host-side plan (the same stream-K split the engine uses)
    int64_t total_pages = 0;
    for (int32_t e = 0; e < n; ++e) {
        if (pos[e] < 0 || pos[e] >= view->context_length) {
            set_msg(err_msg, err_len, "entry %d: position %d outside [0, %d)", e, pos[e],
                    view->context_length);
            return HKV_ERR_RANGE;
        }
        const int32_t np = pos[e] / kPageTokens + 1;
        if (page_off[e + 1] - page_off[e] < np || page_off[e] < 0) {
            set_msg(err_msg, err_len, "entry %d: %d pages listed, position %d needs %d", e,
                    page_off[e + 1] - page_off[e], pos[e], np);
            return HKV_ERR_RANGE;
        }
        for (int32_t i = 0; i < np; ++i) {
            const int32_t p = pages[page_off[e] + i];
            if (p < 0 || p >= view->n_pages) {
                set_msg(err_msg, err_len, "entry %d: page %d outside the pool of %lld", e, p,
                        static_cast<long long>(view->n_pages));
                return HKV_ERR_RANGE;
            }
        }
        total_pages += np;
    }
    if (total_pages * G > INT32_MAX / 2) {
        set_msg(err_msg, err_len, "batch too large (%lld units)",
                static_cast<long long>(total_pages * G));
        return HKV_ERR_RANGE;
    }
    const int32_t W = plan_warps(total_pages * G, static_cast<int64_t>(num_sms) * kAttnWarps);
    const size_t words = plan_words(n, G, total_pages, W);
    // Before any host work that grows with the batch: the largest layout the
    // plan can need.  A segment has one partial per warp (or CTA) it spans, so
    // level-1 partials are at most W + S - 1 (a warp's share starts inside at
    // most one segment it does not finish), and only a segment with p > 16 of
    // them adds group partials and counters, ceil(p / 8) or fewer, so at most
    // parts / 8 + parts / 17 over the batch.
    const size_t S = static_cast<size_t>(n) * G;
    const size_t parts_bound = static_cast<size_t>(W) + S;
    const size_t groups_bound = parts_bound / 8 + parts_bound / 17 + 1;
    const ScratchLayout bound = scratch_layout(S + groups_bound, words, parts_bound + groups_bound);
    if (bound.need > kNoAllocScratchBytes) {
        set_msg(err_msg, err_len,
                "batch may need up to %zu bytes of scratch (%zu descriptor words); the "
                "static scratch holds %zu bytes: split the batch",
                bound.need, words, kNoAllocScratchBytes);
        return HKV_ERR_RANGE;
    }
    std::vector<int32_t> w(words);
    std::vector<const int32_t *> lists(static_cast<size_t>(n));
    for (int32_t e = 0; e < n; ++e) {
        lists[e] = pages + page_off[e];
    }
    const PlanSummary plan = build_plan(w.data(), n, G, pos, lists.data(), total_pages, W);

    const size_t n_counters = S + plan.n_groups;
    const size_t n_partials = static_cast<size_t>(plan.n_parts) + plan.n_groups;
    const ScratchLayout lay = scratch_layout(n_counters, words, n_partials);
    if (lay.need > bound.need) {  // the bound above is a theorem of the plan; keep it honest
        set_msg(err_msg, err_len, "internal: plan needs %zu bytes, bound was %zu", lay.need,
                bound.need);
        return HKV_ERR_INVALID;
    }
    const size_t cnt_off = lay.cnt_off;
    const size_t desc_off = lay.desc_off;
    const size_t po_off = lay.po_off;
    const size_t pml_off = lay.pml_off;
    DeviceError *err = reinterpret_cast<DeviceError *>(scratch);
    int32_t *counters = reinterpret_cast<int32_t *>(scratch + cnt_off);
    int32_t *d = reinterpret_cast<int32_t *>(scratch + desc_off);
    float *part_o = reinterpret_cast<float *>(scratch + po_off);
    float *part_ml = reinterpret_cast<float *>(scratch + pml_off);
    // The merge counters must start at zero (a call that gave up part way can
    // leave some set); the error word keeps its first record until
    // hkv_decode_attn_noalloc_sync_check reads it.
    cudaError_t e = cudaMemsetAsync(scratch + cnt_off, 0, desc_off - cnt_off, stream);
    if (e == cudaSuccess) {
        e = cudaMemcpyAsync(d, w.data(), words * sizeof(int32_t), cudaMemcpyHostToDevice, stream);
    }
    if (e != cudaSuccess) {
        set_msg(err_msg, err_len, "descriptor upload: %s", cudaGetErrorString(e));
        return HKV_ERR_CUDA;
    }
    const BatchView b = bind_plan(d, n, G, plan, W);
    PoolView pv;
    pv.base = static_cast<uint8_t *>(view->pool);
    pv.n_pages = view->n_pages;
    pv.n_layers = view->n_layers;
    pv.n_head_kv = G;
    RopeView rv;
    rv.cos_tab = view->rope_cos;
    rv.sin_tab = view->rope_sin;
    rv.context_length = view->context_length;
    const float scale_log2 =
        (1.0f / std::sqrt(static_cast<float>(kHeadDim))) * 1.4426950408889634f;
    const Exchange no_exchange{nullptr, nullptr, 0, 0, 0, 0};
    launch_attention(pv, rv, b, layer, q_prerope, nullptr, nullptr, part_o, part_ml, counters, out,
                     no_exchange, scale_log2, err, /*overlap_previous=*/false, stream);
    e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_msg(err_msg, err_len, "kernel launch: %s", cudaGetErrorString(e));
        return HKV_ERR_CUDA;
    }
    return HKV_OK;
}

extern "C" int hkv_decode_attn_noalloc_sync_check(hkv_stream stream_h, char *err_msg,
                                                  size_t err_len) {
    set_msg(err_msg, err_len, "%s", "");
    cudaError_t e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream_h));
    if (e != cudaSuccess) {
        set_msg(err_msg, err_len, "stream synchronize: %s", cudaGetErrorString(e));
        return HKV_ERR_CUDA;
    }
    unsigned char *scratch = nullptr;
    const int st = scratch_for_current_device(&scratch, nullptr, err_msg, err_len);
    if (st != HKV_OK) {
        return st;
    }
    DeviceError rec{};
    e = cudaMemcpy(&rec, scratch, sizeof(rec), cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
        set_msg(err_msg, err_len, "reading the error word: %s", cudaGetErrorString(e));
        return HKV_ERR_CUDA;
    }
    if (rec.code == 0) {
        return HKV_OK;
    }
    e = cudaMemset(scratch, 0, sizeof(DeviceError));
    if (e != cudaSuccess) {
        set_msg(err_msg, err_len, "clearing the error word: %s", cudaGetErrorString(e));
        return HKV_ERR_CUDA;
    }
    if (rec.code == kErrTimeout) {
        set_msg(err_msg, err_len,
                "hkv_decode_attn_noalloc: a bounded wait gave up (unit %d, block %d); that "
                "call's output is invalid", rec.a, rec.b);
        return HKV_ERR_TIMEOUT;
    }
    set_msg(err_msg, err_len,
            "hkv_decode_attn_noalloc: bounds check failed (page %d, entry %d); that call's "
            "output is invalid", rec.a, rec.b);
    return HKV_ERR_DEVICE;
}
