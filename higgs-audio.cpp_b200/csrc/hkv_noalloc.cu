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
// so order them.  Each call rewrites what it reads, and clears the error word.
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
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        set_msg(err_msg, err_len, "no current CUDA device");
        return HKV_ERR_CUDA;
    }
    unsigned char *scratch = nullptr;
    {
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
        scratch = g_scratch_ptr[dev];
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
    const int32_t W = plan_warps(total_pages * G, static_cast<int64_t>(g_num_sms[dev]) * kAttnWarps);
    const size_t words = plan_words(n, G, total_pages, W);
    std::vector<int32_t> w(words);
    std::vector<const int32_t *> lists(static_cast<size_t>(n));
    for (int32_t e = 0; e < n; ++e) {
        lists[e] = pages + page_off[e];
    }
    const PlanSummary plan = build_plan(w.data(), n, G, pos, lists.data(), total_pages, W);

    // ---- carve the static scratch:
    //      [error word][merge counters][descriptor][partials o][partials m, l]
    // segment counters then group counters; level-1 then group partials
    const size_t n_counters = static_cast<size_t>(n) * G + plan.n_groups;
    const size_t n_partials = static_cast<size_t>(plan.n_parts) + plan.n_groups;
    const size_t cnt_off = align256(sizeof(DeviceError));
    const size_t desc_off = align256(cnt_off + n_counters * sizeof(int32_t));
    const size_t po_off = align256(desc_off + words * sizeof(int32_t));
    const size_t pml_off = align256(po_off + n_partials * kGqa * kHeadDim * sizeof(float));
    const size_t need = pml_off + n_partials * 2 * kGqa * sizeof(float);
    if (need > kNoAllocScratchBytes) {
        set_msg(err_msg, err_len,
                "batch needs %zu bytes of scratch (%zu partials, %zu descriptor words); the "
                "static scratch holds %zu bytes: split the batch",
                need, n_partials, words, kNoAllocScratchBytes);
        return HKV_ERR_RANGE;
    }
    DeviceError *err = reinterpret_cast<DeviceError *>(scratch);
    int32_t *counters = reinterpret_cast<int32_t *>(scratch + cnt_off);
    int32_t *d = reinterpret_cast<int32_t *>(scratch + desc_off);
    float *part_o = reinterpret_cast<float *>(scratch + po_off);
    float *part_ml = reinterpret_cast<float *>(scratch + pml_off);
    // The error word and the merge counters must start at zero; the array
    // keeps whatever the previous call left.
    cudaError_t e = cudaMemsetAsync(scratch, 0, desc_off, stream);
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
