// hkv_internal.h -- shapes, the page layout and the kernel launch interface
// shared by the host engine (hkv_engine.cpp) and the kernels (hkv_kernels.cu).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace hkv {

// The kernels are specialised for the HiggsAudioV3 / Qwen3-4B attention
// shape: head_dim 128, 4 query heads per KV head, 16-token pages.
constexpr int kHeadDim = 128;
constexpr int kGqa = 4;
constexpr int kPageTokens = 16;
// One head block: 16 token rows x 128 dims of F16 = 4 KiB, contiguous.
constexpr int kHeadBlockBytes = kPageTokens * kHeadDim * 2;
constexpr int kRowBytes = kHeadDim * 2;  // 256 B, 16 chunks of 16 B

// Page layout in HBM (layer-major: one decode launch reads one layer, and its
// reads then stay inside that layer's contiguous slab of n_pages * 64 KiB,
// which keeps the GPU's address translation working set small):
//   block(page, layer, kv, head) = ((layer * n_pages + page) * 2 + kv) * n_head_kv + head
//   byte(page, layer, kv, head, row, chunk) =
//       block * 4096 + row * 256 + (chunk ^ (row & 7)) * 16
// where kv = 0 for K and 1 for V, row = position % 16 and chunk = dim / 8.
// The XOR swizzle of the 16-byte chunks makes the eight rows an ldmatrix
// reads in one phase land in eight different bank groups once a head block
// has been copied verbatim (TMA bulk copy) into shared memory, while a row
// stays sixteen 16-byte pieces for the append's vector stores.
__host__ __device__ inline int64_t head_block_index(int64_t page, int layer, int kv, int head,
                                                   int64_t n_pages, int n_head_kv) {
    return ((static_cast<int64_t>(layer) * n_pages + page) * 2 + kv) * n_head_kv + head;
}
__host__ __device__ inline int swizzled_chunk(int row, int chunk) { return chunk ^ (row & 7); }

// Device-side error record.  Kernels never trap: a failed bounds check or an
// expired bounded wait stores its code here (first writer wins) and the
// kernel returns; hkv_sync_check reads it.
struct DeviceError {
    int32_t code;  // 0, kErrBadIndex or kErrTimeout
    int32_t where; // kernel id
    int32_t a;
    int32_t b;
};
constexpr int32_t kErrBadIndex = 1;
constexpr int32_t kErrTimeout = 2;

// Per-batch descriptor, built on the host once per (slot list, lengths) and
// uploaded in one copy; the pointers below address that device copy.
struct BatchView {
    const int32_t *pos;       // [n]   row being appended = rope position (used)
    const int32_t *ntok;      // [n]   rows attended = used + 1
    const int32_t *npages;    // [n]   pages covering [0, used]
    const int32_t *page_off;  // [n+1] prefix sum of npages into pages[]
    const int32_t *unit_off;  // [n+1] prefix sum of npages * n_head_kv
    const int32_t *part2_off; // [n*n_head_kv + 1] first group partial / group counter of each
    const int4 *seg;          // [n*n_head_kv] per (entry, kv head): {first partial, partials,
                              // first warp, last warp}
    const int4 *warp_start;   // [n_warps][3] per warp: {entry, kv head, page index, pages of
                              // the entry}, {page_off[entry], first three physical pages},
                              // {first unit, end unit, 0, 0}
    const int32_t *pages;     // [page_off[n]] physical pages, entry-major
    int32_t n;
    int32_t total_units;      // sum of npages * n_head_kv: one unit = one head block of K and V
    int32_t n_warps;          // warps the units are shared among (grid * kAttnWarps)
    int32_t n_parts;
    int32_t cta_merge;        // 1: the warps of a CTA pre-merge in shared memory (one
                              // partial per CTA); 0: one partial per warp
    int32_t split_segments;   // segments with more than one partial
    int32_t combine;          // 1: split partials are only stored; the combine launch
                              // that follows merges them (plan_combine)
    int32_t cluster;          // > 0: CTAs per thread-block cluster; cluster k holds segment
                              // k, whose CTA partials meet in the shared memory of the
                              // cluster's first CTA (plan_cluster); 0: no clusters
};

// Partials of one (entry, KV head) are merged by one warp when there are at
// most kMergeSingleMax of them; beyond that in two levels: groups of
// merge_group_size(n) partials, then the group results, so no single warp
// merges a long list.  Host plan and kernel share this function.
constexpr int kMergeSingleMax = 16;
__host__ __device__ inline int merge_group_size(int nparts) {
    int g = 8;
    while (g * g < nparts) {
        ++g;
    }
    return g;  // max(8, ceil(sqrt(nparts)))
}
__host__ __device__ inline int merge_groups(int nparts) {
    if (nparts <= kMergeSingleMax) {
        return 0;
    }
    const int g = merge_group_size(nparts);
    return (nparts + g - 1) / g;
}

struct PoolView {
    uint8_t *base;
    int64_t n_pages;
    int32_t n_layers;
    int32_t n_head_kv;
};

// Where finished outputs go.  n_ranks == 0: the caller's `out` only.
// Otherwise (KV-head split of one batch across ranks) every finished
// (entry, KV head) slice is stored into each rank's exchange region --
// outs[r] + layer * layer_floats + entry * row_floats + col_off + head
// slice, over NVLink for the peers -- and each rank's arrival counter for the
// layer is bumped once.  One output block per layer, so a rank that runs
// ahead never overwrites a layer its peers have not consumed yet.
struct Exchange {
    float *const *outs;       // [n_ranks] output regions (device-visible pointers)
    uint32_t *const *flags;   // [n_ranks] per-layer arrival counters
    int32_t n_ranks;
    int32_t row_floats;       // floats per entry row: 4 * n_head_kv(total) * 128
    int32_t col_off;          // this rank's first column
    int64_t layer_floats;     // floats per layer block (max entries * row_floats)
};

struct RopeView {
    const float *cos_tab;  // [context][64]
    const float *sin_tab;
    int32_t context_length;
};

// Attention launch geometry (fixed per build; the -D overrides exist for
// tuning sweeps).  Default: 8 warps per CTA, one CTA per SM, 2 stages each
// (150 KB of shared memory): two warps on each of the SM's 4 schedulers.
// With 6, warps 2 and 3 had a scheduler each while warps 0/4 and 1/5 shared
// theirs, and per-warp timestamps showed the shared ones finishing ~1 us
// later, every launch; 8 x 2 measured 16 slots of 256-4096 positions +3.3%,
// one request near 32k positions +2.2%, 32 slots of 2k-16k +0.5%, the
// batch-1 backbone step -1.2% against 6 x 2 (4 x 3-4: -12% to -22%).
#ifndef HKV_ATTN_WARPS
#define HKV_ATTN_WARPS 8
#endif
#ifndef HKV_ATTN_STAGES
#define HKV_ATTN_STAGES 2
#endif
// HKV_CUDA_CORES=1 builds the attention's QK and PV on the CUDA cores (exact
// F16 -> F32 conversions, F32 products) instead of the tensor cores: the
// comparison variant, never the default.
#ifndef HKV_CUDA_CORES
#define HKV_CUDA_CORES 0
#endif
constexpr int kAttnWarps = HKV_ATTN_WARPS;    // consumer warps per CTA, one CTA per SM
constexpr int kAttnStages = HKV_ATTN_STAGES;  // TMA ring depth per warp (K+V block per stage)

void launch_append(const PoolView &pool, const RopeView &rope, const BatchView &batch, int layer,
                   const float *k, const float *v, bool apply_rope, DeviceError *err,
                   cudaStream_t stream);
void launch_append_range(const PoolView &pool, const RopeView &rope, const int32_t *range_pages,
                         int64_t pos0, int64_t n_tokens, int layer, const float *k, const float *v,
                         bool apply_rope, DeviceError *err, cudaStream_t stream);
// Split-K decode attention with the merge of split partials folded in (the
// last warp to finish a (slot, KV head) merges).  If k_new / v_new are
// non-null, the warp owning each slot's last page also ropes and writes the
// slot's new K/V row (the fused decode step).  counters: n * n_head_kv
// zero-initialised ints, left zero on exit.  overlap_previous launches with
// programmatic stream serialization: the kernel's prologue (its plan and the
// first copies of this layer's pages) may run before the previous kernel in
// the stream has finished, so the caller may set it only when that kernel
// cannot have written this layer's pages.
void launch_attention(const PoolView &pool, const RopeView &rope, const BatchView &batch, int layer,
                      const float *q, const float *k_new, const float *v_new, float *part_o,
                      float *part_ml, int32_t *counters, float *out, const Exchange &xchg,
                      float scale_log2, DeviceError *err, bool overlap_previous,
                      cudaStream_t stream);
// Bounded wait (one thread) until *flag has reached `target` arrivals
// (wrap-around safe); records kErrTimeout and returns if it never does.
void launch_split_wait(const uint32_t *flag, uint32_t target, DeviceError *err,
                       cudaStream_t stream);
// Copy-on-write of whole pages: pairs[2 i] -> pairs[2 i + 1] (device array of
// n_pairs {source, destination} page ids), every layer, one launch.
void launch_cow_copy(const PoolView &pool, const int32_t *pairs, int32_t n_pairs, DeviceError *err,
                     cudaStream_t stream);
void launch_gather(const PoolView &pool, const int32_t *slot_pages, int64_t pos0, int64_t n,
                   int layer, uint16_t *k_out, uint16_t *v_out, DeviceError *err,
                   cudaStream_t stream);
size_t attention_smem_bytes(bool cta_merge, bool cluster = false);
// Clusters of csize attention CTAs (2..16, the cluster-merge variant) that
// can be resident at once on the current device; 0 if none (cached per
// device).
int attention_cluster_fit(int csize);

}  // namespace hkv
