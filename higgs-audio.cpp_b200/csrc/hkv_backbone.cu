// hkv_backbone.cu -- Q4_K projections of the decode step around the KV path.
//
// The reference's decode graph per layer (src/higgs_pipeline.cpp:5709-5856):
//     normed = rms_norm(h) * attn_norm
//     q, k, v = Wq normed, Wk normed, Wv normed           (mul_mat_f32, :465-469)
//     q = rms_norm_per_head(q) * q_norm; k likewise          (:5727-5733)
//     RoPE(q, k), append k/v, attention                      (the engine's hkv_decode_step)
//     h = h + Wo attn                                        (:5790-5791)
//     m = rms_norm(h) * ffn_norm; g = silu(Wg m) * (Wu m)    (:5806-5822)
//     h = h + Wd g                                           (:5823, :5843)
// and after the last layer logits = Wout (rms_norm(h) * output_norm) (:5858-5863).
// With Q4_K weights GGML's CPU backend quantises each activation row to Q8_K
// and dots it with the weight blocks in integers.  The kernels here do the
// same arithmetic on the GPU:
//
//   * gemv_kernel<mode, 1>: one pass over a Q4_K matrix for one activation
//     vector.  Every CTA first issues its weight loads (1-D bulk copies into a
//     shared-memory ring), then (after the previous kernel in the stream has
//     finished: griddepcontrol.wait) quantises the activation vector to Q8_K
//     in shared memory -- optionally after the RMSNorm, done in double like
//     GGML -- and dots 4-bit weights with 8-bit activations by dp4a.
//   * gemv_kernel<mode, 8>: up to 8 vectors on the tensor cores (integer
//     mma.sync m16n8k32, one k-step = one 32-weight sub-block): 16-row tiles
//     of weights x 8 vectors, the sub-block mins through the same mma.  The
//     CTAs of a cluster share one fragment-order Q8_K image, each quantising
//     a share of the blocks into every CTA's shared memory (distributed
//     shared memory stores).
//     Epilogues of both: store, add a residual, SwiGLU of two matrices, or
//     the per-head RMSNorm of q and k, whose 128 rows span a cluster of 4
//     CTAs that add their sums of squares through distributed shared memory.
//   * q4k_quantize_kernel: the repo's Q4_K encoder (weights for tests and the
//     benchmark; the reference quantises with GGML's tools offline).
//   * embed_kernel / argmax_kernel: embedding rows (text ids or the sum of
//     8 audio-codebook rows) and greedy codes per codebook.
//
// Every copy reads this GPU's own memory into one CTA's shared memory.
#include <cooperative_groups.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/hkv.h"
#include "hkv_device.cuh"
#include "hkv_internal.h"

namespace cg = cooperative_groups;

namespace hkv {
namespace bb {

using namespace dev;

constexpr int kQK = 256;        // weights per Q4_K / Q8_K block
constexpr int kQ4Bytes = 144;   // bytes per Q4_K block
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kWarpsWide = 12;  // consumer warps of the one-CTA-per-SM tensor-core kernels
constexpr int kMaxVec = 8;      // activation vectors of a tensor-core launch: one mma n-tile
constexpr int kMaxVec2 = 16;    // or two n-tiles, when the image of 16 vectors fits
constexpr int kTileRows = 16;   // weight rows of an mma tile
constexpr int kClusterCtas = 4; // CTAs per head in the q/k/v launch (32 rows each)
constexpr int kMaxCols = 16384;

enum Mode { kPlain = 0, kSwiglu = 1, kQkv = 2 };

// Consumer warps of gemv_kernel<mode, nb>: 8, or kWarpsWide for the tensor-core
// kernels that run one CTA per SM (q/k/v keeps 8 to fit two CTAs per SM).
__host__ __device__ constexpr int consumer_warps(int mode, int nb) {
    return nb > 1 && mode != kQkv ? kWarpsWide : kWarps;
}

struct GemvParams {
    const uint8_t *w[3];      // kPlain: w[0]; kSwiglu: gate, up; kQkv: q, k, v
    int32_t row_end[3];       // virtual row boundaries of the matrices (kQkv)
    int32_t rows;             // virtual rows
    int32_t cols;
    int32_t n;                // activation vectors, <= kMaxVec2
    const float *x;           // [n][cols]
    const float *norm;        // nullptr or [cols]
    float eps;
    const float *residual;    // nullptr or [n][rows] (kPlain)
    float *y[3];              // outputs, [n][y_rows[m]] each
    int32_t y_rows[3];
    const float *head_norm[2];  // kQkv: q_norm, k_norm [128]
    int32_t rows_per_cta;     // contiguous weight rows of one CTA
    int32_t chunk_rows;       // rows per ring stage (kTileRows for several vectors)
    int32_t n_stages;         // ring stages (<= kMaxStages)
    int32_t stage_bytes;      // chunk_rows * row bytes * matrices
    int32_t ring_bytes;       // shared memory of the ring
    int32_t empty_count;      // arrivals that free a stage
    int32_t lanes_per_row;    // one vector: 8 or 16 consumer lanes share a row's dot product
    int32_t ksplit;           // several vectors: warps sharing one tile's blocks
    int32_t tensor;           // 1: the tensor-core kernel even for one vector
    int32_t grid_ctas;        // several vectors: CTAs (a multiple of share_ctas)
    int32_t share_ctas;       // several vectors: CTAs of a cluster sharing the activation image
    DeviceError *err;         // bounded-wait timeouts are recorded here
};

// Weight ring of a CTA: n_stages stages of chunk_rows whole rows, chosen per
// launch (plan_rows).  When a CTA's rows fit in kRingCap they are all in
// flight at once, in up to kMaxStages chunks, before the kernel waits for its
// predecessor; otherwise stages of about kStreamStageBytes are refilled as
// the consumer warps release them.
constexpr int kMaxStages = 12;
constexpr int kRingCap = 100 * 1024;
constexpr int kStreamStageBytes = 24 * 1024;
// "full" mbarriers: one per stage, completed once per chunk loaded into it
// (one vector: a warp takes its rows in stage order, so it always waits for
// the phase after the one it saw last); one per tile, used once, for the
// tensor-core kernel, whose warps take tiles out of stage order -- waiting on
// a reused stage's second phase before its first completed would return at
// once, as the first phase's parity differs.
constexpr int kMaxTiles = 24;
constexpr int kBarBytes = 304;              // kMaxTiles full + kMaxStages empty + 1 norm mbarrier
constexpr int kQkvRows = 32;                // rows per CTA in the q/k/v launch (4 per head)
static_assert((kMaxTiles + kMaxStages + 1) * 8 <= kBarBytes && kBarBytes % 16 == 0, "mbarrier area too small");
static_assert(kMaxTiles >= kMaxStages, "the one-vector kernel uses a full barrier per stage");

__device__ __forceinline__ int4 ld_stream(const uint8_t *p) {
    return __ldcs(reinterpret_cast<const int4 *>(p));
}

__device__ __forceinline__ float half_bits(uint32_t bits16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits16 & 0xFFFFu)));
}

// Byte k (0..11) of the packed scales held in three words.
__device__ __forceinline__ uint32_t sbyte(uint32_t s0, uint32_t s1, uint32_t s2, int k) {
    const uint32_t w = k < 4 ? s0 : (k < 8 ? s1 : s2);
    return (w >> (8 * (k & 3))) & 0xFFu;
}

// 6-bit scale and min of sub-block j (0..7) of a Q4_K block.
__device__ __forceinline__ void scale_min(uint32_t s0, uint32_t s1, uint32_t s2, int j, int &sc,
                                          int &m) {
    if (j < 4) {
        sc = static_cast<int>(sbyte(s0, s1, s2, j) & 63u);
        m = static_cast<int>(sbyte(s0, s1, s2, j + 4) & 63u);
    } else {
        sc = static_cast<int>((sbyte(s0, s1, s2, j + 4) & 0x0Fu) |
                              ((sbyte(s0, s1, s2, j - 4) >> 6) << 4));
        m = static_cast<int>((sbyte(s0, s1, s2, j + 4) >> 4) | ((sbyte(s0, s1, s2, j) >> 6) << 4));
    }
}

__device__ __forceinline__ double warp_sum_double(double v) {
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        v += __shfl_xor_sync(0xffffffffu, v, off);
    }
    return v;
}

// Byte offset of 16-byte chunk c (0..3) of 64-byte item j (a block's
// sub-block pair) in a vector's Q8 image.  The chunks of an item are stored
// rotated by (j / 2) mod 4, so the 8 lanes of a load phase, which read the
// same chunk of 8 consecutive items, hit 8 different bank groups.
__device__ __forceinline__ int q8_offset(int j, int c) { return j * 64 + ((c ^ ((j >> 1) & 3)) << 4); }

// Shared-memory image of the Q8_K activations, in one of two layouts:
//  * rows (frag == 0, the one-vector dot products): q [n][cols] with the
//    chunks of each 64-byte item rotated (q8_offset), and s, the sums of q
//    over each 32-element sub-block;
//  * tensor-core fragments (frag == NB, the several-vector kernels): for item
//    j (sub-blocks 2p, 2p+1 of block j / 4) and vector e, 64 bytes at
//    (j * NB + e) * 64, where lane t (0..3) of an mma B fragment finds, at
//    t * 16, elements 8t .. 8t+7 of sub-block 2p then of sub-block 2p+1 --
//    one conflict-free 16-byte load per lane.  No sums: the mins go through
//    the mma as well.
struct Q8View {
    int8_t *q;   // rows: [n][cols]; fragments: [cols / 64][NB][64]
    float *d;    // [n][nsb]
    int32_t *s;  // rows only: [n][nsb * 8]
    double *red; // rows: [kWarps + 1] reduction scratch; fragments: [n * nsb]
                 // per-block sums of squares, then [n] float scales
    int frag;    // 0, or NB of the fragment layout
};

__host__ __device__ inline size_t q8_smem_bytes(int n, int cols, bool frag) {
    const int nsb = cols / kQK;
    size_t b = static_cast<size_t>(n) * cols;          // q
    b = (b + 15) & ~size_t(15);
    b += static_cast<size_t>(n) * nsb * 4;             // d
    b = (b + 15) & ~size_t(15);
    if (!frag) b += static_cast<size_t>(n) * nsb * 8 * 4;  // s
    b = (b + 15) & ~size_t(15);
    // red: kWarps + 1 doubles; fragments: per-block sums of squares and scales
    b += frag ? static_cast<size_t>(n) * nsb * sizeof(double) + static_cast<size_t>(n) * sizeof(float)
              : (kWarps + 1) * sizeof(double);
    b = (b + 15) & ~size_t(15);
    return b;
}

// Shared-memory stride of a weight row in the tensor-core kernel: the row's
// bytes padded to an odd multiple of 32 modulo 128, so the 8-byte fragment
// loads of four consecutive rows (one 16-lane load phase) fall in four
// different 32-byte bank groups (o_proj's 2304-byte rows are a multiple of
// 128 and would put all four in the same banks).
__host__ __device__ constexpr int smem_row_stride(int row_bytes) {
    return row_bytes + ((row_bytes % 128 == 32 || row_bytes % 128 == 96) ? 0
                        : (row_bytes % 128 < 32 ? 32 - row_bytes % 128
                                                : (row_bytes % 128 < 96 ? 96 - row_bytes % 128 : 160 - row_bytes % 128)));
}
static_assert(smem_row_stride(2304) % 128 == 32 && smem_row_stride(1440) == 1440 && smem_row_stride(5472) == 5472,
              "row strides of the backbone's shapes");

// kQkv: the projected rows [nb][kQkvRows] and the cluster's sums of
// squares [kClusterCtas][nb] after the activation image.
__host__ __device__ constexpr int qkv_extra_bytes(int mode, int nb) {
    return mode == kQkv ? nb * kQkvRows * 4 + kClusterCtas * nb * 8 + 16 : 0;
}

__device__ inline Q8View carve_q8(unsigned char *smem, int n, int cols, bool frag) {
    const int nsb = cols / kQK;
    Q8View v;
    size_t off = 0;
    v.q = reinterpret_cast<int8_t *>(smem);
    off = (static_cast<size_t>(n) * cols + 15) & ~size_t(15);
    v.d = reinterpret_cast<float *>(smem + off);
    off = (off + static_cast<size_t>(n) * nsb * 4 + 15) & ~size_t(15);
    v.s = reinterpret_cast<int32_t *>(smem + off);
    if (!frag) off = (off + static_cast<size_t>(n) * nsb * 32 + 15) & ~size_t(15);
    v.red = reinterpret_cast<double *>(smem + off);
    v.frag = frag ? n : 0;
    return v;
}

// Where lane `lane` of a quantising warp stores its 8 values of block b of
// vector e: elements 8 lane .. 8 lane + 7 of the block, i.e. quarter
// (lane & 3) of sub-block lane / 4.
__device__ __forceinline__ int8_t *q8_store_at(const Q8View &a, int cols, int e, int b, int lane) {
    if (a.frag != 0) {
        const int j = b * 4 + (lane >> 3);
        return a.q + (static_cast<size_t>(j) * a.frag + e) * 64 + (lane & 3) * 16 + ((lane >> 2) & 1) * 8;
    }
    return a.q + static_cast<size_t>(e) * cols + q8_offset(b * 4 + (lane >> 3), (lane & 7) >> 1) + (lane & 1) * 8;
}

// Barrier of the kWarps consumer warps only (the producer warp never joins).
__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"r"(kThreads) : "memory");
}

// The same for W consumer warps.
template <int W>
__device__ __forceinline__ void consumer_sync_w() {
    asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");
}

// Q8_K quantisation of one 256-element block held 8 per lane across a warp
// (GGML's quantize_row_q8_K: iscale = -127 / (element of largest magnitude,
// the first on ties), q = min(127, round-half-even(iscale * x)),
// d = 1 / iscale): the lane's 8 bytes (lo, hi), d and the lane's sum of q.
__device__ __forceinline__ void q8_pack(const float (&v)[8], int lane, uint32_t &lo, uint32_t &hi, float &d,
                                        int &qsum) {
    float am = 0.0f, mx = 0.0f;
    int idx = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float ax = fabsf(v[i]);
        if (ax > am) {
            am = ax;
            mx = v[i];
            idx = lane * 8 + i;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, am, off);
        const float om = __shfl_xor_sync(0xffffffffu, mx, off);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (oa > am || (oa == am && oi < idx)) {
            am = oa;
            mx = om;
            idx = oi;
        }
    }
    int q[8];
    d = 0.0f;
    if (am == 0.0f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0;
    } else {
        const float iscale = -127.0f / mx;
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = min(127, __float2int_rn(__fmul_rn(iscale, v[i])));
        d = 1.0f / iscale;
    }
    lo = hi = 0;
    qsum = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        lo |= (static_cast<uint32_t>(q[i]) & 0xFFu) << (8 * i);
        hi |= (static_cast<uint32_t>(q[i + 4]) & 0xFFu) << (8 * i);
        qsum += q[i] + q[i + 4];
    }
}

// The same, written to the shared-memory image.
__device__ __forceinline__ void quantize_block(const float (&v)[8], const Q8View &a, int cols, int nsb,
                                               int e, int b, int lane) {
    uint32_t lo, hi;
    float d;
    int qs;
    q8_pack(v, lane, lo, hi, d, qs);
    *reinterpret_cast<uint2 *>(q8_store_at(a, cols, e, b, lane)) = make_uint2(lo, hi);
    if (a.frag == 0) {
        qs += __shfl_xor_sync(0xffffffffu, qs, 1);
        qs += __shfl_xor_sync(0xffffffffu, qs, 2);
        if ((lane & 3) == 0) a.s[(e * nsb + b) * 8 + (lane >> 2)] = qs;
    }
    if (lane == 0) a.d[e * nsb + b] = d;
}

// The same quantisation for the blocks a warp holds in registers, one per
// slab (block sl * kWarps + warp of slab sl), the slabs' chains interleaved.
// The block maximum: the largest |x| bit pattern by one warp reduction
// (non-negative floats order as unsigned integers), then the lowest lane
// holding it (ballot), whose own first maximum is the block's first one --
// lane l holds elements 8l .. 8l + 7, so lower lanes hold lower indices.
template <int S>
__device__ __forceinline__ void quantize_blocks(const float (&v)[S][8], int n_slabs, const Q8View &a, int cols,
                                                int nsb, int e, int warp, int lane) {
    float mx[S];
    uint32_t am[S];
#pragma unroll
    for (int sl = 0; sl < S; ++sl) {
        float best = 0.0f, val = 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const float ax = fabsf(v[sl][i]);
            if (ax > best) {
                best = ax;
                val = v[sl][i];
            }
        }
        am[sl] = __float_as_uint(best);
        mx[sl] = val;
    }
#pragma unroll
    for (int sl = 0; sl < S; ++sl) {
        const uint32_t top = __reduce_max_sync(0xffffffffu, am[sl]);
        const uint32_t holders = __ballot_sync(0xffffffffu, am[sl] == top);
        mx[sl] = __shfl_sync(0xffffffffu, mx[sl], __ffs(static_cast<int>(holders)) - 1);
        am[sl] = top;
    }
#pragma unroll
    for (int sl = 0; sl < S; ++sl) {
        const int b = sl * kWarps + warp;
        if (sl >= n_slabs || b >= nsb) continue;
        int q[8];
        float d = 0.0f;
        if (am[sl] == 0u) {
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] = 0;
        } else {
            const float iscale = -127.0f / mx[sl];
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] = min(127, __float2int_rn(__fmul_rn(iscale, v[sl][i])));
            d = 1.0f / iscale;
        }
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            lo |= (static_cast<uint32_t>(q[i]) & 0xFFu) << (8 * i);
            hi |= (static_cast<uint32_t>(q[i + 4]) & 0xFFu) << (8 * i);
        }
        *reinterpret_cast<uint2 *>(q8_store_at(a, cols, e, b, lane)) = make_uint2(lo, hi);
        if (a.frag == 0) {
            int qs = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) qs += q[i];
            qs += __shfl_xor_sync(0xffffffffu, qs, 1);
            qs += __shfl_xor_sync(0xffffffffu, qs, 2);
            if ((lane & 3) == 0) a.s[(e * nsb + b) * 8 + (lane >> 2)] = qs;
        }
        if (lane == 0) a.d[e * nsb + b] = d;
    }
}

constexpr int kSlabMax = 5;  // 2048-element slabs held in registers (cols <= 10240)

// Q8_K image of the n activation vectors, optionally of rms_norm(x) * norm
// (sum of squares in double, mean rounded to float, scale = 1 / sqrtf(mean +
// eps), y = (x * scale) * norm as GGML rounds it).  Thread t holds elements
// [8t, 8t + 8) of every 2048-element slab, so warp w holds block 8s + w of
// slab s: one batch of loads, one barrier for the norm, then every block is
// quantised from registers.  Run by the kWarps consumer warps; ends with
// their barrier.  x0: n_vec vectors of p.cols floats.
__device__ bool quantize_activations(const GemvParams &p, const float *x0, int n_vec, const Q8View &a,
                                     double *red, const float *normbuf, uint32_t normbar) {
    if (p.norm != nullptr) {
        // the norm weights were copied into shared memory before the kernel
        // waited for its predecessor
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(normbar, 0))) return false;
    }
    const int nsb = p.cols / kQK;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_slabs = (nsb + kWarps - 1) / kWarps;
    for (int e = 0; e < n_vec; ++e) {
        const float *x = x0 + static_cast<size_t>(e) * p.cols;
        if (n_slabs <= kSlabMax) {
            float v[kSlabMax][8];
#pragma unroll
            for (int sl = 0; sl < kSlabMax; ++sl) {
                const int b = sl * kWarps + warp;
                if (sl < n_slabs && b < nsb) {
                    const float4 u0 = *reinterpret_cast<const float4 *>(x + b * kQK + lane * 8);
                    const float4 u1 = *reinterpret_cast<const float4 *>(x + b * kQK + lane * 8 + 4);
                    v[sl][0] = u0.x; v[sl][1] = u0.y; v[sl][2] = u0.z; v[sl][3] = u0.w;
                    v[sl][4] = u1.x; v[sl][5] = u1.y; v[sl][6] = u1.z; v[sl][7] = u1.w;
                }
            }
            if (p.norm != nullptr) {
                double ss = 0.0;
#pragma unroll
                for (int sl = 0; sl < kSlabMax; ++sl) {
                    const int b = sl * kWarps + warp;
                    if (sl < n_slabs && b < nsb) {
#pragma unroll
                        for (int i = 0; i < 8; ++i) ss += static_cast<double>(__fmul_rn(v[sl][i], v[sl][i]));
                    }
                }
                ss = warp_sum_double(ss);
                if (lane == 0) red[warp] = ss;
                consumer_sync();
                double t = 0.0;
                for (int w = 0; w < kWarps; ++w) t += red[w];
                const float mean = static_cast<float>(t / static_cast<double>(p.cols));
                const float scale = 1.0f / sqrtf(mean + p.eps);
#pragma unroll
                for (int sl = 0; sl < kSlabMax; ++sl) {
                    const int b = sl * kWarps + warp;
                    if (sl < n_slabs && b < nsb) {
                        const float4 w0 = *reinterpret_cast<const float4 *>(normbuf + b * kQK + lane * 8);
                        const float4 w1 = *reinterpret_cast<const float4 *>(normbuf + b * kQK + lane * 8 + 4);
                        const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                        for (int i = 0; i < 8; ++i) v[sl][i] = __fmul_rn(__fmul_rn(v[sl][i], scale), wv[i]);
                    }
                }
            }
            // slabs past the row hold zeros (their blocks are skipped)
#pragma unroll
            for (int sl = 0; sl < kSlabMax; ++sl) {
                const int b = sl * kWarps + warp;
                if (!(sl < n_slabs && b < nsb)) {
#pragma unroll
                    for (int i = 0; i < 8; ++i) v[sl][i] = 0.0f;
                }
            }
            if (n_slabs <= 2) {
                float w2[2][8];
#pragma unroll
                for (int sl = 0; sl < 2; ++sl)
#pragma unroll
                    for (int i = 0; i < 8; ++i) w2[sl][i] = v[sl][i];
                quantize_blocks<2>(w2, n_slabs, a, p.cols, nsb, e, warp, lane);
            } else {
                quantize_blocks<kSlabMax>(v, n_slabs, a, p.cols, nsb, e, warp, lane);
            }
            consumer_sync();  // red[] is reused by the next vector
        } else {
            // wider rows: two passes over x
            float scale = 1.0f;
            if (p.norm != nullptr) {
                double ss = 0.0;
#pragma unroll 4
                for (int i = threadIdx.x; i < p.cols; i += kThreads) {
                    const float xv = x[i];
                    ss += static_cast<double>(__fmul_rn(xv, xv));
                }
                ss = warp_sum_double(ss);
                if (lane == 0) red[warp] = ss;
                consumer_sync();
                double t = 0.0;
                for (int w = 0; w < kWarps; ++w) t += red[w];
                const float mean = static_cast<float>(t / static_cast<double>(p.cols));
                scale = 1.0f / sqrtf(mean + p.eps);
                consumer_sync();
            }
            for (int b = warp; b < nsb; b += kWarps) {
                float v[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const float xv = x[b * kQK + lane * 8 + i];
                    v[i] = p.norm != nullptr ? __fmul_rn(__fmul_rn(xv, scale), normbuf[b * kQK + lane * 8 + i]) : xv;
                }
                quantize_block(v, a, p.cols, nsb, e, b, lane);
            }
            consumer_sync();
        }
    }
    return true;
}

// Every thread of every CTA of the cluster (the producer warp included).
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// The same with nothing to publish: every CTA of the cluster has started.
__device__ __forceinline__ void cluster_sync_started() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
}

// The fragment-order Q8_K image of n_vec vectors (a.frag != 0), shared by
// the kClusterCtas CTAs of a cluster: CTA rank r quantises blocks
// [nsb r / C, nsb (r + 1) / C) of every vector and stores them into the
// image of every CTA of the cluster (distributed shared memory), so each CTA
// reads 1 / C of the activations.  Item it = (vector, block of the share),
// warp w taking items w, w + kWarps, ... with kQuantBatch blocks of loads
// in flight.  With a norm, a first pass stores each block's sum of squares
// (double, 256 products rounded to float as GGML forms them) into every
// CTA, and after a cluster barrier thread e < n_vec adds vector e's in
// block order -- the same scale in every CTA, not depending on the other
// vectors; a second pass reloads, scales (x * scale) * norm and quantises.
// ssp: [n_vec * nsb] doubles then [n_vec] floats.  The caller has passed a
// cluster barrier after every CTA started; this takes one more with a norm
// and ends with one after the image is complete (the producer warp takes the
// same barriers).
constexpr int kQuantBatch = 8;

template <int W>
__device__ bool quantize_activations_frag(const GemvParams &p, const float *x0, int n_vec, const Q8View &a,
                                          double *ssp, const float *normbuf, uint32_t normbar) {
    cg::cluster_group cl = cg::this_cluster();
    const unsigned csize = cl.num_blocks(), rank = cl.block_rank();
    const int nsb = p.cols / kQK;
    const int b0 = static_cast<int>(nsb * rank / csize), nb = static_cast<int>(nsb * (rank + 1) / csize) - b0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int items = n_vec * nb;
    float *scale_s = reinterpret_cast<float *>(ssp + n_vec * nsb);
    bool norm_ok = true;
    auto load = [&](int it, float (&v)[8]) {
        const int e = it / nb, b = b0 + it - e * nb;
        const float *x = x0 + static_cast<size_t>(e) * p.cols + b * kQK + lane * 8;
        const float4 u0 = *reinterpret_cast<const float4 *>(x);
        const float4 u1 = *reinterpret_cast<const float4 *>(x + 4);
        v[0] = u0.x; v[1] = u0.y; v[2] = u0.z; v[3] = u0.w;
        v[4] = u1.x; v[5] = u1.y; v[6] = u1.z; v[7] = u1.w;
    };
    // one batch of blocks per warp: the values stay in registers across the
    // norm's barrier; otherwise the second pass loads them again
    const bool one_batch = items <= W * kQuantBatch;
    float v[kQuantBatch][8];
    auto load_batch = [&](int base) {
#pragma unroll
        for (int u = 0; u < kQuantBatch; ++u) {
            if (base + W * u < items) load(base + W * u, v[u]);
        }
    };
    if (p.norm != nullptr) {
        for (int base = warp; base < items; base += W * kQuantBatch) {
            load_batch(base);
#pragma unroll
            for (int u = 0; u < kQuantBatch; ++u) {
                const int it = base + W * u;
                if (it >= items) continue;
                double ss = 0.0;
#pragma unroll
                for (int i = 0; i < 8; ++i) ss += static_cast<double>(__fmul_rn(v[u][i], v[u][i]));
                ss = warp_sum_double(ss);
                const int e = it / nb, b = b0 + it - e * nb;
                if (lane < static_cast<int>(csize)) *cl.map_shared_rank(ssp + e * nsb + b, lane) = ss;
            }
        }
        cluster_sync_all();
        if (threadIdx.x < n_vec) {
            double t = 0.0;
            for (int b = 0; b < nsb; ++b) t += ssp[threadIdx.x * nsb + b];
            const float mean = static_cast<float>(t / static_cast<double>(p.cols));
            scale_s[threadIdx.x] = 1.0f / sqrtf(mean + p.eps);
        }
        // the norm weights were copied into shared memory before the kernel
        // waited for its predecessor; a warp that gave up still takes every
        // barrier below
        norm_ok = __all_sync(0xffffffffu, mbar_wait_bounded(normbar, 0));
        consumer_sync_w<W>();
    }
    for (int base = warp; base < items; base += W * kQuantBatch) {
        if (p.norm == nullptr || !one_batch) load_batch(base);
#pragma unroll
        for (int u = 0; u < kQuantBatch; ++u) {
            const int it = base + W * u;
            if (it >= items) continue;
            const int e = it / nb, b = b0 + it - e * nb;
            float w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) w[i] = v[u][i];
            if (p.norm != nullptr && norm_ok) {
                const float scale = scale_s[e];
                const float4 w0 = *reinterpret_cast<const float4 *>(normbuf + b * kQK + lane * 8);
                const float4 w1 = *reinterpret_cast<const float4 *>(normbuf + b * kQK + lane * 8 + 4);
                const float wv[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) w[i] = __fmul_rn(__fmul_rn(w[i], scale), wv[i]);
            }
            uint32_t lo, hi;
            float d;
            int qs;
            q8_pack(w, lane, lo, hi, d, qs);
            // lanes l and l + 4 (l & 4 == 0) hold the two halves of one
            // 16-byte chunk of the image: one 16-byte store per chunk
            const uint32_t lo2 = __shfl_down_sync(0xffffffffu, lo, 4);
            const uint32_t hi2 = __shfl_down_sync(0xffffffffu, hi, 4);
            uint4 *dst = reinterpret_cast<uint4 *>(q8_store_at(a, p.cols, e, b, lane));
            float *dd = a.d + e * nsb + b;
            for (unsigned r = 0; r < csize; ++r) {
                if ((lane & 4) == 0) *cl.map_shared_rank(dst, r) = make_uint4(lo, hi, lo2, hi2);
                if (lane == 0) *cl.map_shared_rank(dd, r) = d;
            }
        }
    }
    cluster_sync_all();
    return norm_ok;
}

// Scales and mins of sub-blocks 2*part and 2*part+1 from the packed words
// (bytes 4..15 of a block), branch-free: words of the 6-bit values of
// sub-blocks 0-3 and 4-7, then the two bytes of this pair.
__device__ __forceinline__ void pair_scales(uint32_t s0, uint32_t s1, uint32_t s2, int part, int &sc0,
                                            int &sc1, int &m0, int &m1) {
    const uint32_t sc_lo = s0 & 0x3F3F3F3Fu, mn_lo = s1 & 0x3F3F3F3Fu;
    const uint32_t sc_hi = (s2 & 0x0F0F0F0Fu) | (((s0 >> 6) & 0x03030303u) << 4);
    const uint32_t mn_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | (((s1 >> 6) & 0x03030303u) << 4);
    const uint32_t scw = part < 2 ? sc_lo : sc_hi, mnw = part < 2 ? mn_lo : mn_hi;
    const int sh = 16 * (part & 1);
    sc0 = static_cast<int>((scw >> sh) & 0xFFu);
    sc1 = static_cast<int>((scw >> (sh + 8)) & 0xFFu);
    m0 = static_cast<int>((mnw >> sh) & 0xFFu);
    m1 = static_cast<int>((mnw >> (sh + 8)) & 0xFFu);
}

// Q8_K activations of one (block, sub-block pair) column, held in registers.
struct ActPart {
    int lo[8], hi[8];  // 32 + 32 int8, four per word
    int s0, s1;        // sums over the two sub-blocks
    float d;
};

__device__ __forceinline__ void load_act(ActPart &x, const Q8View &a, int cols, int nsb, int sb, int part,
                                         int e) {
    const int8_t *base = a.q + static_cast<size_t>(e) * cols;
    const int j = sb * 4 + part;
    const int4 a0 = *reinterpret_cast<const int4 *>(base + q8_offset(j, 0));
    const int4 a1 = *reinterpret_cast<const int4 *>(base + q8_offset(j, 1));
    const int4 a2 = *reinterpret_cast<const int4 *>(base + q8_offset(j, 2));
    const int4 a3 = *reinterpret_cast<const int4 *>(base + q8_offset(j, 3));
    x.lo[0] = a0.x; x.lo[1] = a0.y; x.lo[2] = a0.z; x.lo[3] = a0.w;
    x.lo[4] = a1.x; x.lo[5] = a1.y; x.lo[6] = a1.z; x.lo[7] = a1.w;
    x.hi[0] = a2.x; x.hi[1] = a2.y; x.hi[2] = a2.z; x.hi[3] = a2.w;
    x.hi[4] = a3.x; x.hi[5] = a3.y; x.hi[6] = a3.z; x.hi[7] = a3.w;
    const int2 ss = *reinterpret_cast<const int2 *>(a.s + (e * nsb + sb) * 8 + 2 * part);
    x.s0 = ss.x;
    x.s1 = ss.y;
    x.d = a.d[e * nsb + sb];
}

// (d4 d8) * sum(sc * q4 . q8) - (dmin4 d8) * sum(m * bsum) of one block part.
__device__ __forceinline__ float dot_act(const unsigned char *blk, int part, const ActPart &x) {
    const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
    const uint4 q0 = *reinterpret_cast<const uint4 *>(blk + 16 + 32 * part);
    const uint4 q1 = *reinterpret_cast<const uint4 *>(blk + 32 + 32 * part);
    int sc0, sc1, m0, m1;
    pair_scales(hdr.y, hdr.z, hdr.w, part, sc0, sc1, m0, m1);
    const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
    int sum0 = 0, sum1 = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        sum0 = __dp4a(static_cast<int>(qw[k] & 0x0F0F0F0Fu), x.lo[k], sum0);
        sum1 = __dp4a(static_cast<int>((qw[k] >> 4) & 0x0F0F0F0Fu), x.hi[k], sum1);
    }
    const int isum = sc0 * sum0 + sc1 * sum1;
    const int msum = m0 * x.s0 + m1 * x.s1;
    return __fmul_rn(half_bits(hdr.x), x.d) * static_cast<float>(isum) -
           __fmul_rn(half_bits(hdr.x >> 16), x.d) * static_cast<float>(msum);
}

// D = A B + C for a 16x32 tile A of unsigned bytes (Q4_K nibbles or
// broadcast 6-bit mins) and a 32x8 tile B of signed bytes (Q8_K), s32
// accumulators.  Fragments: lane l holds rows l/4 and l/4 + 8 of A and D,
// column l/4 of B; a[0], a[2] (row l/4) and a[1], a[3] (row l/4 + 8) carry k
// quads (l % 4) and (l % 4) + 4, b[0], b[1] the same quads of B, d columns
// 2 (l % 4) and 2 (l % 4) + 1.  Which 32 elements a k slot stands for is
// free as long as A and B agree: here slot quads (t, t + 4) of lane quarter
// t are elements 8t .. 8t + 7 of a sub-block, 8 contiguous bytes on both
// sides.
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// The same with C = 0.
__device__ __forceinline__ void mma_u8s8_zero(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                              uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%10, %10, %10, %10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// Packed 6-bit scales (sc) and mins (mn) of sub-blocks 0-3 (lo) and 4-7
// (hi), one byte each, from bytes 4..15 of a Q4_K block.
struct BlockScales {
    uint32_t sc_lo, sc_hi, mn_lo, mn_hi;
};

__device__ __forceinline__ BlockScales block_scales(uint32_t s0, uint32_t s1, uint32_t s2) {
    BlockScales r;
    r.sc_lo = s0 & 0x3F3F3F3Fu;
    r.mn_lo = s1 & 0x3F3F3F3Fu;
    r.sc_hi = (s2 & 0x0F0F0F0Fu) | (((s0 >> 6) & 0x03030303u) << 4);
    r.mn_hi = ((s2 >> 4) & 0x0F0F0F0Fu) | (((s1 >> 6) & 0x03030303u) << 4);
    return r;
}

// Scale of sub-block sb (0..7; a constant after unrolling), and its min
// copied into all 4 bytes of a word.
__device__ __forceinline__ int sub_scale(const BlockScales &s, int sb) {
    return static_cast<int>(__byte_perm(sb < 4 ? s.sc_lo : s.sc_hi, 0u, 0x4440u | static_cast<uint32_t>(sb & 3)));
}
__device__ __forceinline__ uint32_t sub_min4(const BlockScales &s, int sb) {
    const uint32_t b = static_cast<uint32_t>(sb & 3);
    return __byte_perm(sb < 4 ? s.mn_lo : s.mn_hi, 0u, b | (b << 4) | (b << 8) | (b << 12));
}

// Output of row r (of the CTA) for vector e: t[0] (and t[1], the up
// projection of kSwiglu).
template <int MODE>
__device__ __forceinline__ void store_row(const GemvParams &p, float *res, int row0, int r, int e, float t0,
                                          float t1) {
    const int grow = row0 + r;
    if (MODE == kPlain) {
        const size_t o = static_cast<size_t>(e) * p.rows + grow;
        p.y[0][o] = p.residual != nullptr ? p.residual[o] + t0 : t0;
    } else if (MODE == kSwiglu) {
        const float sl = t0 / (1.0f + expf(-t0));
        p.y[0][static_cast<size_t>(e) * p.rows + grow] = sl * t1;
    } else {
        res[e * kQkvRows + r] = t0;
    }
}

// One CTA streams its p.rows_per_cta contiguous weight rows (of each matrix)
// through a ring of p.n_stages bulk-copy stages in shared memory, issued by a
// producer warp: the first stages before waiting for the previous kernel,
// the rest as stages are released.  Dependents are released at once, so
// consecutive projections overlap their weight streams with each other's
// activation prologue and tail.
//   NB = 1 (one vector, dp4a): each of the kWarps consumer warps owns whole
// rows, 32 / p.lanes_per_row at a time; a lane's items are independent dot
// products kept in four accumulators (the latency of one Q4_K x Q8_K item is
// the limit at batch 1, not bandwidth); the row sum is a fixed-order shuffle
// reduction (deterministic), and the row's stage slot is released by one
// arrival on the stage's "empty" barrier -- no CTA-wide barrier in the loop.
//   NB = 8 / 16 (tensor cores, mma m16n8k32 integer, NB / 8 n-tiles sharing
// each weight fragment): consumer_warps(MODE, NB) consumer warps; the CTAs of
// a cluster build one shared Q8_K image; stages of kTileRows rows, each tile
// of 16 rows x NB vectors taken by p.ksplit warps over disjoint block ranges,
// whose partial sums are added in a fixed order after one consumer barrier.
template <int MODE, int NB>
__global__ void __launch_bounds__(consumer_warps(MODE, NB) * 32 + 32, NB > 1 && MODE != kQkv ? 1 : 2)
    gemv_kernel(GemvParams pin) {
    extern __shared__ __align__(128) unsigned char smem[];
    // Several vectors: one launch covers ceil(n / NB) groups of NB vectors,
    // grid_ctas CTAs per group; a CTA computes for its group exactly what a
    // launch of those vectors alone computes (the same rows, tiles and sums).
    GemvParams p = pin;
    int cta = static_cast<int>(blockIdx.x);
    if (NB > 1) {
        const int grp = cta / pin.grid_ctas;
        cta -= grp * pin.grid_ctas;
        const int e0 = grp * NB;
        p.n = min(NB, pin.n - e0);
        p.x = pin.x + static_cast<size_t>(e0) * pin.cols;
        if (pin.residual != nullptr) p.residual = pin.residual + static_cast<size_t>(e0) * pin.rows;
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            if (pin.y[k] != nullptr) {
                p.y[k] = pin.y[k] + static_cast<size_t>(e0) * (MODE == kQkv ? pin.y_rows[k] : pin.rows);
            }
        }
    }
    constexpr int kMats = MODE == kSwiglu ? 2 : 1;
    constexpr int NT = NB > 1 ? NB / 8 : 1;  // mma n-tiles of 8 vectors
    static_assert(NB == 1 || NB % 8 == 0, "the tensor-core kernel takes 8 vectors per n-tile");
    const int nsb = p.cols / kQK;
    const int row_bytes = nsb * kQ4Bytes;
    const int srow = NB > 1 ? smem_row_stride(row_bytes) : row_bytes;  // row stride in the ring
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int kW = consumer_warps(MODE, NB);  // consumer warps; warp kW is the producer
    const bool producer = warp == kW;
    const int row0 = cta * p.rows_per_cta;
    const int nrows = max(0, min(p.rows, row0 + p.rows_per_cta) - row0);
    const int R = p.chunk_rows;
    const int n_stages = p.n_stages;
    const int stage_bytes = p.stage_bytes;
    const int ring_bytes = p.ring_bytes;
    const int n_chunks = (nrows + R - 1) / R;
    unsigned char *ring = smem;
    const uint32_t full0 = smem_u32(smem + ring_bytes);
    const uint32_t empty0 = full0 + 8 * kMaxTiles;
    const uint32_t normbar = empty0 + 8 * kMaxStages;
    // full barrier of chunk c and the parity of its completion
    auto full_of = [&](int c) { return full0 + 8 * (NB > 1 ? c : c % n_stages); };
    auto full_parity = [&](int c) { return NB > 1 ? 0u : static_cast<uint32_t>((c / n_stages) & 1); };
    int m = 0, mrow0 = row0;
    if (MODE == kQkv) {
        m = row0 < p.row_end[0] ? 0 : (row0 < p.row_end[1] ? 1 : 2);
        mrow0 = row0 - (m == 0 ? 0 : (m == 1 ? p.row_end[0] : p.row_end[1]));
    }
    if (tid == 0) {
        for (int c = 0; c < (NB > 1 ? n_chunks : n_stages); ++c) mbar_init(full_of(c), 1);
        for (int st = 0; st < n_stages; ++st) {
            mbar_init(empty0 + 8 * st, static_cast<uint32_t>(p.empty_count));
        }
        mbar_init(normbar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncthreads();
    // Weights never depend on earlier kernels: the next kernel may start its
    // own weight stream now.
    pdl_trigger();

    unsigned char *after_ring = smem + ring_bytes + kBarBytes;
    const Q8View a = carve_q8(after_ring, NB > 1 ? NB : p.n, p.cols, NB > 1);
    float *normbuf = reinterpret_cast<float *>(after_ring + q8_smem_bytes(NB > 1 ? NB : p.n, p.cols, NB > 1));
    float *res = normbuf + (p.norm != nullptr ? p.cols : 0);  // kQkv [NB][32]
    // several vectors: partial sums [kW][kMats][NT][32 lanes][4]
    float *part = reinterpret_cast<float *>(reinterpret_cast<unsigned char *>(res) + qkv_extra_bytes(MODE, NB));
    bool bad = false;

    if (producer) {
        const uint64_t policy = evict_first_policy();
        const uint8_t *wbase[kMats];
#pragma unroll
        for (int k = 0; k < kMats; ++k) {
            const int wm = MODE == kSwiglu ? k : m;  // selected, not indexed: p stays in registers
            wbase[k] = (wm == 0 ? p.w[0] : (wm == 1 ? p.w[1] : p.w[2])) + static_cast<size_t>(mrow0) * row_bytes;
        }
        int issued = 0;
        // chunk c into its stage (lane 0)
        auto issue = [&](int c) {
            const int r0 = c * R;
            const int rows_c = min(R, nrows - r0);
            const uint32_t bytes = static_cast<uint32_t>(rows_c * row_bytes);
            const uint32_t stage = smem_u32(ring + (c % n_stages) * stage_bytes);
            const uint32_t bar = full_of(c);
            mbar_arrive_expect_tx(bar, bytes * kMats);
#pragma unroll
            for (int k = 0; k < kMats; ++k) {
                if (NB > 1) {
                    // a stage holds each matrix's rows of the chunk back to
                    // back (the ring holds exactly the CTA's rows), one copy
                    // per row where the stride is padded
                    if (srow == row_bytes) {
                        bulk_load(stage + k * rows_c * row_bytes, wbase[k] + static_cast<size_t>(r0) * row_bytes,
                                  bytes, bar, policy);
                    } else {
                        for (int r = 0; r < rows_c; ++r) {
                            bulk_load(stage + (k * rows_c + r) * srow,
                                      wbase[k] + static_cast<size_t>(r0 + r) * row_bytes,
                                      static_cast<uint32_t>(row_bytes), bar, policy);
                        }
                    }
                } else {
                    bulk_load(stage + k * R * row_bytes, wbase[k] + static_cast<size_t>(r0) * row_bytes, bytes,
                              bar, policy);
                }
            }
            issued = c + 1;
        };
        if (lane == 0) {
            if (p.norm != nullptr) {  // the RMSNorm weights, before any weight stage
                const uint32_t bytes = static_cast<uint32_t>(p.cols) * 4u;
                mbar_arrive_expect_tx(normbar, bytes);
                asm volatile(
                    "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                        smem_u32(normbuf)),
                    "l"(p.norm), "r"(bytes), "r"(normbar)
                    : "memory");
            }
            for (int c = 0; c < min(n_chunks, n_stages); ++c) issue(c);  // stages still free
        }
        if constexpr (NB > 1) {
            // the cluster barriers of the consumers' activation prologue:
            // started, sums of squares (with a norm), image complete
            __syncwarp();
            cluster_sync_started();
            if (p.norm != nullptr) cluster_sync_all();
            cluster_sync_all();
        }
        if (lane == 0) {
            for (int c = n_stages; c < n_chunks; ++c) {
                // wait until every row of chunk c - n_stages is done
                const int prev = c - n_stages;
                if (!mbar_wait_bounded(empty0 + 8 * (prev % n_stages), static_cast<uint32_t>((prev / n_stages) & 1))) {
                    if (p.err != nullptr && atomicCAS(&p.err->code, 0, kErrTimeout) == 0) {
                        p.err->where = HKV_KERNEL_GEMV;
                        p.err->a = blockIdx.x;
                        p.err->b = c;
                    }
                    break;
                }
                issue(c);
            }
            // the CTA must not exit with copies in flight: wait (bounded) for
            // the last copy issued into each stage
            for (int c = max(0, issued - n_stages); c < issued; ++c) {
                mbar_wait_bounded(full_of(c), full_parity(c));
            }
            if (p.norm != nullptr) mbar_wait_bounded(normbar, 0);
        }
    } else {
        if constexpr (NB > 1) cluster_sync_started();
        pdl_wait();  // x (and y, residual) belong to the kernels before
        bool qok;
        if constexpr (NB > 1) {
            qok = quantize_activations_frag<kW>(p, p.x, p.n, a, a.red, normbuf, normbar);
        } else {
            qok = quantize_activations(p, p.x, p.n, a, a.red, normbuf, normbar);
        }
        if (!qok) {
            if (tid == 0 && p.err != nullptr && atomicCAS(&p.err->code, 0, kErrTimeout) == 0) {
                p.err->where = HKV_KERNEL_GEMV;
                p.err->a = blockIdx.x;
                p.err->b = -1;
            }
            bad = true;
        }
        if constexpr (NB == 1) {
            // L = p.lanes_per_row lanes per row: lane group q = lane / L of warp
            // w takes CTA rows (32 / L) w + q, then the same plus 32 kWarps / L,
            // ...; within a row, lane l = lane % L takes items l, l + L, ...
            // with four independent accumulators.
            const int items = nsb * 4;
            const int lpr = p.lanes_per_row;
            const int rows_per_warp = 32 / lpr;
            const int qg = lane / lpr, l8 = lane % lpr;
            for (int base = 0; base < nrows && !bad; base += rows_per_warp * kWarps) {
                const int r = base + rows_per_warp * warp + qg;
                const bool has_row = r < nrows;
                const int c = has_row ? r / R : 0, rs = has_row ? r % R : 0;
                const bool ok = !has_row || mbar_wait_bounded(full_of(c), full_parity(c));
                if (!__all_sync(0xffffffffu, ok)) {
                    if (lane == 0 && p.err != nullptr && atomicCAS(&p.err->code, 0, kErrTimeout) == 0) {
                        p.err->where = HKV_KERNEL_GEMV;
                        p.err->a = blockIdx.x;
                        p.err->b = c;
                    }
                    bad = true;
                    break;
                }
                const unsigned char *stage = ring + (c % n_stages) * stage_bytes;
                float acc[kMats][NB][4];
    #pragma unroll
                for (int k = 0; k < kMats; ++k)
    #pragma unroll
                    for (int e = 0; e < NB; ++e)
    #pragma unroll
                        for (int u = 0; u < 4; ++u) acc[k][e][u] = 0.0f;
                if (has_row) {
                    for (int j0 = l8; j0 < items; j0 += 4 * lpr) {
    #pragma unroll
                        for (int u = 0; u < 4; ++u) {
                            const int j = j0 + lpr * u;
                            if (j < items) {
                                const int sb = j >> 2, part = j & 3;
    #pragma unroll
                                for (int e = 0; e < NB; ++e) {
                                    if (e < p.n) {
                                        ActPart ax;
                                        load_act(ax, a, p.cols, nsb, sb, part, e);
    #pragma unroll
                                        for (int k = 0; k < kMats; ++k) {
                                            acc[k][e][u] += dot_act(stage + (k * R + rs) * row_bytes + sb * kQ4Bytes,
                                                                    part, ax);
                                        }
                                    }
                                }
                            }
                        }
                    }
                }
                __syncwarp();
                if (has_row && l8 == 0) mbar_arrive(empty0 + 8 * (c % n_stages));  // the row's bytes are read
                float t[kMats][NB];
    #pragma unroll
                for (int k = 0; k < kMats; ++k)
    #pragma unroll
                    for (int e = 0; e < NB; ++e) {
                        float v = (acc[k][e][0] + acc[k][e][1]) + (acc[k][e][2] + acc[k][e][3]);
    #pragma unroll
                        for (int off = 8; off > 0; off >>= 1) {
                            if (off < lpr) v += __shfl_xor_sync(0xffffffffu, v, off);
                        }
                        t[k][e] = v;
                    }
                if (has_row && l8 == 0) {
    #pragma unroll
                    for (int e = 0; e < NB; ++e) {
                        if (e < p.n) store_row<MODE>(p, res, row0, r, e, t[0][e], t[kMats - 1][e]);
                    }
                }
            }
        } else {
            // Tile i = CTA rows 16 i .. 16 i + 15, in stage i % n_stages;
            // item it = tile it / ks, blocks [nsb s / ks, nsb (s + 1) / ks)
            // of slice s = it % ks.  Per block and matrix, lane (g, t) keeps
            // the s32 sums of rows g, g + 8 for vectors 2t, 2t + 1: the
            // scaled nibble products sum_j sc_j (q4 . q8)_j and, through the
            // same mma with the min broadcast as A, sum_j m_j bsum_j; then
            // (d4 d8) isum - (dmin4 d8) msum joins the float accumulator.
            constexpr uint32_t kLo = 0x0F0F0F0Fu;
            const int ks = p.ksplit;
            const int tiles = (nrows + kTileRows - 1) / kTileRows;
            const int n_items = tiles * ks;
            const int g = lane >> 2, tq = lane & 3;
            float4 *part4 = reinterpret_cast<float4 *>(part);
            for (int it = warp; it < n_items && !bad; it += kW) {
                const int tile = it / ks, slice = it - tile * ks;
                const bool ok = mbar_wait_bounded(full_of(tile), full_parity(tile));
                if (!__all_sync(0xffffffffu, ok)) {
                    if (lane == 0 && p.err != nullptr && atomicCAS(&p.err->code, 0, kErrTimeout) == 0) {
                        p.err->where = HKV_KERNEL_GEMV;
                        p.err->a = blockIdx.x;
                        p.err->b = tile;
                    }
                    bad = true;
                    break;
                }
                const unsigned char *stage = ring + (tile % n_stages) * stage_bytes;
                const int rows_t = min(kTileRows, nrows - tile * kTileRows);  // >= 1
                const int r_lo = tile * kTileRows + g;  // CTA rows r_lo and r_lo + 8
                // rows past the tile read its last row; their sums are dropped
                const int gl = min(g, rows_t - 1), gh = min(g + 8, rows_t - 1);
                const int sb0 = nsb * slice / ks, sb1 = nsb * (slice + 1) / ks;
                const unsigned char *wl0[kMats], *wh0[kMats];  // rows gl, gh at block 0
#pragma unroll
                for (int k = 0; k < kMats; ++k) {
                    wl0[k] = stage + static_cast<size_t>(k * rows_t + gl) * srow;
                    wh0[k] = stage + static_cast<size_t>(k * rows_t + gh) * srow;
                }
                const int8_t *act = a.q + static_cast<size_t>(g) * 64 + tq * 16;
                float acc[kMats][NT][4];
#pragma unroll
                for (int k = 0; k < kMats; ++k)
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int i = 0; i < 4; ++i) acc[k][nt][i] = 0.0f;
                for (int sb = sb0; sb < sb1; ++sb) {
                    const int boff = sb * kQ4Bytes;
                    BlockScales sl[kMats], sh[kMats];
                    uint32_t dl[kMats], dh[kMats];  // f16 bits: d | dmin << 16
                    int isum[kMats][NT][4], ma[kMats][NT][4], mb[kMats][NT][4];
#pragma unroll
                    for (int k = 0; k < kMats; ++k) {
                        const uint4 hl = *reinterpret_cast<const uint4 *>(wl0[k] + boff);
                        const uint4 hh = *reinterpret_cast<const uint4 *>(wh0[k] + boff);
                        sl[k] = block_scales(hl.y, hl.z, hl.w);
                        sh[k] = block_scales(hh.y, hh.z, hh.w);
                        dl[k] = hl.x;
                        dh[k] = hh.x;
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                            for (int i = 0; i < 4; ++i) isum[k][nt][i] = ma[k][nt][i] = mb[k][nt][i] = 0;
                    }
#pragma unroll
                    for (int pp = 0; pp < 4; ++pp) {
                        uint4 bq[NT];
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            bq[nt] = *reinterpret_cast<const uint4 *>(
                                act + (static_cast<size_t>(sb * 4 + pp) * NB + nt * 8) * 64);
                        }
                        const int qoff = boff + 16 + 32 * pp + 8 * tq;
#pragma unroll
                        for (int k = 0; k < kMats; ++k) {
                            const uint2 wl = *reinterpret_cast<const uint2 *>(wl0[k] + qoff);
                            const uint2 wh = *reinterpret_cast<const uint2 *>(wh0[k] + qoff);
                            const uint32_t a0 = wl.x & kLo, a1 = wh.x & kLo, a2 = wl.y & kLo, a3 = wh.y & kLo;
                            const uint32_t h0 = (wl.x >> 4) & kLo, h1 = (wh.x >> 4) & kLo;
                            const uint32_t h2 = (wl.y >> 4) & kLo, h3 = (wh.y >> 4) & kLo;
                            const uint32_t m0l = sub_min4(sl[k], 2 * pp), m0h = sub_min4(sh[k], 2 * pp);
                            const uint32_t m1l = sub_min4(sl[k], 2 * pp + 1), m1h = sub_min4(sh[k], 2 * pp + 1);
                            const int s0l = sub_scale(sl[k], 2 * pp), s1l = sub_scale(sl[k], 2 * pp + 1);
                            const int s0h = sub_scale(sh[k], 2 * pp), s1h = sub_scale(sh[k], 2 * pp + 1);
#pragma unroll
                            for (int nt = 0; nt < NT; ++nt) {
                                int c0[4], c1[4];
                                mma_u8s8_zero(c0, a0, a1, a2, a3, bq[nt].x, bq[nt].y);
                                mma_u8s8_zero(c1, h0, h1, h2, h3, bq[nt].z, bq[nt].w);
                                mma_u8s8(ma[k][nt], m0l, m0h, m0l, m0h, bq[nt].x, bq[nt].y);
                                mma_u8s8(mb[k][nt], m1l, m1h, m1l, m1h, bq[nt].z, bq[nt].w);
                                isum[k][nt][0] += s0l * c0[0] + s1l * c1[0];
                                isum[k][nt][1] += s0l * c0[1] + s1l * c1[1];
                                isum[k][nt][2] += s0h * c0[2] + s1h * c1[2];
                                isum[k][nt][3] += s0h * c0[3] + s1h * c1[3];
                            }
                        }
                    }
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt) {
                        const int e0 = nt * 8 + 2 * tq;
                        const float d8[2] = {a.d[e0 * nsb + sb], a.d[(e0 + 1) * nsb + sb]};
#pragma unroll
                        for (int k = 0; k < kMats; ++k) {
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const uint32_t dd = i < 2 ? dl[k] : dh[k];
                                const float y8 = d8[i & 1];
                                acc[k][nt][i] += __fmul_rn(half_bits(dd), y8) * static_cast<float>(isum[k][nt][i]) -
                                                 __fmul_rn(half_bits(dd >> 16), y8) *
                                                     static_cast<float>(ma[k][nt][i] + mb[k][nt][i]);
                            }
                        }
                    }
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty0 + 8 * (tile % n_stages));  // this slice of the tile is read
                if (ks == 1) {
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int r = r_lo + 8 * (i >> 1), e = nt * 8 + 2 * tq + (i & 1);
                            if (r < nrows && e < p.n) {
                                store_row<MODE>(p, res, row0, r, e, acc[0][nt][i], acc[kMats - 1][nt][i]);
                            }
                        }
                } else {
#pragma unroll
                    for (int k = 0; k < kMats; ++k)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
                            part4[((it * kMats + k) * NT + nt) * 32 + lane] =
                                make_float4(acc[k][nt][0], acc[k][nt][1], acc[k][nt][2], acc[k][nt][3]);
                        }
                }
            }
            if (ks > 1) {
                // tiles * ks <= kW: every item above was one warp's only one
                consumer_sync_w<kW>();
                for (int tile = warp; tile < tiles && !bad; tile += kW) {
                    float t[kMats][NT][4];
#pragma unroll
                    for (int k = 0; k < kMats; ++k)
#pragma unroll
                        for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
                            for (int i = 0; i < 4; ++i) t[k][nt][i] = 0.0f;
                            for (int s2 = 0; s2 < ks; ++s2) {
                                const float4 v = part4[(((tile * ks + s2) * kMats + k) * NT + nt) * 32 + lane];
                                t[k][nt][0] += v.x;
                                t[k][nt][1] += v.y;
                                t[k][nt][2] += v.z;
                                t[k][nt][3] += v.w;
                            }
                        }
                    const int r_lo = tile * kTileRows + g;
#pragma unroll
                    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
                        for (int i = 0; i < 4; ++i) {
                            const int r = r_lo + 8 * (i >> 1), e = nt * 8 + 2 * tq + (i & 1);
                            if (r < nrows && e < p.n) {
                                store_row<MODE>(p, res, row0, r, e, t[0][nt][i], t[kMats - 1][nt][i]);
                            }
                        }
                }
            }
        }
    }

    if (MODE == kQkv) {
        // q / k / v rows; the 4 CTAs of a cluster hold the 128 rows of one
        // head.  Each CTA stores its sums of squares into slot (its rank) of
        // every CTA of the cluster, so after the one cluster barrier each CTA
        // reads only its own shared memory and may leave at once.  Every
        // thread of every CTA takes the barriers, even after a timeout.
        bad = __syncthreads_or(bad) != 0;
        double *part_ss = reinterpret_cast<double *>(res + NB * kQkvRows);  // [kClusterCtas][NB]
        cg::cluster_group cl = cg::this_cluster();
        const bool normed = m < 2;  // the same for every CTA of the cluster
        const int rank = static_cast<int>(cl.block_rank());
        if (normed && warp == 0) {
            for (int e = 0; e < p.n; ++e) {
                const float v = bad ? 0.0f : res[e * kQkvRows + lane];
                const double ss = warp_sum_double(static_cast<double>(__fmul_rn(v, v)));
                if (lane < kClusterCtas) *cl.map_shared_rank(part_ss + rank * NB + e, lane) = ss;
            }
        }
        cl.sync();
        __shared__ float scale_s[NB];
        if (normed && tid < p.n) {
            double total = 0.0;
            for (int r = 0; r < kClusterCtas; ++r) total += part_ss[r * NB + tid];
            const float mean = static_cast<float>(total / static_cast<double>(kHeadDim));
            scale_s[tid] = 1.0f / sqrtf(mean + p.eps);
        }
        __syncthreads();
        if (!bad) {
            const int dim0 = static_cast<int>(cl.block_rank()) * kQkvRows;
            // matrix m's output and norm, selected without indexing p's arrays
            // by a runtime value (which would move p to local memory)
            float *const ym = m == 0 ? p.y[0] : (m == 1 ? p.y[1] : p.y[2]);
            const int yrows = m == 0 ? p.y_rows[0] : (m == 1 ? p.y_rows[1] : p.y_rows[2]);
            const float *const hn = m == 0 ? p.head_norm[0] : p.head_norm[1];
            for (int i = tid; i < p.n * kQkvRows; i += static_cast<int>(blockDim.x)) {
                const int e = i / kQkvRows, r = i % kQkvRows;
                if (r < nrows) {
                    float v = res[e * kQkvRows + r];
                    if (normed) v = __fmul_rn(__fmul_rn(v, scale_s[e]), hn[dim0 + r]);
                    ym[static_cast<size_t>(e) * yrows + mrow0 + r] = v;
                }
            }
        }
    }
}

// ------------------------------------------------------------------ encoder
// The repo's Q4_K encoder: per 32-weight sub-block, min' = min(min, 0),
// scale = (max - min') / 15, offset m = -min'; the 8 scales and offsets are
// quantised to 6 bits against d = max scale / 63 and dmin = max offset / 63
// (both stored as f16), and each weight to round((w + dmin*m) / (d*sc)) in
// [0, 15].  One warp per 256-weight block.
__global__ void q4k_quantize_kernel(const float *w, int64_t n_blocks, uint8_t *out) {
    __shared__ uint8_t qbuf[kWarps][kQK];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t b = static_cast<int64_t>(blockIdx.x) * kWarps + warp;
    if (b >= n_blocks) return;
    const float *x = w + b * kQK + lane * 8;
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = x[i];
    float mn = v[0], mx = v[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) {
        mn = fminf(mn, v[i]);
        mx = fmaxf(mx, v[i]);
    }
#pragma unroll
    for (int off = 1; off < 4; off <<= 1) {
        mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, off));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    }
    mn = fminf(mn, 0.0f);
    const float scale = (mx - mn) / 15.0f;
    const float offs = -mn;
    float smax = scale, omax = offs;
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        smax = fmaxf(smax, __shfl_xor_sync(0xffffffffu, smax, off));
        omax = fmaxf(omax, __shfl_xor_sync(0xffffffffu, omax, off));
    }
    const __half dh = __float2half_rn(smax / 63.0f);
    const __half mh = __float2half_rn(omax / 63.0f);
    const float df = __half2float(dh), mf = __half2float(mh);
    const int sc = df > 0.0f ? min(63, max(0, __float2int_rn(scale / df))) : 0;
    const int mq = mf > 0.0f ? min(63, max(0, __float2int_rn(offs / mf))) : 0;
    const float ds = df * static_cast<float>(sc), dm = mf * static_cast<float>(mq);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int q = ds > 0.0f ? min(15, max(0, __float2int_rn((v[i] + dm) / ds))) : 0;
        qbuf[warp][lane * 8 + i] = static_cast<uint8_t>(q);
    }
    // gather the sub-block scales / offsets: sub-block j is held by lanes 4j..4j+3
    int scj[8], mqj[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        scj[j] = __shfl_sync(0xffffffffu, sc, 4 * j);
        mqj[j] = __shfl_sync(0xffffffffu, mq, 4 * j);
    }
    __syncwarp();
    uint8_t *blk = out + b * kQ4Bytes;
    // quants: byte 32*pair + l holds sub-block 2*pair (low nibble) and 2*pair+1
    // (high nibble) at position l; lane writes bytes 4*lane .. 4*lane+3.
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int byte = 4 * lane + i;
        const int pair = byte >> 5, l = byte & 31;
        const uint32_t lo = qbuf[warp][64 * pair + l], hi = qbuf[warp][64 * pair + 32 + l];
        word |= (lo | (hi << 4)) << (8 * i);
    }
    reinterpret_cast<uint32_t *>(blk + 16)[lane] = word;
    if (lane == 0) {
        uint8_t s[12];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            s[j] = static_cast<uint8_t>((scj[j] & 63) | ((scj[j + 4] >> 4) << 6));
            s[j + 4] = static_cast<uint8_t>((mqj[j] & 63) | ((mqj[j + 4] >> 4) << 6));
            s[j + 8] = static_cast<uint8_t>((scj[j + 4] & 0x0F) | ((mqj[j + 4] & 0x0F) << 4));
        }
        uint32_t h[4];
        h[0] = static_cast<uint32_t>(__half_as_ushort(dh)) |
               (static_cast<uint32_t>(__half_as_ushort(mh)) << 16);
        std::memcpy(&h[1], s, 12);
        reinterpret_cast<uint4 *>(blk)[0] = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

// ----------------------------------------------------------- embeddings
// out[e] = sum over j < k of row ids[e*k + j] of a Q4_K table (+ j * stride),
// decoded like GGML's dequantize_row_q4_K (d*sc and dmin*m rounded first),
// summed in j order (the reference's chain of ggml_add, :2919-2924).  One CTA
// per (256-column block, entry), one thread per column.
__global__ void __launch_bounds__(kQK) embed_kernel(const uint8_t *table, int64_t table_rows,
                                                     int32_t cols, const int32_t *ids, int32_t k,
                                                     int32_t id_stride, int32_t n, float *out,
                                                     DeviceError *err) {
    pdl_wait();
    const int sb = blockIdx.x, e = blockIdx.y;
    const int nsb = cols / kQK;
    if (e >= n || sb >= nsb) return;
    const int pos = threadIdx.x;
    const int pair = pos >> 6, hi = (pos >> 5) & 1, l = pos & 31;
    float acc = 0.0f;
    for (int j = 0; j < k; ++j) {
        const int32_t code = ids[e * k + j];
        const int64_t id = static_cast<int64_t>(code) + static_cast<int64_t>(j) * id_stride;
        if (code < 0 || (k > 1 && code >= id_stride) || id >= table_rows) {
            if (pos == 0 && atomicCAS(&err->code, 0, kErrBadIndex) == 0) {
                err->where = HKV_KERNEL_EMBED;
                err->a = e;
                err->b = static_cast<int32_t>(id);
            }
            continue;
        }
        const uint8_t *blk = table + (id * nsb + sb) * kQ4Bytes;
        const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
        const float d = half_bits(hdr.x), dmin = half_bits(hdr.x >> 16);
        int sc, m;
        scale_min(hdr.y, hdr.z, hdr.w, 2 * pair + hi, sc, m);
        const uint32_t q = (blk[16 + 32 * pair + l] >> (4 * hi)) & 0x0Fu;
        const float v = __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)),
                                  __fmul_rn(dmin, static_cast<float>(m)));
        acc = j == 0 ? v : __fadd_rn(acc, v);
    }
    out[static_cast<size_t>(e) * cols + sb * kQK + pos] = acc;
}

// codes[e][c] = the first index of the largest of logits[e][c*size .. +size).
__global__ void argmax_kernel(const float *logits, int32_t n_books, int32_t size, int32_t n,
                              int32_t *codes) {
    pdl_wait();
    const int e = blockIdx.x;
    const int c = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (e >= n || c >= n_books) return;
    const float *x = logits + (static_cast<size_t>(e) * n_books + c) * size;
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int i = lane; i < size; i += 32) {
        if (x[i] > best) {
            best = x[i];
            idx = i;
        }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (ob > best || (ob == best && oi < idx)) {
            best = ob;
            idx = oi;
        }
    }
    if (lane == 0) codes[e * n_books + c] = idx == 0x7fffffff ? 0 : idx;
}

// ------------------------------------------------------------- launchers
size_t gemv_smem(int mode, int nb, int n, int cols, int ring_bytes, bool has_norm, int ksplit = 1) {
    const bool frag = nb > 1;
    size_t b = static_cast<size_t>(ring_bytes) + kBarBytes + q8_smem_bytes(frag ? nb : n, cols, frag) +
               (has_norm ? static_cast<size_t>(cols) * 4 : 0) + qkv_extra_bytes(mode, nb);
    if (frag && ksplit > 1) {  // partial sums of the split tiles
        b += static_cast<size_t>(consumer_warps(mode, nb)) * (mode == kSwiglu ? 2 : 1) * (nb / 8) * 32 *
             sizeof(float4);
    }
    return b;
}

// Dynamic shared memory a launch may use on `dev` (the opt-in maximum less
// room for the kernel's static shared memory).
int smem_cap_of(int dev) {
    static std::mutex mu;
    static int cap[64] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64) return 227 * 1024 - 1024;
    if (cap[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess || v <= 0) {
            v = 227 * 1024;
        }
        cap[dev] = v - 1024;
    }
    return cap[dev];
}

int num_sms_of(int dev) {
    static std::mutex mu;
    static int sms[64] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64) return 148;
    if (sms[dev] == 0) {
        int v = 0;
        if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
        sms[dev] = v;
    }
    return sms[dev];
}

template <int MODE, int NB>
cudaError_t launch_one(const GemvParams &p, cudaStream_t stream) {
    auto kern = gemv_kernel<MODE, NB>;
    const size_t smem = gemv_smem(MODE, NB, p.n, p.cols, p.ring_bytes, p.norm != nullptr, p.ksplit);
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    cudaError_t st = cudaGetDevice(&dev);
    if (st != cudaSuccess) return st;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 64 && !done[dev]) {
            st = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_cap_of(dev));
            if (st != cudaSuccess) return st;
            // All of the SM's unified memory as shared memory: a CTA of the
            // next projection (launched early, see pdl_trigger) then fits
            // beside one of this kernel and streams its weights meanwhile.
            st = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      cudaSharedmemCarveoutMaxShared);
            if (st != cudaSuccess) return st;
            done[dev] = true;
        }
    }
    cudaLaunchConfig_t cfg = {};
    // several vectors: grid_ctas CTAs per group of NB vectors, all groups in one grid
    cfg.gridDim = dim3(static_cast<unsigned>(NB > 1 ? p.grid_ctas * ((p.n + NB - 1) / NB)
                                                    : (p.rows + p.rows_per_cta - 1) / p.rows_per_cta));
    cfg.blockDim = dim3(consumer_warps(MODE, NB) * 32 + 32);  // consumer warps + one producer warp
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int na = 1;
    if (MODE == kQkv || NB > 1) {  // a head's 4 CTAs; the CTAs sharing an activation image
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = NB > 1 ? p.share_ctas : kClusterCtas;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

// Shared memory of a CTA that must fit twice on one SM (228 KB, less 1 KB
// the hardware keeps per CTA).
constexpr size_t kPairSmem = (228 - 2) * 1024 / 2;

// Ring of a CTA whose rpc rows (unit bytes each, all matrices) are all in
// flight: the fewest rows per stage that need no more than kMaxStages stages.
void ring_all_in_flight(int rpc, int unit, GemvParams &p) {
    p.chunk_rows = (rpc + kMaxStages - 1) / kMaxStages;
    p.n_stages = (rpc + p.chunk_rows - 1) / p.chunk_rows;
    p.stage_bytes = p.chunk_rows * unit;
}

// Dependent item iterations of a CTA's dot products (passes over its rows
// times item rounds per pass) with lpr lanes per row.
int dot_rounds(int rpc, int items, int lpr) {
    const int slots = kWarps * (32 / lpr);
    return ((rpc + slots - 1) / slots) * ((items + 4 * lpr - 1) / (4 * lpr));
}

// Lanes per row: 16 when a CTA's rows then all fit in one pass (two rows per
// consumer warp), else 8.  Fewer lanes per row only moved the work onto
// fewer warps (gate/up: 4 lanes per row was 3% slower than 8).
int plan_lanes(int rpc) { return rpc <= kWarps * 2 ? 16 : 8; }

// Rows per CTA of a single-vector launch: one CTA per SM (32 rows for
// q/k/v, a quarter head, for the per-head norm), or two CTAs per SM when
// that needs fewer dependent dot-product rounds (half the rows each, more
// lanes per row) and both rings then hold all their rows in shared memory
// that two CTAs can share -- which is always the case for the FFN's gate and
// up, whose rows per SM do not fit one ring: every weight byte is then
// requested before the kernel waits for its predecessor, instead of half of
// them in bursts after the first rows are done.
int single_vector_rows(const GemvParams &p, int mode, int dev) {
    if (mode == kQkv) return kQkvRows;
    const int mats = mode == kSwiglu ? 2 : 1;
    const int unit = p.cols / kQK * kQ4Bytes * mats;
    const int items = p.cols / kQK * 4;
    const int sms = num_sms_of(dev);
    const int rpc1 = std::max(1, (p.rows + sms - 1) / sms);
    const int rpc2 = std::max(1, (p.rows + 2 * sms - 1) / (2 * sms));
    GemvParams q = p;
    ring_all_in_flight(rpc2, unit, q);
    const bool pair_fits = static_cast<int64_t>(rpc2) * unit <= kRingCap &&
                           gemv_smem(mode, 1, 1, p.cols, q.n_stages * q.stage_bytes, p.norm != nullptr) <= kPairSmem;
    const bool one_fits = static_cast<int64_t>(rpc1) * unit <= kRingCap;
    const int r1 = dot_rounds(rpc1, items, plan_lanes(rpc1));
    const int r2 = dot_rounds(rpc2, items, plan_lanes(rpc2));
    return pair_fits && (!one_fits || r2 < r1) ? rpc2 : rpc1;
}

// Ring plan of a one-vector (dp4a) launch: single_vector_rows.  The lanes
// per row -- and with them the order in which a row's products are summed --
// come from the shape alone.  A ring that cannot hold its CTA's rows streams
// them through stages of about kStreamStageBytes.
void plan_rows(GemvParams &p, int mode, int dev) {
    const int mats = mode == kSwiglu ? 2 : 1;
    const int unit = p.cols / kQK * kQ4Bytes * mats;
    const int rpc_single = single_vector_rows(p, mode, dev);
    p.rows_per_cta = rpc_single;
    if (static_cast<int64_t>(p.rows_per_cta) * unit <= kRingCap) {
        ring_all_in_flight(p.rows_per_cta, unit, p);
    } else {
        p.chunk_rows = std::max(1, std::min(p.rows_per_cta, kStreamStageBytes / unit));
        p.n_stages = std::max(2, std::min(kMaxStages, kRingCap / (p.chunk_rows * unit)));
        p.stage_bytes = p.chunk_rows * unit;
    }
    p.ring_bytes = p.n_stages * p.stage_bytes;
    p.empty_count = p.chunk_rows;
    p.lanes_per_row = plan_lanes(rpc_single);
    p.ksplit = 1;
}

// CTAs sharing one activation image in the tensor-core kernel: the 4 of a
// head for q/k/v; 4 (each reads a quarter of the activations) where the rows
// of ceil(rows / 132) CTAs -- as many 4-CTA clusters as fit on a B200 at one
// CTA per SM -- fit in shared memory; 2 for the FFN's gate/up pair, whose
// 9728 rows need all 148 SMs to stay in flight.
int share_ctas_of(int mode) { return mode == kSwiglu ? 2 : kClusterCtas; }

// Clusters of csize CTAs that fit on `dev` at once with one CTA per SM (the
// tensor-core kernel's shared memory), for grids of one wave.
int max_clusters_of(int dev, int csize) {
    static std::mutex mu;
    static int cache[64][kClusterCtas + 1] = {};
    std::lock_guard<std::mutex> lock(mu);
    const bool cached = dev >= 0 && dev < 64 && csize >= 1 && csize <= kClusterCtas;
    if (cached && cache[dev][csize] != 0) return cache[dev][csize];
    int v = num_sms_of(dev) / csize;
    auto kern = gemv_kernel<kPlain, kMaxVec>;
    const int smem = smem_cap_of(dev);
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) == cudaSuccess) {
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(static_cast<unsigned>(num_sms_of(dev)));
        cfg.blockDim = dim3(consumer_warps(kPlain, kMaxVec) * 32 + 32);
        cfg.dynamicSmemBytes = static_cast<size_t>(smem);
        cudaLaunchAttribute attr;
        attr.id = cudaLaunchAttributeClusterDimension;
        attr.val.clusterDim.x = static_cast<unsigned>(csize);
        attr.val.clusterDim.y = 1;
        attr.val.clusterDim.z = 1;
        cfg.attrs = &attr;
        cfg.numAttrs = 1;
        int n = 0;
        if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) == cudaSuccess && n > 0) v = std::min(v, n);
    }
    (void)cudaGetLastError();
    v = std::max(v, 1);
    if (cached) cache[dev][csize] = v;
    return v;
}

// Plan of a several-vector (tensor-core) launch, in clusters of
// kClusterCtas CTAs sharing the activation image: as many CTAs as fit at
// once with one per SM (a multiple of kClusterCtas; 32 rows each for q/k/v,
// a quarter head), ceil(rows / CTAs) rows each, stages of kTileRows
// rows; ksplit warps share a tile's blocks when the CTA has fewer tiles than
// warps (each slice at least 2 blocks).  All rows in flight when they fit
// beside the activation image, else as many 16-row stages as fit (>= 2).
// The split depends on the shape only, so a vector's results do not depend
// on how many others share the launch.  False when not even two stages fit.
bool plan_tiles(GemvParams &p, int mode, int dev, int nb) {
    const int mats = mode == kSwiglu ? 2 : 1;
    const int nsb = p.cols / kQK;
    const int unit = smem_row_stride(nsb * kQ4Bytes) * mats;  // ring bytes per row
    const int csize = share_ctas_of(mode);
    p.share_ctas = csize;
    if (mode == kQkv) {
        p.rows_per_cta = kQkvRows;
        p.grid_ctas = (p.rows + kQkvRows - 1) / kQkvRows;  // whole heads: a multiple of 4
    } else {
        const int ctas = csize * max_clusters_of(dev, csize);
        p.rows_per_cta = std::max(1, (p.rows + ctas - 1) / ctas);
        const int used = (p.rows + p.rows_per_cta - 1) / p.rows_per_cta;
        p.grid_ctas = (used + csize - 1) / csize * csize;
    }
    const int rpc = p.rows_per_cta;
    const int tiles = (rpc + kTileRows - 1) / kTileRows;
    if (tiles > kMaxTiles) return false;
    p.chunk_rows = kTileRows;
    p.stage_bytes = kTileRows * unit;
    p.ksplit = std::max(1, std::min(consumer_warps(mode, nb) / tiles, nsb / 2));
    p.empty_count = p.ksplit;
    p.lanes_per_row = 1;
    const size_t fixed = gemv_smem(mode, nb, nb, p.cols, 0, p.norm != nullptr, p.ksplit);
    const size_t cap = static_cast<size_t>(smem_cap_of(dev));
    if (fixed >= cap) return false;
    const size_t budget = cap - fixed;
    // a stage holds each matrix's rows of its tile back to back: all rows
    // in flight take rpc * unit bytes
    const size_t all = static_cast<size_t>(rpc) * unit;
    if (tiles <= kMaxStages && all <= budget) {
        p.n_stages = tiles;
        p.ring_bytes = static_cast<int32_t>(all);
        return true;
    }
    p.n_stages = static_cast<int32_t>(std::min<size_t>(kMaxStages, budget / p.stage_bytes));
    p.ring_bytes = p.n_stages * p.stage_bytes;
    return p.n_stages >= 2;
}

// Vectors e0 .. e0 + count - 1 of p.
GemvParams vector_slice(const GemvParams &p, int mode, int e0, int count) {
    GemvParams q = p;
    q.n = count;
    q.x = p.x + static_cast<size_t>(e0) * p.cols;
    if (q.residual) q.residual += static_cast<size_t>(e0) * p.rows;
    for (int k = 0; k < 3; ++k) {
        if (q.y[k]) q.y[k] += static_cast<size_t>(e0) * (mode == kQkv ? p.y_rows[k] : p.rows);
    }
    return q;
}

// One vector: the dp4a kernel (plan_rows), unless p.tensor.  Several (or
// p.tensor): the tensor-core kernel, kMaxVec2 or kMaxVec vectors per launch
// (each launch reads the weights once); if no plan fits shared memory, one
// dp4a launch per vector.  The two kernels sum in different orders: a caller that
// wants a vector's result not to depend on its batch-mates fixes p.tensor.
template <int MODE>
cudaError_t launch_gemv(GemvParams p, cudaStream_t stream, int64_t *launches = nullptr) {
    int dev = 0;
    cudaError_t st = cudaGetDevice(&dev);
    if (st != cudaSuccess) return st;
    if (p.n > 1 || p.tensor != 0) {
        // 16 vectors per launch where their image fits beside the weights
        // (the same tiles, slices and sums as 8 per launch: bit-identical)
        // (all groups of 16 or 8 vectors in one grid: gemv_kernel)
        GemvParams t2 = p;
        if (p.n > kMaxVec && plan_tiles(t2, MODE, dev, kMaxVec2)) {
            st = launch_one<MODE, kMaxVec2>(t2, stream);
            if (st == cudaSuccess && launches != nullptr) ++*launches;
            return st;
        }
        GemvParams t = p;
        if (plan_tiles(t, MODE, dev, kMaxVec)) {
            st = launch_one<MODE, kMaxVec>(t, stream);
            if (st == cudaSuccess && launches != nullptr) ++*launches;
            return st;
        }
    }
    GemvParams one = p;  // one vector per launch
    one.n = 1;
    plan_rows(one, MODE, dev);
    if (gemv_smem(MODE, 1, 1, p.cols, one.ring_bytes, p.norm != nullptr) > static_cast<size_t>(smem_cap_of(dev))) {
        return cudaErrorInvalidValue;
    }
    for (int e0 = 0; e0 < p.n; ++e0) {
        st = launch_one<MODE, 1>(vector_slice(one, MODE, e0, 1), stream);
        if (st != cudaSuccess) return st;
        if (launches != nullptr) ++*launches;
    }
    return cudaSuccess;
}

void set_msg(char *buf, size_t len, const char *fmt, ...) __attribute__((format(printf, 3, 4)));
void set_msg(char *buf, size_t len, const char *fmt, ...) {
    if (buf == nullptr || len == 0) return;
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, len, fmt, ap);
    va_end(ap);
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace bb
}  // namespace hkv

using namespace hkv;
using namespace hkv::bb;

// Device error word of the standalone projection calls (hkv_q4k_gemv /
// hkv_q4k_qkv): a bounded wait that gave up is recorded here and reported
// by hkv_q4k_sync_check.  Host code only takes its address, per device.
static __device__ hkv::DeviceError g_q4k_err;

namespace {
std::mutex g_q4k_err_mu;
hkv::DeviceError *g_q4k_err_ptr[64] = {};

hkv::DeviceError *q4k_err_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_q4k_err_mu);
    if (g_q4k_err_ptr[dev] == nullptr) {
        void *ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_q4k_err) != cudaSuccess) return nullptr;
        g_q4k_err_ptr[dev] = static_cast<hkv::DeviceError *>(ptr);
    }
    return g_q4k_err_ptr[dev];
}
}  // namespace

// ============================================================== C ABI
extern "C" int hkv_q4k_quantize(const float *w, int64_t rows, int64_t cols, void *blocks,
                                hkv_stream stream, char *err_msg, size_t err_len) {
    if (w == nullptr || blocks == nullptr || rows <= 0 || cols <= 0 || cols % kQK != 0) {
        set_msg(err_msg, err_len, "hkv_q4k_quantize: need rows > 0 and cols a positive multiple of 256");
        return HKV_ERR_INVALID;
    }
    if (!aligned16(w) || !aligned16(blocks)) {
        set_msg(err_msg, err_len, "hkv_q4k_quantize: pointers must be 16-byte aligned");
        return HKV_ERR_INVALID;
    }
    const int64_t n_blocks = rows * (cols / kQK);
    const int64_t grid = (n_blocks + kWarps - 1) / kWarps;
    q4k_quantize_kernel<<<static_cast<unsigned>(grid), kThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        w, n_blocks, static_cast<uint8_t *>(blocks));
    const cudaError_t st = cudaGetLastError();
    if (st != cudaSuccess) {
        set_msg(err_msg, err_len, "hkv_q4k_quantize: %s", cudaGetErrorString(st));
        return HKV_ERR_CUDA;
    }
    return HKV_OK;
}

namespace {

int check_gemv_shape(int64_t rows, int64_t cols, int32_t n, const void *x, const void *y,
                     char *err_msg, size_t err_len, const char *who) {
    if (rows <= 0 || rows > (1 << 30) || cols <= 0 || cols % kQK != 0 || cols > kMaxCols) {
        set_msg(err_msg, err_len, "%s: rows must be positive and cols a multiple of 256 up to %d", who,
                kMaxCols);
        return HKV_ERR_INVALID;
    }
    if (n <= 0) {
        set_msg(err_msg, err_len, "%s: n must be positive", who);
        return HKV_ERR_INVALID;
    }
    if (x == nullptr || y == nullptr || !aligned16(x) || !aligned16(y)) {
        set_msg(err_msg, err_len, "%s: x and y must be non-null 16-byte aligned device pointers", who);
        return HKV_ERR_INVALID;
    }
    return HKV_OK;
}

int finish(cudaError_t st, char *err_msg, size_t err_len, const char *who) {
    if (st != cudaSuccess) {
        set_msg(err_msg, err_len, "%s: %s", who, cudaGetErrorString(st));
        return HKV_ERR_CUDA;
    }
    return HKV_OK;
}

}  // namespace

extern "C" int hkv_q4k_gemv(const hkv_q4k_gemv_args *a, hkv_stream stream, char *err_msg,
                            size_t err_len) {
    const char *who = "hkv_q4k_gemv";
    if (a == nullptr) {
        set_msg(err_msg, err_len, "%s: null arguments", who);
        return HKV_ERR_INVALID;
    }
    int st = check_gemv_shape(a->rows, a->cols, a->n, a->x, a->y, err_msg, err_len, who);
    if (st != HKV_OK) return st;
    const bool swiglu = a->w_up != nullptr;
    if (a->w == nullptr || !aligned16(a->w) || (swiglu && !aligned16(a->w_up)) ||
        (a->norm != nullptr && !aligned16(a->norm)) ||
        (a->residual != nullptr && !aligned16(a->residual))) {
        set_msg(err_msg, err_len, "%s: weight, norm and residual pointers must be 16-byte aligned", who);
        return HKV_ERR_INVALID;
    }
    if (swiglu && a->residual != nullptr) {
        set_msg(err_msg, err_len, "%s: the SwiGLU form takes no residual", who);
        return HKV_ERR_INVALID;
    }
    GemvParams p = {};
    p.w[0] = static_cast<const uint8_t *>(a->w);
    p.w[1] = static_cast<const uint8_t *>(a->w_up);
    p.rows = static_cast<int32_t>(a->rows);
    p.tensor = a->tensor_cores != 0 ? 1 : 0;
    p.row_end[0] = p.row_end[1] = p.row_end[2] = p.rows;
    p.cols = static_cast<int32_t>(a->cols);
    p.n = a->n;
    p.x = a->x;
    p.norm = a->norm;
    p.eps = a->eps;
    p.residual = a->residual;
    p.y[0] = a->y;
    p.y_rows[0] = p.rows;
    p.err = q4k_err_word();
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    return finish(swiglu ? launch_gemv<kSwiglu>(p, s) : launch_gemv<kPlain>(p, s), err_msg, err_len, who);
}

extern "C" int hkv_q4k_qkv(const hkv_q4k_qkv_args *a, hkv_stream stream, char *err_msg, size_t err_len) {
    const char *who = "hkv_q4k_qkv";
    if (a == nullptr) {
        set_msg(err_msg, err_len, "%s: null arguments", who);
        return HKV_ERR_INVALID;
    }
    const int64_t rq = static_cast<int64_t>(a->n_head) * kHeadDim;
    const int64_t rk = static_cast<int64_t>(a->n_head_kv) * kHeadDim;
    if (a->n_head <= 0 || a->n_head_kv <= 0 || a->n_head % a->n_head_kv != 0) {
        set_msg(err_msg, err_len, "%s: need n_head a positive multiple of n_head_kv", who);
        return HKV_ERR_INVALID;
    }
    int st = check_gemv_shape(rq + 2 * rk, a->cols, a->n, a->x, a->q_out, err_msg, err_len, who);
    if (st != HKV_OK) return st;
    const void *ptrs[] = {a->wq, a->wk, a->wv, a->q_norm, a->k_norm, a->k_out, a->v_out};
    for (const void *q : ptrs) {
        if (q == nullptr || !aligned16(q)) {
            set_msg(err_msg, err_len, "%s: weights, norms and outputs must be 16-byte aligned device pointers",
                    who);
            return HKV_ERR_INVALID;
        }
    }
    if (a->norm != nullptr && !aligned16(a->norm)) {
        set_msg(err_msg, err_len, "%s: norm must be 16-byte aligned", who);
        return HKV_ERR_INVALID;
    }
    GemvParams p = {};
    p.w[0] = static_cast<const uint8_t *>(a->wq);
    p.w[1] = static_cast<const uint8_t *>(a->wk);
    p.w[2] = static_cast<const uint8_t *>(a->wv);
    p.row_end[0] = static_cast<int32_t>(rq);
    p.row_end[1] = static_cast<int32_t>(rq + rk);
    p.row_end[2] = static_cast<int32_t>(rq + 2 * rk);
    p.rows = p.row_end[2];
    p.cols = static_cast<int32_t>(a->cols);
    p.n = a->n;
    p.x = a->x;
    p.norm = a->norm;
    p.eps = a->eps;
    p.y[0] = a->q_out;
    p.y[1] = a->k_out;
    p.y[2] = a->v_out;
    p.y_rows[0] = static_cast<int32_t>(rq);
    p.y_rows[1] = p.y_rows[2] = static_cast<int32_t>(rk);
    p.head_norm[0] = a->q_norm;
    p.head_norm[1] = a->k_norm;
    p.tensor = a->tensor_cores != 0 ? 1 : 0;
    p.err = q4k_err_word();
    return finish(launch_gemv<kQkv>(p, static_cast<cudaStream_t>(stream)), err_msg, err_len, who);
}

extern "C" int hkv_q4k_sync_check(hkv_stream stream, char *err_msg, size_t err_len) {
    const char *who = "hkv_q4k_sync_check";
    cudaError_t st = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
    if (st != cudaSuccess) return finish(st, err_msg, err_len, who);
    hkv::DeviceError *w = q4k_err_word();
    if (w == nullptr) return finish(cudaErrorInvalidSymbol, err_msg, err_len, who);
    hkv::DeviceError e{};
    st = cudaMemcpy(&e, w, sizeof(e), cudaMemcpyDeviceToHost);
    if (st != cudaSuccess) return finish(st, err_msg, err_len, who);
    if (e.code != 0) {
        const hkv::DeviceError zero{};
        cudaMemcpy(w, &zero, sizeof(zero), cudaMemcpyHostToDevice);
        set_msg(err_msg, err_len, "%s: a weight copy of CTA %d did not complete", who, e.a);
        return HKV_ERR_TIMEOUT;
    }
    return HKV_OK;
}

// Internal launchers used by the backbone driver (hkv_backbone_host.cpp).
namespace hkv {
namespace bb {

cudaError_t launch_embed(const uint8_t *table, int64_t table_rows, int32_t cols, const int32_t *ids,
                         int32_t k, int32_t id_stride, int32_t n, float *out, DeviceError *err,
                         cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(cols / kQK), static_cast<unsigned>(n));
    cfg.blockDim = dim3(kQK);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, embed_kernel, table, table_rows, cols, ids, k, id_stride, n, out, err);
}

cudaError_t launch_argmax(const float *logits, int32_t n_books, int32_t size, int32_t n, int32_t *codes,
                          cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(n));
    cfg.blockDim = dim3(static_cast<unsigned>(32 * n_books));
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, argmax_kernel, logits, n_books, size, n, codes);
}

}  // namespace bb
}  // namespace hkv

// ====================================================== backbone object
struct hkv_backbone {
    hkv_engine *kv = nullptr;
    hkv_config cfg{};
    hkv_backbone_weights w{};
    std::vector<hkv_backbone_layer> layers;
    int32_t max_batch = 0;
    int32_t q_rows = 0, kv_rows = 0, logit_rows = 0;
    float *hidden = nullptr, *q = nullptr, *k = nullptr, *v = nullptr, *attn = nullptr;
    float *gated = nullptr, *logits = nullptr;
    int32_t *codes = nullptr, *ids = nullptr;
    int32_t *ids_host = nullptr;      // pinned staging for hkv_backbone_embed_text
    cudaEvent_t ids_done = nullptr;   // the staging copy has been read
    hkv::DeviceError *err = nullptr;
    int64_t launches = 0;             // kernels launched by this backbone (the engine counts its own)
    std::string last_error;
};

namespace {

int bb_fail(hkv_backbone *bb, int status, const char *fmt, ...) __attribute__((format(printf, 3, 4)));
int bb_fail(hkv_backbone *bb, int status, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    if (bb != nullptr) bb->last_error = buf;
    return status;
}

int bb_cuda(hkv_backbone *bb, cudaError_t st, const char *what) {
    if (st == cudaSuccess) return HKV_OK;
    return bb_fail(bb, HKV_ERR_CUDA, "%s: %s", what, cudaGetErrorString(st));
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        if (prev >= 0) cudaSetDevice(prev);
    }
};

void free_buffers(hkv_backbone *bb) {
    for (void *p : {static_cast<void *>(bb->hidden), static_cast<void *>(bb->q), static_cast<void *>(bb->k),
                    static_cast<void *>(bb->v), static_cast<void *>(bb->attn), static_cast<void *>(bb->gated),
                    static_cast<void *>(bb->logits), static_cast<void *>(bb->codes),
                    static_cast<void *>(bb->ids), static_cast<void *>(bb->err)}) {
        if (p != nullptr) cudaFree(p);
    }
    if (bb->ids_host != nullptr) cudaFreeHost(bb->ids_host);
    if (bb->ids_done != nullptr) cudaEventDestroy(bb->ids_done);
}

GemvParams plain_params(const void *w, int32_t rows, int32_t cols, int32_t n, const float *x,
                        const float *norm, float eps, const float *residual, float *y,
                        hkv::DeviceError *err) {
    GemvParams p = {};
    p.err = err;
    p.w[0] = static_cast<const uint8_t *>(w);
    p.rows = rows;
    p.row_end[0] = p.row_end[1] = p.row_end[2] = rows;
    p.cols = cols;
    p.n = n;
    p.x = x;
    p.norm = norm;
    p.eps = eps;
    p.residual = residual;
    p.y[0] = y;
    p.y_rows[0] = rows;
    return p;
}

}  // namespace

extern "C" {

int hkv_backbone_create(hkv_engine *kv, const hkv_backbone_weights *w, int32_t max_batch,
                        hkv_backbone **out) {
    if (kv == nullptr || w == nullptr || out == nullptr || max_batch <= 0) {
        return HKV_ERR_INVALID;
    }
    *out = nullptr;
    auto *bb = new hkv_backbone();
    hkv_engine_config(kv, &bb->cfg);
    const hkv_config &c = bb->cfg;
    if (c.device < 0) {
        delete bb;
        return HKV_ERR_NO_DEVICE;
    }
    if (w->hidden <= 0 || w->hidden % kQK != 0 || w->hidden > kMaxCols || w->ffn <= 0 ||
        w->ffn % kQK != 0 || w->ffn > kMaxCols || w->n_codebooks <= 0 || w->n_codebooks > 32 ||
        w->codebook_size <= 0 || w->text_vocab <= 0 || c.head_dim != kHeadDim ||
        static_cast<int64_t>(c.n_head) * kHeadDim > kMaxCols || w->layers == nullptr) {
        delete bb;
        return HKV_ERR_INVALID;
    }
    bool ok = aligned16(w->token_embd) && aligned16(w->audio_embd) && aligned16(w->output_norm) &&
              aligned16(w->audio_output) && w->token_embd && w->audio_embd && w->output_norm &&
              w->audio_output;
    for (int32_t l = 0; ok && l < c.n_layers; ++l) {
        const hkv_backbone_layer &L = w->layers[l];
        for (const void *q : {L.attn_q, L.attn_k, L.attn_v, L.attn_output, L.ffn_gate, L.ffn_up,
                              L.ffn_down, static_cast<const void *>(L.attn_norm),
                              static_cast<const void *>(L.ffn_norm),
                              static_cast<const void *>(L.attn_q_norm),
                              static_cast<const void *>(L.attn_k_norm)}) {
            ok = ok && q != nullptr && aligned16(q);
        }
    }
    if (!ok) {  // every weight must be a 16-byte aligned device pointer
        delete bb;
        return HKV_ERR_INVALID;
    }
    bb->kv = kv;
    bb->w = *w;
    bb->layers.assign(w->layers, w->layers + c.n_layers);
    bb->w.layers = nullptr;
    bb->max_batch = max_batch;
    bb->q_rows = c.n_head * kHeadDim;
    bb->kv_rows = c.n_head_kv * kHeadDim;
    bb->logit_rows = w->n_codebooks * w->codebook_size;
    DeviceGuard g(c.device);
    const size_t B = static_cast<size_t>(max_batch);
    cudaError_t st = cudaSuccess;
    auto alloc = [&](auto **p, size_t bytes) {
        if (st == cudaSuccess) st = cudaMalloc(reinterpret_cast<void **>(p), std::max<size_t>(bytes, 16));
    };
    alloc(&bb->hidden, B * w->hidden * 4);
    alloc(&bb->q, B * bb->q_rows * 4);
    alloc(&bb->k, B * bb->kv_rows * 4);
    alloc(&bb->v, B * bb->kv_rows * 4);
    alloc(&bb->attn, B * bb->q_rows * 4);
    alloc(&bb->gated, B * w->ffn * 4);
    alloc(&bb->logits, B * bb->logit_rows * 4);
    alloc(&bb->codes, B * w->n_codebooks * 4);
    alloc(&bb->ids, B * 4);
    alloc(&bb->err, sizeof(hkv::DeviceError));
    if (st == cudaSuccess) st = cudaMallocHost(reinterpret_cast<void **>(&bb->ids_host), B * 4);
    if (st == cudaSuccess) st = cudaEventCreateWithFlags(&bb->ids_done, cudaEventDisableTiming);
    if (st == cudaSuccess) st = cudaMemset(bb->err, 0, sizeof(hkv::DeviceError));
    if (st == cudaSuccess) st = cudaMemset(bb->codes, 0, B * w->n_codebooks * 4);
    if (st == cudaSuccess) st = cudaMemset(bb->hidden, 0, B * w->hidden * 4);
    if (st != cudaSuccess) {
        free_buffers(bb);
        delete bb;
        return HKV_ERR_CUDA;
    }
    *out = bb;
    return HKV_OK;
}

void hkv_backbone_destroy(hkv_backbone *bb) {
    if (bb == nullptr) return;
    DeviceGuard g(bb->cfg.device);
    cudaDeviceSynchronize();
    free_buffers(bb);
    delete bb;
}

const char *hkv_backbone_last_error(const hkv_backbone *bb) {
    return bb == nullptr ? "null backbone" : bb->last_error.c_str();
}

int hkv_backbone_embed_text(hkv_backbone *bb, int32_t n, const int32_t *ids, hkv_stream stream) {
    if (bb == nullptr) return HKV_ERR_INVALID;
    if (n <= 0 || n > bb->max_batch || ids == nullptr) {
        return bb_fail(bb, HKV_ERR_INVALID, "hkv_backbone_embed_text: n must be in [1, %d]", bb->max_batch);
    }
    for (int32_t e = 0; e < n; ++e) {
        if (ids[e] < 0 || ids[e] >= bb->w.text_vocab) {
            return bb_fail(bb, HKV_ERR_RANGE, "hkv_backbone_embed_text: id %d of entry %d outside [0, %lld)",
                           ids[e], e, static_cast<long long>(bb->w.text_vocab));
        }
    }
    DeviceGuard g(bb->cfg.device);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    int st = bb_cuda(bb, cudaEventSynchronize(bb->ids_done), "hkv_backbone_embed_text");
    if (st != HKV_OK) return st;
    std::memcpy(bb->ids_host, ids, static_cast<size_t>(n) * 4);
    st = bb_cuda(bb, cudaMemcpyAsync(bb->ids, bb->ids_host, static_cast<size_t>(n) * 4,
                                     cudaMemcpyHostToDevice, s), "hkv_backbone_embed_text");
    if (st != HKV_OK) return st;
    st = bb_cuda(bb, cudaEventRecord(bb->ids_done, s), "hkv_backbone_embed_text");
    if (st != HKV_OK) return st;
    ++bb->launches;
    return bb_cuda(bb, launch_embed(static_cast<const uint8_t *>(bb->w.token_embd), bb->w.text_vocab,
                                    bb->w.hidden, bb->ids, 1, 0, n, bb->hidden, bb->err, s),
                   "hkv_backbone_embed_text");
}

int hkv_backbone_embed_codes(hkv_backbone *bb, int32_t n, const int32_t *codes, hkv_stream stream) {
    if (bb == nullptr) return HKV_ERR_INVALID;
    if (n <= 0 || n > bb->max_batch) {
        return bb_fail(bb, HKV_ERR_INVALID, "hkv_backbone_embed_codes: n must be in [1, %d]", bb->max_batch);
    }
    if (codes != nullptr && (reinterpret_cast<uintptr_t>(codes) & 3u) != 0) {
        return bb_fail(bb, HKV_ERR_INVALID, "hkv_backbone_embed_codes: codes must be 4-byte aligned");
    }
    DeviceGuard g(bb->cfg.device);
    ++bb->launches;
    return bb_cuda(bb, launch_embed(static_cast<const uint8_t *>(bb->w.audio_embd),
                                    static_cast<int64_t>(bb->logit_rows), bb->w.hidden,
                                    codes != nullptr ? codes : bb->codes, bb->w.n_codebooks,
                                    bb->w.codebook_size, n, bb->hidden, bb->err,
                                    static_cast<cudaStream_t>(stream)),
                   "hkv_backbone_embed_codes");
}

int hkv_backbone_decode(hkv_backbone *bb, int32_t n, const int32_t *slots, int32_t want_logits,
                        hkv_stream stream) {
    if (bb == nullptr) return HKV_ERR_INVALID;
    if (n <= 0 || n > bb->max_batch || slots == nullptr) {
        return bb_fail(bb, HKV_ERR_INVALID, "hkv_backbone_decode: n must be in [1, %d]", bb->max_batch);
    }
    DeviceGuard g(bb->cfg.device);
    const cudaStream_t s = static_cast<cudaStream_t>(stream);
    const hkv_backbone_weights &w = bb->w;
    const float eps = w.rms_eps;
    // one kernel family for every batch size of this backbone, so a
    // request's results do not depend on how many share its step
    const int32_t tc = bb->max_batch > 1 ? 1 : 0;
    auto with_tc = [tc](GemvParams q) {
        q.tensor = tc;
        return q;
    };
    for (int32_t l = 0; l < bb->cfg.n_layers; ++l) {
        const hkv_backbone_layer &L = bb->layers[static_cast<size_t>(l)];
        // q, k, v with the per-head norms (:5709-5733)
        GemvParams p = {};
        p.w[0] = static_cast<const uint8_t *>(L.attn_q);
        p.w[1] = static_cast<const uint8_t *>(L.attn_k);
        p.w[2] = static_cast<const uint8_t *>(L.attn_v);
        p.row_end[0] = bb->q_rows;
        p.row_end[1] = bb->q_rows + bb->kv_rows;
        p.row_end[2] = bb->q_rows + 2 * bb->kv_rows;
        p.rows = p.row_end[2];
        p.cols = w.hidden;
        p.n = n;
        p.x = bb->hidden;
        p.norm = L.attn_norm;
        p.eps = eps;
        p.y[0] = bb->q;
        p.y[1] = bb->k;
        p.y[2] = bb->v;
        p.y_rows[0] = bb->q_rows;
        p.y_rows[1] = p.y_rows[2] = bb->kv_rows;
        p.head_norm[0] = L.attn_q_norm;
        p.head_norm[1] = L.attn_k_norm;
        p.err = bb->err;
        p.tensor = tc;
        int st = bb_cuda(bb, launch_gemv<kQkv>(p, s, &bb->launches), "hkv_backbone_decode: q/k/v");
        if (st != HKV_OK) return st;
        // RoPE + append + attention (:5734-5786)
        st = hkv_decode_step(bb->kv, l, n, slots, bb->q, bb->k, bb->v, bb->attn, stream);
        if (st != HKV_OK) {
            return bb_fail(bb, st, "hkv_backbone_decode: layer %d: %s", l, hkv_last_error(bb->kv));
        }
        // h = h + Wo attn (:5790-5791)
        st = bb_cuda(bb, launch_gemv<kPlain>(with_tc(plain_params(L.attn_output, w.hidden, bb->q_rows, n, bb->attn,
                                                                  nullptr, eps, bb->hidden, bb->hidden, bb->err)),
                                             s, &bb->launches),
                     "hkv_backbone_decode: o_proj");
        if (st != HKV_OK) return st;
        // g = silu(Wg m) * (Wu m), m = rms_norm(h) * ffn_norm (:5806-5822)
        GemvParams f = plain_params(L.ffn_gate, w.ffn, w.hidden, n, bb->hidden, L.ffn_norm, eps, nullptr,
                                    bb->gated, bb->err);
        f.w[1] = static_cast<const uint8_t *>(L.ffn_up);
        f.tensor = tc;
        st = bb_cuda(bb, launch_gemv<kSwiglu>(f, s, &bb->launches), "hkv_backbone_decode: gate/up");
        if (st != HKV_OK) return st;
        // h = h + Wd g (:5823, :5843)
        st = bb_cuda(bb, launch_gemv<kPlain>(with_tc(plain_params(L.ffn_down, w.hidden, w.ffn, n, bb->gated,
                                                                  nullptr, eps, bb->hidden, bb->hidden, bb->err)),
                                             s, &bb->launches),
                     "hkv_backbone_decode: down");
        if (st != HKV_OK) return st;
    }
    int st = hkv_slot_advance(bb->kv, n, slots, 1);
    if (st != HKV_OK) {
        return bb_fail(bb, st, "hkv_backbone_decode: advance: %s", hkv_last_error(bb->kv));
    }
    if (want_logits) {
        // logits = a.output (rms_norm(h) * output_norm) (:5858-5863), greedy codes
        st = bb_cuda(bb, launch_gemv<kPlain>(with_tc(plain_params(w.audio_output, bb->logit_rows, w.hidden, n,
                                                                  bb->hidden, w.output_norm, eps, nullptr,
                                                                  bb->logits, bb->err)),
                                             s, &bb->launches),
                     "hkv_backbone_decode: output head");
        if (st != HKV_OK) return st;
        st = bb_cuda(bb, launch_argmax(bb->logits, w.n_codebooks, w.codebook_size, n, bb->codes, s),
                     "hkv_backbone_decode: argmax");
        if (st != HKV_OK) return st;
        ++bb->launches;
    }
    return HKV_OK;
}

int hkv_backbone_kernel_launches(const hkv_backbone *bb, int64_t *launches) {
    if (bb == nullptr || launches == nullptr) return HKV_ERR_INVALID;
    *launches = bb->launches;
    return HKV_OK;
}

int hkv_backbone_buffers(const hkv_backbone *bb, float **hidden, float **logits, int32_t **codes) {
    if (bb == nullptr) return HKV_ERR_INVALID;
    if (hidden) *hidden = bb->hidden;
    if (logits) *logits = bb->logits;
    if (codes) *codes = bb->codes;
    return HKV_OK;
}

int hkv_backbone_sync_check(hkv_backbone *bb, hkv_stream stream) {
    if (bb == nullptr) return HKV_ERR_INVALID;
    DeviceGuard g(bb->cfg.device);
    int st = bb_cuda(bb, cudaStreamSynchronize(static_cast<cudaStream_t>(stream)), "hkv_backbone_sync_check");
    if (st != HKV_OK) return st;
    hkv::DeviceError e{};
    st = bb_cuda(bb, cudaMemcpy(&e, bb->err, sizeof(e), cudaMemcpyDeviceToHost), "hkv_backbone_sync_check");
    if (st != HKV_OK) return st;
    if (e.code != 0) {
        cudaMemset(bb->err, 0, sizeof(e));
        if (e.code == kErrTimeout) {
            return bb_fail(bb, HKV_ERR_TIMEOUT, "weight copy of CTA %d, stage %d did not complete", e.a, e.b);
        }
        return bb_fail(bb, HKV_ERR_DEVICE, "embedding id %d of entry %d outside the table", e.b, e.a);
    }
    return HKV_OK;
}

}  // extern "C"
