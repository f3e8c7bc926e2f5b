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
//   * gemv_kernel: one pass over a Q4_K matrix, HBM-bound.  Every CTA first
//     issues its first weight loads, then (after the previous kernel in the
//     stream has finished: griddepcontrol.wait) quantises the activation
//     vectors to Q8_K in shared memory -- optionally after the RMSNorm, done
//     in double like GGML -- and streams the rest of its rows with 16-byte
//     loads two superblocks ahead, dotting 4-bit weights with 8-bit
//     activations by dp4a.  Epilogues: store, add a residual, SwiGLU of two
//     matrices, or the per-head RMSNorm of q and k, whose 128 rows span a
//     cluster of 4 CTAs that add their sums of squares through distributed
//     shared memory.
//   * q4k_quantize_kernel: the repo's Q4_K encoder (weights for tests and the
//     benchmark; the reference quantises with GGML's tools offline).
//   * embed_kernel / argmax_kernel: embedding rows (text ids or the sum of
//     8 audio-codebook rows) and greedy codes per codebook.
//
// No TMA, no multicast: plain vector loads of this GPU's own memory.
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
#include "hkv_internal.h"

namespace cg = cooperative_groups;

namespace hkv {
namespace bb {

constexpr int kQK = 256;        // weights per Q4_K / Q8_K block
constexpr int kQ4Bytes = 144;   // bytes per Q4_K block
constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;
constexpr int kMaxVec = 8;      // activation vectors per launch
constexpr int kClusterCtas = 4; // CTAs per head in the q/k/v launch (32 rows each)
constexpr int kMaxCols = 16384;

enum Mode { kPlain = 0, kSwiglu = 1, kQkv = 2 };

struct GemvParams {
    const uint8_t *w[3];      // kPlain: w[0]; kSwiglu: gate, up; kQkv: q, k, v
    int32_t row_end[3];       // virtual row boundaries of the matrices (kQkv)
    int32_t rows;             // virtual rows
    int32_t cols;
    int32_t n;                // activation vectors, <= kMaxVec
    const float *x;           // [n][cols]
    const float *norm;        // nullptr or [cols]
    float eps;
    const float *residual;    // nullptr or [n][rows] (kPlain)
    float *y[3];              // outputs, [n][y_rows[m]] each
    int32_t y_rows[3];
    const float *head_norm[2];  // kQkv: q_norm, k_norm [128]
};

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

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

// Shared-memory image of the Q8_K activations.
struct Q8View {
    int8_t *q;   // [n][cols]
    float *d;    // [n][nsb]
    int32_t *s;  // [n][nsb * 8]: sum of q over each 32-element sub-block
    double *red; // [kWarps + 1] reduction scratch
};

__host__ __device__ inline size_t q8_smem_bytes(int n, int cols) {
    const int nsb = cols / kQK;
    size_t b = static_cast<size_t>(n) * cols;          // q
    b = (b + 15) & ~size_t(15);
    b += static_cast<size_t>(n) * nsb * 4;             // d
    b = (b + 15) & ~size_t(15);
    b += static_cast<size_t>(n) * nsb * 8 * 4;         // s
    b = (b + 15) & ~size_t(15);
    b += (kWarps + 1) * sizeof(double);                // red
    b = (b + 15) & ~size_t(15);
    return b;
}

__device__ inline Q8View carve_q8(unsigned char *smem, int n, int cols) {
    const int nsb = cols / kQK;
    Q8View v;
    size_t off = 0;
    v.q = reinterpret_cast<int8_t *>(smem);
    off = (static_cast<size_t>(n) * cols + 15) & ~size_t(15);
    v.d = reinterpret_cast<float *>(smem + off);
    off = (off + static_cast<size_t>(n) * nsb * 4 + 15) & ~size_t(15);
    v.s = reinterpret_cast<int32_t *>(smem + off);
    off = (off + static_cast<size_t>(n) * nsb * 32 + 15) & ~size_t(15);
    v.red = reinterpret_cast<double *>(smem + off);
    return v;
}

// Q8_K quantisation of the n activation vectors (GGML's quantize_row_q8_K:
// iscale = -127 / (element of largest magnitude, the first on ties),
// q = min(127, round-half-even(iscale * x)), d = 1 / iscale), optionally of
// rms_norm(x) * norm (sum of squares in double, mean rounded to float,
// scale = 1 / sqrtf(mean + eps)).  Ends with a CTA barrier.
__device__ void quantize_activations(const GemvParams &p, const Q8View &a) {
    const int nsb = p.cols / kQK;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int e = 0; e < p.n; ++e) {
        const float *x = p.x + static_cast<size_t>(e) * p.cols;
        float scale = 1.0f;
        if (p.norm != nullptr) {
            double s = 0.0;
            for (int i = threadIdx.x; i < p.cols; i += kThreads) {
                const float v = x[i];
                s += static_cast<double>(__fmul_rn(v, v));
            }
            s = warp_sum_double(s);
            if (lane == 0) a.red[warp] = s;
            __syncthreads();
            if (threadIdx.x == 0) {
                double t = 0.0;
                for (int w = 0; w < kWarps; ++w) t += a.red[w];
                a.red[kWarps] = t;
            }
            __syncthreads();
            const float mean = static_cast<float>(a.red[kWarps] / static_cast<double>(p.cols));
            scale = 1.0f / sqrtf(mean + p.eps);
            __syncthreads();  // a.red is reused by the next vector
        }
        for (int b = warp; b < nsb; b += kWarps) {
            const int base = b * kQK + lane * 8;
            const float4 u0 = *reinterpret_cast<const float4 *>(x + base);
            const float4 u1 = *reinterpret_cast<const float4 *>(x + base + 4);
            float v[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
            if (p.norm != nullptr) {
                const float4 w0 = *reinterpret_cast<const float4 *>(p.norm + base);
                const float4 w1 = *reinterpret_cast<const float4 *>(p.norm + base + 4);
                const float w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
                for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], scale), w[i]);
            }
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
            float d = 0.0f;
            if (am == 0.0f) {
#pragma unroll
                for (int i = 0; i < 8; ++i) q[i] = 0;
            } else {
                const float iscale = -127.0f / mx;
#pragma unroll
                for (int i = 0; i < 8; ++i) q[i] = min(127, __float2int_rn(__fmul_rn(iscale, v[i])));
                d = 1.0f / iscale;
            }
            uint32_t lo = 0, hi = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                lo |= (static_cast<uint32_t>(q[i]) & 0xFFu) << (8 * i);
                hi |= (static_cast<uint32_t>(q[i + 4]) & 0xFFu) << (8 * i);
            }
            *reinterpret_cast<uint2 *>(a.q + static_cast<size_t>(e) * p.cols + base) = make_uint2(lo, hi);
            int qs = 0;
#pragma unroll
            for (int i = 0; i < 8; ++i) qs += q[i];
            qs += __shfl_xor_sync(0xffffffffu, qs, 1);
            qs += __shfl_xor_sync(0xffffffffu, qs, 2);
            if ((lane & 3) == 0) a.s[(e * nsb + b) * 8 + (lane >> 2)] = qs;
            if (lane == 0) a.d[e * nsb + b] = d;
        }
    }
    __syncthreads();
}

// One thread's share of a Q4_K block: the 16-byte header and the 32 bytes of
// quants of sub-block pair `part` (sub-blocks 2*part and 2*part + 1).
struct BlockPart {
    int4 hdr, q0, q1;
};

__device__ __forceinline__ void load_part(BlockPart &b, const uint8_t *blk, int part) {
    b.hdr = ld_stream(blk);
    b.q0 = ld_stream(blk + 16 + 32 * part);
    b.q1 = ld_stream(blk + 32 + 32 * part);
}

// Partial dot product of one block part with activation vector e.
__device__ __forceinline__ float dot_part(const BlockPart &b, const Q8View &a, int cols, int nsb,
                                          int sb, int part, int e) {
    const uint32_t h0 = static_cast<uint32_t>(b.hdr.x);
    const float d4 = half_bits(h0);
    const float dm4 = half_bits(h0 >> 16);
    int sc0, m0, sc1, m1;
    const uint32_t s0 = b.hdr.y, s1 = b.hdr.z, s2 = b.hdr.w;
    scale_min(s0, s1, s2, 2 * part, sc0, m0);
    scale_min(s0, s1, s2, 2 * part + 1, sc1, m1);
    const int4 *ap = reinterpret_cast<const int4 *>(a.q + static_cast<size_t>(e) * cols + sb * kQK +
                                                    64 * part);
    const int4 a0 = ap[0], a1 = ap[1], a2 = ap[2], a3 = ap[3];
    const uint32_t qw[8] = {(uint32_t)b.q0.x, (uint32_t)b.q0.y, (uint32_t)b.q0.z, (uint32_t)b.q0.w,
                            (uint32_t)b.q1.x, (uint32_t)b.q1.y, (uint32_t)b.q1.z, (uint32_t)b.q1.w};
    const int alo[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
    const int ahi[8] = {a2.x, a2.y, a2.z, a2.w, a3.x, a3.y, a3.z, a3.w};
    int sum0 = 0, sum1 = 0;
#pragma unroll
    for (int k = 0; k < 8; ++k) {
        sum0 = __dp4a(static_cast<int>(qw[k] & 0x0F0F0F0Fu), alo[k], sum0);
        sum1 = __dp4a(static_cast<int>((qw[k] >> 4) & 0x0F0F0F0Fu), ahi[k], sum1);
    }
    const int isum = sc0 * sum0 + sc1 * sum1;
    const int32_t *ss = a.s + (e * nsb + sb) * 8 + 2 * part;
    const int msum = m0 * ss[0] + m1 * ss[1];
    const float d8 = a.d[e * nsb + sb];
    return __fmul_rn(d4, d8) * static_cast<float>(isum) - __fmul_rn(dm4, d8) * static_cast<float>(msum);
}

// TPR threads per weight row (8 or 32); NB activation vectors (1 or kMaxVec).
template <int TPR, int MODE, int NB>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(GemvParams p) {
    extern __shared__ __align__(16) unsigned char smem[];
    constexpr int kRowsPerWarp = 32 / TPR;
    constexpr int kRows = kWarps * kRowsPerWarp;
    constexpr int kStep = TPR / 4;  // blocks per row per iteration
    constexpr int kMats = MODE == kSwiglu ? 2 : 1;
    const int nsb = p.cols / kQK;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int local_row = warp * kRowsPerWarp + lane / TPR;
    const int row = blockIdx.x * kRows + local_row;
    const int t = lane % TPR;
    const int sb0 = t >> 2, part = t & 3;
    const bool ok = row < p.rows;
    int m = 0, row_in = row;
    if (MODE == kQkv) {
        m = row < p.row_end[0] ? 0 : (row < p.row_end[1] ? 1 : 2);
        row_in = row - (m == 0 ? 0 : p.row_end[m - 1]);
    }
    const size_t row_bytes = static_cast<size_t>(nsb) * kQ4Bytes;
    const uint8_t *wr[kMats];
#pragma unroll
    for (int k = 0; k < kMats; ++k) {
        wr[k] = ok ? p.w[MODE == kSwiglu ? k : m] + static_cast<size_t>(row_in) * row_bytes : nullptr;
    }

    // Weights do not depend on the previous kernel: start streaming them
    // before waiting for it.
    BlockPart cur[2][kMats], nxt[2][kMats];
    auto load2 = [&](int base, BlockPart (&buf)[2][kMats]) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int sb = base + u * kStep;
            if (ok && sb < nsb) {
#pragma unroll
                for (int k = 0; k < kMats; ++k) load_part(buf[u][k], wr[k] + sb * kQ4Bytes, part);
            }
        }
    };
    load2(sb0, cur);

    pdl_wait();
    const Q8View a = carve_q8(smem, p.n, p.cols);
    quantize_activations(p, a);

    float acc[kMats][NB];
#pragma unroll
    for (int k = 0; k < kMats; ++k)
#pragma unroll
        for (int e = 0; e < NB; ++e) acc[k][e] = 0.0f;

    for (int base = sb0; base < nsb; base += 2 * kStep) {
        if (base + 2 * kStep < nsb) load2(base + 2 * kStep, nxt);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            const int sb = base + u * kStep;
            if (ok && sb < nsb) {
#pragma unroll
                for (int k = 0; k < kMats; ++k)
#pragma unroll
                    for (int e = 0; e < NB; ++e)
                        if (e < p.n) acc[k][e] += dot_part(cur[u][k], a, p.cols, nsb, sb, part, e);
            }
        }
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
            for (int k = 0; k < kMats; ++k) cur[u][k] = nxt[u][k];
    }
    pdl_trigger();

#pragma unroll
    for (int k = 0; k < kMats; ++k)
#pragma unroll
        for (int e = 0; e < NB; ++e)
#pragma unroll
            for (int off = TPR / 2; off > 0; off >>= 1)
                acc[k][e] += __shfl_xor_sync(0xffffffffu, acc[k][e], off);

    if (MODE == kPlain) {
        if (ok && t == 0) {
#pragma unroll
            for (int e = 0; e < NB; ++e) {
                if (e < p.n) {
                    const size_t o = static_cast<size_t>(e) * p.rows + row;
                    p.y[0][o] = p.residual != nullptr ? p.residual[o] + acc[0][e] : acc[0][e];
                }
            }
        }
    } else if (MODE == kSwiglu) {
        if (ok && t == 0) {
#pragma unroll
            for (int e = 0; e < NB; ++e) {
                if (e < p.n) {
                    const float g = acc[0][e];
                    const float s = g / (1.0f + expf(-g));
                    p.y[0][static_cast<size_t>(e) * p.rows + row] = s * acc[1][e];
                }
            }
        }
    } else {
        // q / k / v rows; the 4 CTAs of a cluster hold the 128 rows of one head.
        float *res = reinterpret_cast<float *>(smem + q8_smem_bytes(p.n, p.cols));  // [NB][kRows]
        double *part_ss = reinterpret_cast<double *>(res + NB * kRows);             // [NB]
        if (t == 0) {
#pragma unroll
            for (int e = 0; e < NB; ++e)
                if (e < p.n) res[e * kRows + local_row] = acc[0][e];
        }
        __syncthreads();
        cg::cluster_group cl = cg::this_cluster();
        const bool normed = m < 2;  // the same for every CTA of the cluster
        if (normed && warp == 0) {
            for (int e = 0; e < p.n; ++e) {
                const float v = res[e * kRows + lane];
                const double s = warp_sum_double(static_cast<double>(__fmul_rn(v, v)));
                if (lane == 0) part_ss[e] = s;
            }
        }
        cl.sync();
        __shared__ float scale_s[NB];
        if (normed && threadIdx.x < p.n) {
            const int e = threadIdx.x;
            double total = 0.0;
            for (int r = 0; r < kClusterCtas; ++r) total += *cl.map_shared_rank(part_ss + e, r);
            const float mean = static_cast<float>(total / static_cast<double>(kHeadDim));
            scale_s[e] = 1.0f / sqrtf(mean + p.eps);
        }
        cl.sync();  // every CTA has read its peers' sums before any of them exits
        const int dim0 = static_cast<int>(cl.block_rank()) * kRows;
        const int row0 = blockIdx.x * kRows;
        const int mrow0 = row0 - (m == 0 ? 0 : p.row_end[m - 1]);
        for (int i = threadIdx.x; i < p.n * kRows; i += kThreads) {
            const int e = i / kRows, r = i % kRows;
            if (row0 + r < p.rows) {
                float v = res[e * kRows + r];
                if (normed) v = __fmul_rn(__fmul_rn(v, scale_s[e]), p.head_norm[m][dim0 + r]);
                p.y[m][static_cast<size_t>(e) * p.y_rows[m] + mrow0 + r] = v;
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
// summed in j order (the reference's chain of ggml_add, :2919-2924).
__global__ void embed_kernel(const uint8_t *table, int64_t table_rows, int32_t cols,
                             const int32_t *ids, int32_t k, int32_t id_stride, int32_t n,
                             float *out, DeviceError *err) {
    pdl_wait();
    const int e = blockIdx.x;
    if (e >= n) return;
    const int nsb = cols / kQK;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) {
        const int sb = i / kQK, pos = i % kQK;
        const int pair = pos >> 6, hi = (pos >> 5) & 1, l = pos & 31;
        float acc = 0.0f;
        for (int j = 0; j < k; ++j) {
            const int32_t code = ids[e * k + j];
            const int64_t id = static_cast<int64_t>(code) + static_cast<int64_t>(j) * id_stride;
            if (code < 0 || (k > 1 && code >= id_stride) || id >= table_rows) {
                if (atomicCAS(&err->code, 0, kErrBadIndex) == 0) {
                    err->where = HKV_KERNEL_EMBED;
                    err->a = e;
                    err->b = static_cast<int32_t>(id);
                }
                continue;
            }
            const uint8_t *blk = table + (id * nsb + sb) * kQ4Bytes;
            uint16_t dbits, mbits;
            memcpy(&dbits, blk, 2);
            memcpy(&mbits, blk + 2, 2);
            const float d = __half2float(__ushort_as_half(dbits));
            const float dmin = __half2float(__ushort_as_half(mbits));
            int sc, m;
            const uint32_t *sw = reinterpret_cast<const uint32_t *>(blk + 4);
            scale_min(sw[0], sw[1], sw[2], 2 * pair + hi, sc, m);
            const uint32_t q = (blk[16 + 32 * pair + l] >> (4 * hi)) & 0x0Fu;
            const float v = __fsub_rn(__fmul_rn(__fmul_rn(d, static_cast<float>(sc)), static_cast<float>(q)),
                                      __fmul_rn(dmin, static_cast<float>(m)));
            acc = j == 0 ? v : __fadd_rn(acc, v);
        }
        out[static_cast<size_t>(e) * cols + i] = acc;
    }
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
size_t gemv_smem(int mode, int nb, int n, int cols, int tpr) {
    size_t b = q8_smem_bytes(n, cols);
    if (mode == kQkv) {
        const int rows = kWarps * (32 / tpr);
        b += static_cast<size_t>(nb) * rows * sizeof(float) + static_cast<size_t>(nb) * sizeof(double) + 16;
    }
    return b;
}

template <int TPR, int MODE, int NB>
cudaError_t launch_one(const GemvParams &p, cudaStream_t stream) {
    constexpr int kRows = kWarps * (32 / TPR);
    auto kern = gemv_kernel<TPR, MODE, NB>;
    const size_t smem = gemv_smem(MODE, NB, p.n, p.cols, TPR);
    // Opt in to the largest dynamic shared memory once per device.
    static std::mutex mu;
    static bool done[64] = {};
    int dev = 0;
    cudaError_t st = cudaGetDevice(&dev);
    if (st != cudaSuccess) return st;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (dev < 64 && !done[dev]) {
            st = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(q8_smem_bytes(kMaxVec, kMaxCols) + 64 * 1024));
            if (st != cudaSuccess) return st;
            done[dev] = true;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((p.rows + kRows - 1) / kRows));
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    int na = 1;
    if (MODE == kQkv) {
        attr[1].id = cudaLaunchAttributeClusterDimension;
        attr[1].val.clusterDim.x = kClusterCtas;
        attr[1].val.clusterDim.y = 1;
        attr[1].val.clusterDim.z = 1;
        na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, kern, p);
}

template <int MODE>
cudaError_t launch_gemv(GemvParams p, cudaStream_t stream) {
    // Chunks of at most kMaxVec vectors; one vector takes the NB = 1 kernel.
    const int n_total = p.n;
    for (int e0 = 0; e0 < n_total; e0 += kMaxVec) {
        GemvParams q = p;
        q.n = std::min(kMaxVec, n_total - e0);
        q.x = p.x + static_cast<size_t>(e0) * p.cols;
        if (q.residual) q.residual += static_cast<size_t>(e0) * p.rows;
        for (int k = 0; k < 3; ++k) {
            if (q.y[k]) q.y[k] += static_cast<size_t>(e0) * (MODE == kQkv ? p.y_rows[k] : p.rows);
        }
        cudaError_t st;
        // Rows per CTA: 32 (8 threads per row) for tall matrices, 8 (a warp per
        // row) when 32-row CTAs would leave SMs idle.
        const bool tall = MODE == kQkv || p.rows >= 4096;
        if (q.n == 1) {
            st = tall ? launch_one<8, MODE, 1>(q, stream)
                      : (MODE == kQkv ? cudaErrorInvalidValue : launch_one<32, MODE == kQkv ? kPlain : MODE, 1>(q, stream));
        } else {
            st = tall ? launch_one<8, MODE, kMaxVec>(q, stream)
                      : (MODE == kQkv ? cudaErrorInvalidValue
                                      : launch_one<32, MODE == kQkv ? kPlain : MODE, kMaxVec>(q, stream));
        }
        if (st != cudaSuccess) return st;
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
    p.row_end[0] = p.row_end[1] = p.row_end[2] = p.rows;
    p.cols = static_cast<int32_t>(a->cols);
    p.n = a->n;
    p.x = a->x;
    p.norm = a->norm;
    p.eps = a->eps;
    p.residual = a->residual;
    p.y[0] = a->y;
    p.y_rows[0] = p.rows;
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
    return finish(launch_gemv<kQkv>(p, static_cast<cudaStream_t>(stream)), err_msg, err_len, who);
}

// Internal launchers used by the backbone driver (hkv_backbone_host.cpp).
namespace hkv {
namespace bb {

cudaError_t launch_embed(const uint8_t *table, int64_t table_rows, int32_t cols, const int32_t *ids,
                         int32_t k, int32_t id_stride, int32_t n, float *out, DeviceError *err,
                         cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(n));
    cfg.blockDim = dim3(kThreads);
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
                        const float *norm, float eps, const float *residual, float *y) {
    GemvParams p = {};
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
        int st = bb_cuda(bb, launch_gemv<kQkv>(p, s), "hkv_backbone_decode: q/k/v");
        if (st != HKV_OK) return st;
        // RoPE + append + attention (:5734-5786)
        st = hkv_decode_step(bb->kv, l, n, slots, bb->q, bb->k, bb->v, bb->attn, stream);
        if (st != HKV_OK) {
            return bb_fail(bb, st, "hkv_backbone_decode: layer %d: %s", l, hkv_last_error(bb->kv));
        }
        // h = h + Wo attn (:5790-5791)
        st = bb_cuda(bb, launch_gemv<kPlain>(plain_params(L.attn_output, w.hidden, bb->q_rows, n, bb->attn,
                                                          nullptr, eps, bb->hidden, bb->hidden), s),
                     "hkv_backbone_decode: o_proj");
        if (st != HKV_OK) return st;
        // g = silu(Wg m) * (Wu m), m = rms_norm(h) * ffn_norm (:5806-5822)
        GemvParams f = plain_params(L.ffn_gate, w.ffn, w.hidden, n, bb->hidden, L.ffn_norm, eps, nullptr,
                                    bb->gated);
        f.w[1] = static_cast<const uint8_t *>(L.ffn_up);
        st = bb_cuda(bb, launch_gemv<kSwiglu>(f, s), "hkv_backbone_decode: gate/up");
        if (st != HKV_OK) return st;
        // h = h + Wd g (:5823, :5843)
        st = bb_cuda(bb, launch_gemv<kPlain>(plain_params(L.ffn_down, w.hidden, w.ffn, n, bb->gated, nullptr,
                                                          eps, bb->hidden, bb->hidden), s),
                     "hkv_backbone_decode: down");
        if (st != HKV_OK) return st;
    }
    int st = hkv_slot_advance(bb->kv, n, slots, 1);
    if (st != HKV_OK) {
        return bb_fail(bb, st, "hkv_backbone_decode: advance: %s", hkv_last_error(bb->kv));
    }
    if (want_logits) {
        // logits = a.output (rms_norm(h) * output_norm) (:5858-5863), greedy codes
        st = bb_cuda(bb, launch_gemv<kPlain>(plain_params(w.audio_output, bb->logit_rows, w.hidden, n,
                                                          bb->hidden, w.output_norm, eps, nullptr,
                                                          bb->logits), s),
                     "hkv_backbone_decode: output head");
        if (st != HKV_OK) return st;
        st = bb_cuda(bb, launch_argmax(bb->logits, w.n_codebooks, w.codebook_size, n, bb->codes, s),
                     "hkv_backbone_decode: argmax");
        if (st != HKV_OK) return st;
    }
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
        return bb_fail(bb, HKV_ERR_DEVICE, "embedding id %d of entry %d outside the table", e.b, e.a);
    }
    return HKV_OK;
}

}  // extern "C"
