// hkv_kernels.cu -- sm_100a kernels of the paged KV decode engine.
//
//   append_kernel     fused NEOX RoPE (BF16 table) + F32->F16 + row write into
//                     the row's physical page, one warp per (row, KV head),
//                     one 16-byte store per lane.
//   attention_kernel  split-K ("stream-K") flash-decode over all slots of a
//                     batch: the flattened (slot, KV head, page) unit range is
//                     cut into equal shares, one per warp; each warp streams
//                     its head blocks through a private ring of TMA bulk
//                     copies (cp.async.bulk + mbarrier) and keeps the 4 query
//                     heads of its KV head together so every K/V byte is read
//                     from HBM once.  QK^T and PV run on the tensor cores
//                     (mma.sync m16n8k16, F32 accumulate) with each F32
//                     operand split into an F16 high part and an F16 residual
//                     that ride in the otherwise-empty columns of the n=8
//                     tile, which keeps products at F32 accuracy.  Online
//                     softmax in base 2 with warp-shuffle reductions.  A
//                     warp whose share covers a whole (slot, KV head) writes
//                     the output; otherwise each share writes a partial
//                     (m, l, o) and the last share to finish (atomic ticket)
//                     merges them (log-sum-exp) into the head-major output.
//                     In the fused decode step the warp owning a slot's last
//                     page also ropes and writes the slot's new K/V row.
//   gather_kernel     logical [pos][kv_head][dim] view of one slot's layer.
//
// Waits on mbarriers are bounded (clock64 budget); a kernel that gives up
// records kErrTimeout in the DeviceError word, drains its own copies (again
// bounded) and returns.  Bounds checks record kErrBadIndex and skip the
// access.  No kernel traps.
#include <cuda_fp16.h>
#include <stdint.h>

#include <mutex>

#include "hkv_device.cuh"
#include "hkv_internal.h"

namespace hkv {
namespace {

using namespace dev;

constexpr int kStageBytes = 2 * kHeadBlockBytes;  // K block + V block
constexpr int kQcStride = 136;                     // halves per staged-query row (272 B)
constexpr int kQcBytes = 8 * kQcStride * 2;        // 8 rows: 4 heads x {hi, lo}
constexpr int kPBufBytes = 16 * 16;                // 16 tokens x 8 halves
constexpr int kBarBytes = (kAttnStages * 8 + 15) / 16 * 16;  // one 8-byte mbarrier per stage
constexpr int kWarpSmem = kAttnStages * kStageBytes + kQcBytes + kPBufBytes + kBarBytes;
// CTA-level partials: two slots per warp (the run a warp does not start, and
// the run it starts), each o[4][128] + (m, l)[4]; then one ticket per run.
constexpr int kCtaPartFloats = kGqa * kHeadDim + 2 * kGqa;
constexpr int kCtaPartBytes = kCtaPartFloats * 4;
constexpr int kCtaSmem = kAttnWarps * 2 * kCtaPartBytes + 32;
// Cluster merge (plan_cluster): one partial slot per CTA of the cluster, used
// in the cluster's first CTA, then the mbarrier that counts the filled slots.
constexpr int kMaxCluster = 16;
constexpr int kClusterSmem = kMaxCluster * kCtaPartBytes + 16;
constexpr int kWhereAppend = 0;
constexpr int kWhereAttn = 1;
constexpr int kWhereGather = 3;
constexpr int kWhereCow = 4;
constexpr int kWhereSplitWait = 5;

static_assert(kWarpSmem % 16 == 0, "per-warp shared region must keep 16-byte alignment");
static_assert(kBarBytes >= 8 * kAttnStages, "every stage needs its mbarrier inside the warp's region");
static_assert(kAttnWarps * kWarpSmem + kCtaSmem + kClusterSmem <= 227 * 1024,
              "attention CTA exceeds shared memory");
static_assert(kCtaPartBytes % 16 == 0, "CTA partial slots must keep 16-byte alignment");
static_assert(kAttnWarps <= 8, "one run ticket per warp in 32 bytes");

__device__ __forceinline__ void record_error(DeviceError *err, int code, int where, int a, int b) {
    if (atomicCAS(&err->code, 0, code) == 0) {
        err->where = where;
        err->a = a;
        err->b = b;
    }
}

// ------------------------------------------------------- ldmatrix / mma
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2,
                                        uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t &r0, uint32_t &r1,
                                              uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr)
                 : "memory");
}
__device__ __forceinline__ void ldsm_x2_trans(uint32_t addr, uint32_t &r0, uint32_t &r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16 {%0,%1}, [%2];"
                 : "=r"(r0), "=r"(r1)
                 : "r"(addr)
                 : "memory");
}
// D = A(16x16, row) * B(16x8, col) + D, F16 inputs, F32 accumulators.
__device__ __forceinline__ void mma_16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
    const __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ float f16_residual(float x) {
    return __fsub_rn(x, __half2float(__float2half_rn(x)));
}
__device__ __forceinline__ void st_shared_u32(uint32_t addr, uint32_t v) {
    asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
__device__ __forceinline__ void st_shared_u16(uint32_t addr, uint16_t v) {
    asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}
// Shared-memory accessors of the CUDA-core variant (HKV_CUDA_CORES) only.
#if HKV_CUDA_CORES
__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_shared_f32x2(uint32_t addr, float a, float b) {
    asm volatile("st.shared.v2.f32 [%0], {%1,%2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void st_shared_f32x4(uint32_t addr, float4 v) {
    asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(v.x), "f"(v.y), "f"(v.z),
                 "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ float ld_shared_f32(uint32_t addr) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ float4 ld_shared_f32x4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ uint4 ld_shared_u32x4(uint32_t addr) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}
__device__ __forceinline__ uint2 ld_shared_u32x2(uint32_t addr) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr) : "memory");
    return v;
}
__device__ __forceinline__ float2 half2_bits_to_float2(uint32_t u) {
    return __half22float2(*reinterpret_cast<const __half2 *>(&u));
}
#endif
__device__ __forceinline__ void st_shared_zero16(uint32_t addr) {
    asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(addr), "r"(0) : "memory");
}

// ------------------------------------------------ thread-block cluster
// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_f32x4(uint32_t addr, float4 v) {
    asm volatile("st.shared::cluster.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "f"(v.x), "f"(v.y),
                 "f"(v.z), "f"(v.w)
                 : "memory");
}
__device__ __forceinline__ void st_cluster_f32x2(uint32_t addr, float a, float b) {
    asm volatile("st.shared::cluster.v2.f32 [%0], {%1,%2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void cluster_arrive() { asm volatile("barrier.cluster.arrive;" ::: "memory"); }
__device__ __forceinline__ void cluster_wait() { asm volatile("barrier.cluster.wait;" ::: "memory"); }
// Arrival on an mbarrier of another CTA of the cluster (release: this
// thread's earlier cluster stores are visible to whoever completes the wait).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint32_t bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(bar), "r"(parity)
        : "memory");
    return ok != 0;
}
// True when the phase with `parity` completed within the budget.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint32_t bar, uint32_t parity) {
    const long long t0 = clock64();
    while (!mbar_try_wait_cluster(bar, parity)) {
        if (clock64() - t0 > kWaitBudgetCycles) {
            return false;
        }
    }
    return true;
}

// NEOX rotation of one (x0, x1) pair with the reference's rounding: two
// separately rounded products, then a rounded difference / sum (ggml_mul,
// ggml_sub, ggml_add are separate graph nodes, src/higgs_pipeline.cpp:503-504).
__device__ __forceinline__ float rope_lo(float x0, float x1, float c, float s) {
    return __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
}
__device__ __forceinline__ float rope_hi(float x0, float x1, float c, float s) {
    return __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

__device__ __forceinline__ void load8(const float *p, float (&x)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4 *>(p));
    const float4 b = __ldg(reinterpret_cast<const float4 *>(p + 4));
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

// ===================================================================== append
// One warp per (row, KV head).  Lanes 0-15 write the sixteen 16-byte chunks
// of the K row, lanes 16-31 those of the V row.
template <bool kRope, bool kRange>
__global__ void __launch_bounds__(128) append_kernel(PoolView pool, RopeView rope, BatchView batch,
                                                     const int32_t *__restrict__ range_pages,
                                                     int64_t pos0, int64_t n_rows, int layer,
                                                     const float *__restrict__ k,
                                                     const float *__restrict__ v,
                                                     DeviceError *err) {
    const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    const int G = pool.n_head_kv;
    const int64_t row = warp / G;
    const int head = static_cast<int>(warp - row * G);
    if (row >= n_rows) {
        return;
    }
    int64_t pos;
    int64_t page;
    if (kRange) {
        pos = pos0 + row;
        page = range_pages[(pos >> 4) - (pos0 >> 4)];
    } else {
        pos = batch.pos[row];
        page = batch.pages[batch.page_off[row] + (pos >> 4)];
    }
    if (page < 0 || page >= pool.n_pages || pos < 0 || pos >= rope.context_length) {
        if (lane == 0) {
            record_error(err, kErrBadIndex, kWhereAppend, static_cast<int>(page),
                         static_cast<int>(pos));
        }
        return;
    }
    const int r = static_cast<int>(pos & 15);
    const bool is_v = lane >= 16;
    const int c = lane & 15;
    const float *src = (is_v ? v : k) + (row * G + head) * kHeadDim;
    float y[8];
    if (is_v || !kRope) {
        load8(src + c * 8, y);
    } else {
        const float *cr = rope.cos_tab + pos * (kHeadDim / 2);
        const float *sr = rope.sin_tab + pos * (kHeadDim / 2);
        const int i0 = (c & 7) * 8;  // index into the half
        float x0[8], x1[8], cs[8], sn[8];
        load8(src + i0, x0);
        load8(src + i0 + kHeadDim / 2, x1);
        load8(cr + i0, cs);
        load8(sr + i0, sn);
        if (c < 8) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                y[j] = rope_lo(x0[j], x1[j], cs[j], sn[j]);
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                y[j] = rope_hi(x0[j], x1[j], cs[j], sn[j]);
            }
        }
    }
    uint4 packed;
    packed.x = pack_half2(y[0], y[1]);
    packed.y = pack_half2(y[2], y[3]);
    packed.z = pack_half2(y[4], y[5]);
    packed.w = pack_half2(y[6], y[7]);
    uint8_t *dst = pool.base +
                   head_block_index(page, layer, is_v ? 1 : 0, head, pool.n_pages, G) *
                       kHeadBlockBytes +
                   r * kRowBytes + swizzled_chunk(r, c) * 16;
    *reinterpret_cast<uint4 *>(dst) = packed;
}

// ================================================================== attention
struct Cursor {
    int e;      // batch entry
    int h;      // KV head
    int i;      // page index within the slot
    int np;     // pages of entry e
    int pbase;  // page_off[e]
};

__device__ __forceinline__ void advance(const BatchView &b, int G, Cursor &c) {
    if (++c.i == c.np) {
        c.i = 0;
        if (++c.h == G) {
            c.h = 0;
            if (++c.e < b.n) {
                c.np = b.npages[c.e];
                c.pbase = b.page_off[c.e];
            }
        }
    }
}

__device__ __forceinline__ int64_t checked_page(const PoolView &pool, int64_t page, int e,
                                                DeviceError *err) {
    if (page < 0 || page >= pool.n_pages) {
        record_error(err, kErrBadIndex, kWhereAttn, static_cast<int>(page), e);
        return 0;  // keep every access in bounds; the result is flagged as invalid
    }
    return page;
}

__device__ __forceinline__ void issue_unit(const PoolView &pool, int layer, int64_t page, int h,
                                           uint32_t stage, uint32_t bar, uint64_t policy) {
    const uint8_t *kb =
        pool.base +
        head_block_index(page, layer, 0, h, pool.n_pages, pool.n_head_kv) * kHeadBlockBytes;
    const uint8_t *vb = kb + static_cast<int64_t>(pool.n_head_kv) * kHeadBlockBytes;
    mbar_arrive_expect_tx(bar, kStageBytes);
    bulk_load(stage, kb, kHeadBlockBytes, bar, policy);
    bulk_load(stage + kHeadBlockBytes, vb, kHeadBlockBytes, bar, policy);
}

// The new K/V row of one (slot, KV head): lanes 0-15 rope and convert the
// sixteen 8-dim chunks of K, lanes 16-31 convert those of V (same arithmetic
// as append_kernel).  Returns the lane's 16-byte chunk.
__device__ __forceinline__ uint4 new_row_chunk(const RopeView &rope, const float *k_row,
                                               const float *v_row, int pos, int lane) {
    const bool is_v = lane >= 16;
    const int c = lane & 15;
    float y[8];
    if (is_v) {
        load8(v_row + c * 8, y);
    } else {
        const float *cr = rope.cos_tab + static_cast<int64_t>(pos) * (kHeadDim / 2);
        const float *sr = rope.sin_tab + static_cast<int64_t>(pos) * (kHeadDim / 2);
        const int i0 = (c & 7) * 8;
        float x0[8], x1[8], cs[8], sn[8];
        load8(k_row + i0, x0);
        load8(k_row + i0 + kHeadDim / 2, x1);
        load8(cr + i0, cs);
        load8(sr + i0, sn);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            y[j] = c < 8 ? rope_lo(x0[j], x1[j], cs[j], sn[j]) : rope_hi(x0[j], x1[j], cs[j], sn[j]);
        }
    }
    uint4 packed;
    packed.x = pack_half2(y[0], y[1]);
    packed.y = pack_half2(y[2], y[3]);
    packed.z = pack_half2(y[4], y[5]);
    packed.w = pack_half2(y[6], y[7]);
    return packed;
}

// Merge of one (slot, KV head)'s partials by the warp that finished last.
// Partials were written by other SMs in this launch: read them through L2.
// Lane p holds the (m, l) of partial p (loaded in parallel, reduced by
// shuffles); the partial outputs are then streamed with the weights
// broadcast from their owner lane, several partials in flight at a time.
// Result of a merge before normalisation: o = sum_p w_p o_p, l = sum_p w_p l_p
// with w_p = 2^(m_p - m); the final output is o / l, a group partial keeps
// (o, m, l) as is.
struct Merged {
    float4 o[kGqa];  // this lane's 4 dims of each head
    float m[kGqa];
    float l[kGqa];
};

__device__ __forceinline__ void merge_partials(const float *part_o, const float *part_ml, int p0,
                                               int nparts, int lane, Merged &res) {
    float mx[kGqa];
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
        mx[j] = -INFINITY;
    }
    for (int p = lane; p < nparts; p += 32) {
        const float4 *pm = reinterpret_cast<const float4 *>(part_ml + static_cast<int64_t>(p0 + p) * (2 * kGqa));
        const float4 a = __ldcg(pm);
        const float4 b = __ldcg(pm + 1);
        mx[0] = fmaxf(mx[0], a.x);
        mx[1] = fmaxf(mx[1], a.z);
        mx[2] = fmaxf(mx[2], b.x);
        mx[3] = fmaxf(mx[3], b.z);
    }
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], off));
        }
    }
    float4 acc[kGqa];
    float den[kGqa];
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
        acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        den[j] = 0.f;
    }
    for (int base = 0; base < nparts; base += 32) {
        // weights of the partials base .. base+31, one per lane
        float w[kGqa] = {0.f, 0.f, 0.f, 0.f};
        if (base + lane < nparts) {
            const float4 *pm = reinterpret_cast<const float4 *>(
                part_ml + static_cast<int64_t>(p0 + base + lane) * (2 * kGqa));
            const float4 a = __ldcg(pm);
            const float4 b = __ldcg(pm + 1);
            w[0] = exp2f(a.x - mx[0]);
            w[1] = exp2f(a.z - mx[1]);
            w[2] = exp2f(b.x - mx[2]);
            w[3] = exp2f(b.z - mx[3]);
            den[0] += w[0] * a.y;
            den[1] += w[1] * a.w;
            den[2] += w[2] * b.y;
            den[3] += w[3] * b.w;
        }
        const int cnt = min(32, nparts - base);
#pragma unroll 4
        for (int t = 0; t < cnt; ++t) {
            const float4 *po = reinterpret_cast<const float4 *>(
                part_o + static_cast<int64_t>(p0 + base + t) * (kGqa * kHeadDim));
#pragma unroll
            for (int j = 0; j < kGqa; ++j) {
                const float wt = __shfl_sync(0xffffffffu, w[j], t);
                const float4 ov = __ldcg(po + j * (kHeadDim / 4) + lane);
                acc[j].x += wt * ov.x;
                acc[j].y += wt * ov.y;
                acc[j].z += wt * ov.z;
                acc[j].w += wt * ov.w;
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            den[j] += __shfl_xor_sync(0xffffffffu, den[j], off);
        }
    }
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
        res.o[j] = acc[j];
        res.m[j] = mx[j];
        res.l[j] = den[j];
    }
}

// The same merge with every load of kBatch partials issued before their
// weighted sums (a merge is a chain of L2 round trips, so the batch size sets
// its latency); the sums are taken in the same partial order.  The first
// batch of outputs goes out with the (m, l) loads, since the outputs do not
// depend on the weights.  Used for the merges of a warp's last segment, after
// its main loop, where the registers of the loop are free.
__device__ __forceinline__ void merge_partials_wide(const float *part_o, const float *part_ml, int p0,
                                               int nparts, int lane, Merged &res) {
    constexpr int kBatch = 8;  // partial outputs in flight per lane
    float4 ov[kBatch][kGqa];
    auto load_batch = [&](int t0) {
#pragma unroll
        for (int t = 0; t < kBatch; ++t) {
            if (t0 + t < nparts) {
                const float4 *po = reinterpret_cast<const float4 *>(
                    part_o + static_cast<int64_t>(p0 + t0 + t) * (kGqa * kHeadDim));
#pragma unroll
                for (int j = 0; j < kGqa; ++j) {
                    ov[t][j] = __ldcg(po + j * (kHeadDim / 4) + lane);
                }
            }
        }
    };
    load_batch(0);
    float mx[kGqa];
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
        mx[j] = -INFINITY;
    }
    // (m, l) of partial lane (kept for the weights: at most 32 partials are
    // merged at once in practice; more take another pass)
    float4 ml_a = make_float4(-INFINITY, 0.f, -INFINITY, 0.f), ml_b = ml_a;
    for (int p = lane; p < nparts; p += 32) {
        const float4 *pm = reinterpret_cast<const float4 *>(part_ml + static_cast<int64_t>(p0 + p) * (2 * kGqa));
        const float4 a = __ldcg(pm);
        const float4 b = __ldcg(pm + 1);
        if (p == lane) {
            ml_a = a;
            ml_b = b;
        }
        mx[0] = fmaxf(mx[0], a.x);
        mx[1] = fmaxf(mx[1], a.z);
        mx[2] = fmaxf(mx[2], b.x);
        mx[3] = fmaxf(mx[3], b.z);
    }
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            mx[j] = fmaxf(mx[j], __shfl_xor_sync(0xffffffffu, mx[j], off));
        }
    }
    float4 acc[kGqa];
    float den[kGqa];
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
        acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        den[j] = 0.f;
    }
    for (int base = 0; base < nparts; base += 32) {
        // weights of the partials base .. base+31, one per lane
        float w[kGqa] = {0.f, 0.f, 0.f, 0.f};
        if (base + lane < nparts) {
            float4 a = ml_a, b = ml_b;
            if (base > 0) {
                const float4 *pm = reinterpret_cast<const float4 *>(
                    part_ml + static_cast<int64_t>(p0 + base + lane) * (2 * kGqa));
                a = __ldcg(pm);
                b = __ldcg(pm + 1);
            }
            w[0] = exp2f(a.x - mx[0]);
            w[1] = exp2f(a.z - mx[1]);
            w[2] = exp2f(b.x - mx[2]);
            w[3] = exp2f(b.z - mx[3]);
            den[0] += w[0] * a.y;
            den[1] += w[1] * a.w;
            den[2] += w[2] * b.y;
            den[3] += w[3] * b.w;
        }
        const int cnt = min(32, nparts - base);
        for (int t0 = 0; t0 < cnt; t0 += kBatch) {
            // all loads of the batch first (the first batch is in flight
            // already), then the weighted sums in order
            if (base + t0 > 0) {
                load_batch(base + t0);
            }
#pragma unroll
            for (int t = 0; t < kBatch; ++t) {
                if (t0 + t < cnt) {
#pragma unroll
                    for (int j = 0; j < kGqa; ++j) {
                        const float wt = __shfl_sync(0xffffffffu, w[j], t0 + t);
                        acc[j].x += wt * ov[t][j].x;
                        acc[j].y += wt * ov[t][j].y;
                        acc[j].z += wt * ov[t][j].z;
                        acc[j].w += wt * ov[t][j].w;
                    }
                }
            }
        }
    }
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            den[j] += __shfl_xor_sync(0xffffffffu, den[j], off);
        }
    }
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
        res.o[j] = acc[j];
        res.m[j] = mx[j];
        res.l[j] = den[j];
    }
}

// Merge of m partials in shared memory, partial k at base(k), in order k.
template <class Base>
__device__ __forceinline__ void merge_smem_partials(Base base, int m, int lane, Merged &res) {
    float mx[kGqa];
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
        mx[j] = -INFINITY;
    }
    for (int k = 0; k < m; ++k) {
        const float *ml = base(k) + kGqa * kHeadDim;
#pragma unroll
        for (int j = 0; j < kGqa; ++j) {
            mx[j] = fmaxf(mx[j], ml[2 * j]);
        }
    }
#pragma unroll
    for (int j = 0; j < kGqa; ++j) {
        res.o[j] = make_float4(0.f, 0.f, 0.f, 0.f);
        res.l[j] = 0.f;
        res.m[j] = mx[j];
    }
    for (int k = 0; k < m; ++k) {
        const float *pk = base(k);
        const float *ml = pk + kGqa * kHeadDim;
#pragma unroll
        for (int j = 0; j < kGqa; ++j) {
            const float w = exp2f(ml[2 * j] - mx[j]);
            res.l[j] += w * ml[2 * j + 1];
            const float4 ov = reinterpret_cast<const float4 *>(pk + j * kHeadDim)[lane];
            res.o[j].x += w * ov.x;
            res.o[j].y += w * ov.y;
            res.o[j].z += w * ov.z;
            res.o[j].w += w * ov.w;
        }
    }
}

// The m partials a run of warps left in its CTA's slots (slot of warp k: 1
// for the run's first warp, 0 for the others), in warp order.
__device__ __forceinline__ void merge_cta(const float *slots, int w0, int m, int lane, Merged &res) {
    merge_smem_partials([&](int k) { return slots + (2 * (w0 + k) + (k == 0 ? 1 : 0)) * kCtaPartFloats; },
                        m, lane, res);
}

// The C CTA partials of a cluster, slot k from the CTA of rank k, in rank order.
__device__ __forceinline__ void merge_cluster(const float *slots, int m, int lane, Merged &res) {
    merge_smem_partials([&](int k) { return slots + k * kCtaPartFloats; }, m, lane, res);
}

__device__ __forceinline__ float4 normalised(const Merged &r, int j) {
    const float inv = 1.f / r.l[j];
    return make_float4(r.o[j].x * inv, r.o[j].y * inv, r.o[j].z * inv, r.o[j].w * inv);
}

// Destination of the 4 x 128 output floats of (entry e, KV head h).
__device__ __forceinline__ float *out_slice(float *out, const Exchange &x, int r, int layer, int e,
                                            int h, int G) {
    if (x.n_ranks == 0) {
        return out + (static_cast<int64_t>(e) * (kGqa * G) + kGqa * h) * kHeadDim;
    }
    return x.outs[r] + layer * x.layer_floats + static_cast<int64_t>(e) * x.row_floats + x.col_off +
           kGqa * h * kHeadDim;
}

// After a warp has stored a finished slice everywhere: the warp barrier
// orders every lane's stores before lane 0, whose system-scope release fence
// (cumulative) orders them before its arrival counts; the counts are
// fire-and-forget reductions, one per rank, so the warp does not wait for
// their round trips.
__device__ __forceinline__ void signal_arrival(const Exchange &x, int layer, int lane) {
    if (x.n_ranks == 0) {
        return;
    }
    __syncwarp();
    if (lane == 0) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int r = 0; r < x.n_ranks; ++r) {
            asm volatile("red.relaxed.sys.global.add.u32 [%0], 1;" ::"l"(x.flags[r] + layer) : "memory");
        }
    }
}

// kCluster (with kCtaMerge): the launch is in clusters of batch.cluster CTAs,
// one (slot, KV head) segment per cluster (plan_cluster).
template <bool kAppend, bool kCtaMerge, bool kCluster>
__global__ void __launch_bounds__(kAttnWarps * 32, 1)
    attention_kernel(PoolView pool, RopeView rope, BatchView batch, int layer,
                     const float *__restrict__ q, const float *__restrict__ k_new,
                     const float *__restrict__ v_new, float *__restrict__ part_o,
                     float *__restrict__ part_ml, int32_t *__restrict__ counters,
                     float *__restrict__ out, Exchange xchg, float scale_log2, DeviceError *err) {
    extern __shared__ __align__(1024) uint8_t smem[];
    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    const int gw = blockIdx.x * kAttnWarps + wid;
    const int G = pool.n_head_kv;
    const int W = batch.n_warps;
    static_assert(kCtaMerge || !kCluster, "the cluster merge starts from the CTA merge");
    float *cta_slots = reinterpret_cast<float *>(smem + kAttnWarps * kWarpSmem);
    int *run_ticket = reinterpret_cast<int *>(smem + kAttnWarps * kWarpSmem + kAttnWarps * 2 * kCtaPartBytes);
    float *cl_slots = reinterpret_cast<float *>(smem + kAttnWarps * kWarpSmem + kCtaSmem);
    const uint32_t cl_bar = smem_u32(smem + kAttnWarps * kWarpSmem + kCtaSmem + kMaxCluster * kCtaPartBytes);
    if (kCtaMerge) {
        if (threadIdx.x < kAttnWarps) {
            run_ticket[threadIdx.x] = 0;
        }
        if (kCluster && threadIdx.x == 0) {
            mbar_init(cl_bar, static_cast<uint32_t>(batch.cluster));  // used in the first CTA
            fence_barrier_init();
        }
        __syncthreads();  // the only CTA barrier: before any warp can leave
        if (kCluster) {
            // Every thread arrives before it can leave; a CTA's last warp waits
            // (barrier.cluster.wait) before its first store into another CTA,
            // so that CTA's barrier is initialised by then.
            cluster_arrive();
        }
    }
    if (gw >= W) {
        return;
    }
    // The plan hands each warp its share, its starting cursor and the
    // physical pages of its first units in three 16-byte records, so the
    // first copies go out without a chain of dependent loads.
    const int4 ws0 = batch.warp_start[3 * gw];
    const int4 ws1 = batch.warp_start[3 * gw + 1];
    const int4 ws2 = batch.warp_start[3 * gw + 2];
    const int u_begin = ws2.x;
    const int u_end = ws2.y;
    if (u_begin >= u_end) {
        return;
    }
    const uint32_t stage0 = smem_u32(smem + wid * kWarpSmem);
    const uint32_t qc = stage0 + kAttnStages * kStageBytes;
    const uint32_t pbuf = qc + kQcBytes;
    const uint32_t bar0 = pbuf + kPBufBytes;
    const uint64_t policy = evict_first_policy();

    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < kAttnStages; ++s) {
            mbar_init(bar0 + 8 * s, 1);
        }
        fence_barrier_init();
    }
    __syncwarp();

    Cursor cons;
    cons.e = ws0.x;
    cons.h = ws0.y;
    cons.i = ws0.z;
    cons.np = ws0.w;
    cons.pbase = ws1.x;
    // Producer (lane 0): issue the first stages, then keep the page id of the
    // next unit to issue already loaded, one iteration ahead of its use.
    Cursor prod = cons;
    int64_t next_page = 0;
    if (lane == 0) {
        const int first_pages[3] = {ws1.y, ws1.z, ws1.w};
#pragma unroll
        for (int s = 0; s < kAttnStages; ++s) {
            if (u_begin + s < u_end) {
                const int64_t page = checked_page(
                    pool, s < 3 ? first_pages[s] : batch.pages[prod.pbase + prod.i], prod.e, err);
                issue_unit(pool, layer, page, prod.h, stage0 + s * kStageBytes, bar0 + 8 * s, policy);
                advance(batch, G, prod);
            }
        }
        if (u_begin + kAttnStages < u_end) {
            next_page = batch.pages[prod.pbase + prod.i];
        }
    }

    // Programmatic dependent launch: everything above only reads this launch's
    // plan and this layer's pages; q / k / v may come from the kernel before,
    // and the partials, counters and outputs may still be in use by it, so
    // wait for it here (a no-op when launched without the attribute).
    asm volatile("griddepcontrol.wait;" ::: "memory");

    const int r7 = lane & 7;
    const int mi = lane >> 3;
    // Per-lane byte offsets inside a head block for the ldmatrix row addresses.
    const int k_row_off = (r7 + ((mi & 1) << 3)) * kRowBytes;
    const int v_row_off = (r7 + ((mi >> 1) << 3)) * kRowBytes;
    const int k_chunk_hi = mi >> 1;
    const int v_chunk_hi = mi & 1;
    const bool lo_side = (lane & 2) != 0;  // columns 4-7: F16 residual parts
    const float kNegInf = -INFINITY;

    float o[8][4];
    uint32_t qb[8][2];
#if HKV_CUDA_CORES
    // CUDA-core variant: this lane's 4 dims (4 lane .. 4 lane + 3) of each of
    // the 4 query heads, over all tokens of the segment so far
    float4 acc[kGqa];
#endif
    float m_a = kNegInf, m_b = kNegInf, l_a = 0.f, l_b = 0.f;
    int seg_e = 0, seg_h = 0, seg_pos = 0, part = 0, p_first = 0, nparts = 1, ntok = 0;
    int run_w0 = wid, run_m = 1;  // this CTA's warps of the current segment: w0 .. w0 + m - 1

    auto flush = [&](bool after_loop) {
#if HKV_CUDA_CORES
        // Lay the CUDA-core accumulators out as the tensor-core fragments the
        // rest of the flush reads (the staged q is no longer needed: its area
        // holds them; lanes of the F16-residual columns get zeros).
        __syncwarp();
#pragma unroll
        for (int j = 0; j < kGqa; ++j) {
            st_shared_f32x4(qc + (j * kHeadDim + 4 * lane) * 4, acc[j]);
        }
        __syncwarp();
        {
            const int ha = (lane & 1) * 2;
            const int g = lane >> 2;
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                o[mt][0] = lo_side ? 0.f : ld_shared_f32(qc + (ha * kHeadDim + 16 * mt + g) * 4);
                o[mt][1] = lo_side ? 0.f : ld_shared_f32(qc + ((ha + 1) * kHeadDim + 16 * mt + g) * 4);
                o[mt][2] = lo_side ? 0.f : ld_shared_f32(qc + (ha * kHeadDim + 16 * mt + g + 8) * 4);
                o[mt][3] = lo_side ? 0.f : ld_shared_f32(qc + ((ha + 1) * kHeadDim + 16 * mt + g + 8) * 4);
            }
        }
        __syncwarp();
#endif
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                o[mt][j] += __shfl_xor_sync(0xffffffffu, o[mt][j], 2);
            }
        }
        l_a += __shfl_xor_sync(0xffffffffu, l_a, 4);
        l_a += __shfl_xor_sync(0xffffffffu, l_a, 8);
        l_a += __shfl_xor_sync(0xffffffffu, l_a, 16);
        l_b += __shfl_xor_sync(0xffffffffu, l_b, 4);
        l_b += __shfl_xor_sync(0xffffffffu, l_b, 8);
        l_b += __shfl_xor_sync(0xffffffffu, l_b, 16);
        const int ha = (lane & 1) * 2;
        const int d0 = lane >> 2;
        const int n_dst = xchg.n_ranks == 0 ? 1 : xchg.n_ranks;
        if (nparts == 1 && run_m == 1) {
            // The whole (slot, KV head) was this warp's: write the output.
            if (!lo_side) {
                const float ia = 1.f / l_a;
                const float ib = 1.f / l_b;
                for (int r = 0; r < n_dst; ++r) {
                    float *ob = out_slice(out, xchg, r, layer, seg_e, seg_h, G);
#pragma unroll
                    for (int mt = 0; mt < 8; ++mt) {
                        ob[ha * kHeadDim + 16 * mt + d0] = o[mt][0] * ia;
                        ob[(ha + 1) * kHeadDim + 16 * mt + d0] = o[mt][1] * ib;
                        ob[ha * kHeadDim + 16 * mt + d0 + 8] = o[mt][2] * ia;
                        ob[(ha + 1) * kHeadDim + 16 * mt + d0 + 8] = o[mt][3] * ib;
                    }
                }
            }
            signal_arrival(xchg, layer, lane);
            return;
        }
        // This warp's (o, m, l): into its shared-memory slot when other warps
        // of the CTA share the segment, else straight to the global partial.
        float *po;
        float *pm;
        if (run_m > 1) {
            po = cta_slots + (2 * wid + (wid == run_w0 ? 1 : 0)) * kCtaPartFloats;
            pm = po + kGqa * kHeadDim;
        } else {
            po = part_o + static_cast<int64_t>(part) * (kGqa * kHeadDim);
            pm = part_ml + static_cast<int64_t>(part) * (2 * kGqa);
        }
        if (!lo_side) {
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
                po[ha * kHeadDim + 16 * mt + d0] = o[mt][0];
                po[(ha + 1) * kHeadDim + 16 * mt + d0] = o[mt][1];
                po[ha * kHeadDim + 16 * mt + d0 + 8] = o[mt][2];
                po[(ha + 1) * kHeadDim + 16 * mt + d0 + 8] = o[mt][3];
            }
            if (d0 == 0) {
                pm[ha * 2] = m_a;
                pm[ha * 2 + 1] = l_a;
                pm[ha * 2 + 2] = m_b;
                pm[ha * 2 + 3] = l_b;
            }
        }
        const int eh = seg_e * G + seg_h;
        if (run_m > 1) {
            __threadfence_block();
            __syncwarp();
            int rt = 0;
            if (lane == 0) {
                rt = atomicAdd(run_ticket + run_w0, 1);
            }
            rt = __shfl_sync(0xffffffffu, rt, 0);
            if (rt != run_m - 1) {
                return;  // another warp of the run merges
            }
            __threadfence_block();
            Merged cres;
            merge_cta(cta_slots, run_w0, run_m, lane, cres);
            if (nparts == 1) {
                // the whole segment lived in this CTA: the output
                for (int r = 0; r < n_dst; ++r) {
                    float4 *ob = reinterpret_cast<float4 *>(out_slice(out, xchg, r, layer, seg_e, seg_h, G));
#pragma unroll
                    for (int j = 0; j < kGqa; ++j) {
                        ob[j * (kHeadDim / 4) + lane] = normalised(cres, j);
                    }
                }
                signal_arrival(xchg, layer, lane);
                return;
            }
            if (kCluster) {
                // The CTA's partial goes to slot `rank` in the cluster's first
                // CTA, whose last warp merges the slots in rank order once all
                // have arrived on its barrier, and writes the output.
                const int rank = part - p_first;  // = the CTA's rank in its cluster
                cluster_wait();
                const uint32_t slot = cluster_map(smem_u32(cl_slots + rank * kCtaPartFloats), 0);
#pragma unroll
                for (int j = 0; j < kGqa; ++j) {
                    st_cluster_f32x4(slot + (j * kHeadDim + 4 * lane) * 4, cres.o[j]);
                }
                if (lane == 0) {
#pragma unroll
                    for (int j = 0; j < kGqa; ++j) {
                        st_cluster_f32x2(slot + (kGqa * kHeadDim + 2 * j) * 4, cres.m[j], cres.l[j]);
                    }
                }
                __syncwarp();
                if (lane == 0) {
                    asm volatile("fence.acq_rel.cluster;" ::: "memory");
                    mbar_arrive_remote(cluster_map(cl_bar, 0));
                }
                if (rank != 0) {
                    return;
                }
                if (!__all_sync(0xffffffffu, mbar_wait_cluster_bounded(cl_bar, 0))) {
                    if (lane == 0) {
                        record_error(err, kErrTimeout, kWhereAttn, seg_h, blockIdx.x);
                    }
                    return;
                }
                Merged res;
                merge_cluster(cl_slots, nparts, lane, res);
                for (int r = 0; r < n_dst; ++r) {
                    float4 *ob = reinterpret_cast<float4 *>(out_slice(out, xchg, r, layer, seg_e, seg_h, G));
#pragma unroll
                    for (int j = 0; j < kGqa; ++j) {
                        ob[j * (kHeadDim / 4) + lane] = normalised(res, j);
                    }
                }
                signal_arrival(xchg, layer, lane);
                return;
            }
            // the CTA's partial of the segment
            float4 *gpo = reinterpret_cast<float4 *>(part_o + static_cast<int64_t>(part) * (kGqa * kHeadDim));
#pragma unroll
            for (int j = 0; j < kGqa; ++j) {
                gpo[j * (kHeadDim / 4) + lane] = cres.o[j];
            }
            if (lane == 0) {
                float *gpm = part_ml + static_cast<int64_t>(part) * (2 * kGqa);
#pragma unroll
                for (int j = 0; j < kGqa; ++j) {
                    gpm[2 * j] = cres.m[j];
                    gpm[2 * j + 1] = cres.l[j];
                }
            }
        }
        if (batch.combine) {
            // The combine launch that follows merges the stored partials once
            // this grid has completed: no fence or ticket here.
            return;
        }
        // Publish the partial; the last of a group of partials merges the
        // group, and the last group (or the only one) produces the output.
        const int n_groups = merge_groups(nparts);
        if (n_groups != 0) __threadfence();
        __syncwarp();
        const int j_part = part - p_first;
        const int n_seg = batch.n * G;  // segment counters come first, then group counters
        auto finish = [&](const Merged &res) {
            for (int r = 0; r < n_dst; ++r) {
                float4 *ob = reinterpret_cast<float4 *>(out_slice(out, xchg, r, layer, seg_e, seg_h, G));
#pragma unroll
                for (int j = 0; j < kGqa; ++j) {
                    ob[j * (kHeadDim / 4) + lane] = normalised(res, j);
                }
            }
            if (lane == 0) {
                counters[eh] = 0;  // ready for the next launch
            }
            signal_arrival(xchg, layer, lane);
        };
        if (n_groups == 0) {
            // One acquire-release ticket instead of a fence on either side of
            // a relaxed one: its release publishes the whole warp's partial
            // (the lanes' stores are ordered before it by the warp barrier
            // above), and for the last warp its acquire orders the merge's
            // loads (after the barrier below) after every other warp's
            // release.  16 slots of 256-4096 positions +1.2%.
            int ticket = 0;
            if (lane == 0) {
                asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], 1;"
                             : "=r"(ticket)
                             : "l"(counters + eh)
                             : "memory");
            }
            ticket = __shfl_sync(0xffffffffu, ticket, 0);
            __syncwarp();
            if (ticket == nparts - 1) {
                Merged res;
                if (after_loop) {
                    merge_partials_wide(part_o, part_ml, p_first, nparts, lane, res);
                } else {
                    merge_partials(part_o, part_ml, p_first, nparts, lane, res);
                }
                finish(res);
            }
            return;
        }
        const int gsz = merge_group_size(nparts);
        const int g = j_part / gsz;
        const int g_size = min(gsz, nparts - g * gsz);
        const int g_index = batch.part2_off[eh] + g;
        int ticket = 0;
        if (lane == 0) {
            ticket = atomicAdd(counters + n_seg + g_index, 1);
        }
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket != g_size - 1) {
            return;
        }
        __threadfence();
        Merged grp;
        if (after_loop) {
            merge_partials_wide(part_o, part_ml, p_first + g * gsz, g_size, lane, grp);
        } else {
            merge_partials(part_o, part_ml, p_first + g * gsz, g_size, lane, grp);
        }
        {
            // the group partial, stored after the level-1 partials
            const int gp = batch.n_parts + g_index;
            float4 *po = reinterpret_cast<float4 *>(part_o + static_cast<int64_t>(gp) * (kGqa * kHeadDim));
#pragma unroll
            for (int j = 0; j < kGqa; ++j) {
                po[j * (kHeadDim / 4) + lane] = grp.o[j];
            }
            if (lane == 0) {
                float *pm = part_ml + static_cast<int64_t>(gp) * (2 * kGqa);
#pragma unroll
                for (int j = 0; j < kGqa; ++j) {
                    pm[2 * j] = grp.m[j];
                    pm[2 * j + 1] = grp.l[j];
                }
                counters[n_seg + g_index] = 0;
            }
        }
        __threadfence();
        __syncwarp();
        if (lane == 0) {
            ticket = atomicAdd(counters + eh, 1);
        }
        ticket = __shfl_sync(0xffffffffu, ticket, 0);
        if (ticket == n_groups - 1) {
            __threadfence();
            Merged res;
            if (after_loop) {
                merge_partials_wide(part_o, part_ml, batch.n_parts + batch.part2_off[eh], n_groups, lane, res);
            } else {
                merge_partials(part_o, part_ml, batch.n_parts + batch.part2_off[eh], n_groups, lane, res);
            }
            finish(res);
        }
    };

    for (int u = u_begin, k = 0; u < u_end; ++u, ++k) {
        const int s = k % kAttnStages;
        const uint32_t parity = static_cast<uint32_t>(k / kAttnStages) & 1u;
        if (u == u_begin || cons.i == 0) {
            if (u != u_begin) {
                flush(false);
            }
            // ---- new (entry, KV head) share: stage RoPE'd q as F16 hi/lo rows
            seg_e = cons.e;
            seg_h = cons.h;
            seg_pos = batch.pos[seg_e];
            ntok = seg_pos + 1;
            {
                // {first partial, partials, first warp, last warp} of the segment
                const int4 sg = batch.seg[seg_e * G + seg_h];
                p_first = sg.x;
                nparts = sg.y;
                if (kCtaMerge) {
                    // partials are per CTA: the warps of one CTA that share
                    // the segment merge theirs in shared memory first
                    const int cta = static_cast<int>(blockIdx.x);
                    part = sg.x + (cta - sg.z / kAttnWarps);
                    const int run_lo = max(sg.z, cta * kAttnWarps);
                    const int run_hi = min(sg.w, cta * kAttnWarps + kAttnWarps - 1);
                    run_w0 = run_lo - cta * kAttnWarps;
                    run_m = run_hi - run_lo + 1;
                } else {
                    part = sg.x + (gw - sg.z);
                    run_m = 1;
                }
            }
            const float *cr = rope.cos_tab + static_cast<int64_t>(seg_pos) * (kHeadDim / 2);
            const float *sr = rope.sin_tab + static_cast<int64_t>(seg_pos) * (kHeadDim / 2);
            const float *qe = q + (static_cast<int64_t>(seg_e) * (kGqa * G) + kGqa * seg_h) * kHeadDim;
#pragma unroll
            for (int half = 0; half < 2; ++half) {
                const int i = lane + 32 * half;
                const float c = __ldg(cr + i);
                const float sn = __ldg(sr + i);
#pragma unroll
                for (int j = 0; j < kGqa; ++j) {
                    const float x0 = __ldg(qe + j * kHeadDim + i);
                    const float x1 = __ldg(qe + j * kHeadDim + i + kHeadDim / 2);
                    const float y0 = rope_lo(x0, x1, c, sn);
                    const float y1 = rope_hi(x0, x1, c, sn);
#if HKV_CUDA_CORES
                    st_shared_f32(qc + (j * kHeadDim + i) * 4, y0);
                    st_shared_f32(qc + (j * kHeadDim + i + 64) * 4, y1);
                    continue;
#endif
                    const __half h0 = __float2half_rn(y0);
                    const __half h1 = __float2half_rn(y1);
                    const __half l0 = __float2half_rn(__fsub_rn(y0, __half2float(h0)));
                    const __half l1 = __float2half_rn(__fsub_rn(y1, __half2float(h1)));
                    st_shared_u16(qc + (j * kQcStride + i) * 2, __half_as_ushort(h0));
                    st_shared_u16(qc + (j * kQcStride + i + 64) * 2, __half_as_ushort(h1));
                    st_shared_u16(qc + ((j + 4) * kQcStride + i) * 2, __half_as_ushort(l0));
                    st_shared_u16(qc + ((j + 4) * kQcStride + i + 64) * 2, __half_as_ushort(l1));
                }
            }
            __syncwarp();
#if HKV_CUDA_CORES
#pragma unroll
            for (int j = 0; j < kGqa; ++j) {
                acc[j] = make_float4(0.f, 0.f, 0.f, 0.f);
            }
#else
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                ldsm_x4(qc + (r7 * kQcStride + jj * 32 + mi * 8) * 2, qb[2 * jj][0],
                        qb[2 * jj][1], qb[2 * jj + 1][0], qb[2 * jj + 1][1]);
            }
#endif
#pragma unroll
            for (int mt = 0; mt < 8; ++mt) {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    o[mt][j] = 0.f;
                }
            }
            m_a = m_b = kNegInf;
            l_a = l_b = 0.f;
        }

        // ---- wait for this unit's K and V head blocks
        const uint32_t bar = bar0 + 8 * s;
        const bool ok = __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity));
        if (!ok) {
            if (lane == 0) {
                record_error(err, kErrTimeout, kWhereAttn, u, blockIdx.x);
            }
            // Drain the copies this warp still has in flight, then leave.
            for (int j = 1; j < kAttnStages && u + j < u_end; ++j) {
                const int kk = k + j;
                mbar_wait_bounded(bar0 + 8 * (kk % kAttnStages),
                                  static_cast<uint32_t>(kk / kAttnStages) & 1u);
            }
            return;
        }
        const uint32_t kt = stage0 + s * kStageBytes;
        const uint32_t vt = kt + kHeadBlockBytes;
        const int row0 = cons.i * kPageTokens;
        const int valid = min(kPageTokens, ntok - row0);
        if (valid < kPageTokens) {
            // Rows past the slot's length hold whatever the page had before;
            // zero them in shared memory so 0 * garbage cannot poison PV.
            for (int idx = lane; idx < (kPageTokens - valid) * 16; idx += 32) {
                st_shared_zero16(vt + (valid + (idx >> 4)) * kRowBytes + (idx & 15) * 16);
            }
        }
        if (kAppend && cons.i == cons.np - 1) {
            // Fused append: this warp owns the slot's last page for this KV
            // head, so it writes the new row to HBM and into its copy of the
            // page (the copy arrived without it).
            const int r = seg_pos & 15;
            const int c = lane & 15;
            const bool is_v = lane >= 16;
            const int64_t row_base = (static_cast<int64_t>(seg_e) * G + seg_h) * kHeadDim;
            const uint4 chunk = new_row_chunk(rope, k_new + row_base, v_new + row_base, seg_pos, lane);
            const int64_t page = checked_page(pool, batch.pages[cons.pbase + cons.i], seg_e, err);
            uint8_t *dst = pool.base +
                           head_block_index(page, layer, is_v ? 1 : 0, seg_h, pool.n_pages, G) *
                               kHeadBlockBytes +
                           r * kRowBytes + swizzled_chunk(r, c) * 16;
            *reinterpret_cast<uint4 *>(dst) = chunk;
            const uint32_t sdst = (is_v ? vt : kt) + r * kRowBytes + swizzled_chunk(r, c) * 16;
            asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(sdst), "r"(chunk.x),
                         "r"(chunk.y), "r"(chunk.z), "r"(chunk.w)
                         : "memory");
        }
        if (valid < kPageTokens || (kAppend && cons.i == cons.np - 1)) {
            fence_proxy_async_smem();
            __syncwarp();
        }

#if HKV_CUDA_CORES
        // ---- CUDA cores: this lane's partial scores of tokens g and g + 8 for
        // heads ha, ha + 1 over its half of the dims (the lanes of the other
        // half hold the rest; the shuffle below adds them), F16 K converted
        // exactly, F32 products.  Lanes of the upper half walk their chunks
        // rotated by four so a load phase hits eight bank groups.
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
        float sd[4] = {0.f, 0.f, 0.f, 0.f};
        {
            const int hsel = (lane >> 1) & 1;
            const int ha = (lane & 1) * 2;
            const int g = lane >> 2;
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const int c = hsel * 8 + ((i + 4 * hsel) & 7);
                const uint4 k0 = ld_shared_u32x4(kt + g * kRowBytes + ((c ^ g) << 4));
                const uint4 k1 = ld_shared_u32x4(kt + (g + 8) * kRowBytes + ((c ^ g) << 4));
                const float4 qa0 = ld_shared_f32x4(qc + (ha * kHeadDim + c * 8) * 4);
                const float4 qa1 = ld_shared_f32x4(qc + (ha * kHeadDim + c * 8 + 4) * 4);
                const float4 qb0 = ld_shared_f32x4(qc + ((ha + 1) * kHeadDim + c * 8) * 4);
                const float4 qb1 = ld_shared_f32x4(qc + ((ha + 1) * kHeadDim + c * 8 + 4) * 4);
                const float qa[8] = {qa0.x, qa0.y, qa0.z, qa0.w, qa1.x, qa1.y, qa1.z, qa1.w};
                const float qbv[8] = {qb0.x, qb0.y, qb0.z, qb0.w, qb1.x, qb1.y, qb1.z, qb1.w};
                const uint32_t kw0[4] = {k0.x, k0.y, k0.z, k0.w};
                const uint32_t kw1[4] = {k1.x, k1.y, k1.z, k1.w};
                float *acc_s = (i & 1) ? sd : sc;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f0 = half2_bits_to_float2(kw0[e]);
                    const float2 f1 = half2_bits_to_float2(kw1[e]);
                    acc_s[0] = fmaf(f0.x, qa[2 * e], fmaf(f0.y, qa[2 * e + 1], acc_s[0]));
                    acc_s[1] = fmaf(f0.x, qbv[2 * e], fmaf(f0.y, qbv[2 * e + 1], acc_s[1]));
                    acc_s[2] = fmaf(f1.x, qa[2 * e], fmaf(f1.y, qa[2 * e + 1], acc_s[2]));
                    acc_s[3] = fmaf(f1.x, qbv[2 * e], fmaf(f1.y, qbv[2 * e + 1], acc_s[3]));
                }
            }
        }
#else
        // ---- S^T[token][col] = K[token][:] . Qc[col][:]   (col 0-3 hi, 4-7 lo)
        // Two accumulators (even / odd k-steps) halve the dependent mma chain.
        float sc[4] = {0.f, 0.f, 0.f, 0.f};
        float sd[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int ks = 0; ks < 8; ks += 2) {
            uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
            ldsm_x4(kt + k_row_off + (((2 * ks + k_chunk_hi) ^ r7) << 4), a0, a1, a2, a3);
            ldsm_x4(kt + k_row_off + (((2 * ks + 2 + k_chunk_hi) ^ r7) << 4), b0, b1, b2, b3);
            mma_16816(sc, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
            mma_16816(sd, b0, b1, b2, b3, qb[ks + 1][0], qb[ks + 1][1]);
        }
#endif
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            sc[j] += sd[j];
            sc[j] += __shfl_xor_sync(0xffffffffu, sc[j], 2);
        }
        const int tok = row0 + (lane >> 2);
        const float s0 = tok < ntok ? sc[0] * scale_log2 : kNegInf;      // head a, row g
        const float s1 = tok < ntok ? sc[1] * scale_log2 : kNegInf;      // head b, row g
        const float s2 = tok + 8 < ntok ? sc[2] * scale_log2 : kNegInf;  // head a, row g+8
        const float s3 = tok + 8 < ntok ? sc[3] * scale_log2 : kNegInf;  // head b, row g+8
        float mx_a = fmaxf(s0, s2);
        float mx_b = fmaxf(s1, s3);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
            mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
            mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
        }
        const float mn_a = fmaxf(m_a, mx_a);
        const float mn_b = fmaxf(m_b, mx_b);
        const float alpha_a = exp2f(m_a - mn_a);
        const float alpha_b = exp2f(m_b - mn_b);
        const float p0 = exp2f(s0 - mn_a);
        const float p1 = exp2f(s1 - mn_b);
        const float p2 = exp2f(s2 - mn_a);
        const float p3 = exp2f(s3 - mn_b);
        l_a = l_a * alpha_a + (p0 + p2);
        l_b = l_b * alpha_b + (p1 + p3);
        m_a = mn_a;
        m_b = mn_b;
#if HKV_CUDA_CORES
        // ---- CUDA cores: p (F32) to shared memory as [token][head], then each
        // lane accumulates its 4 dims of every head over the 16 tokens.
        {
            const int ha = (lane & 1) * 2;
            const int g = lane >> 2;
            if (!lo_side) {
                st_shared_f32x2(pbuf + (g * kGqa + ha) * 4, p0, p1);
                st_shared_f32x2(pbuf + ((g + 8) * kGqa + ha) * 4, p2, p3);
            }
            // the rescale of every head: lane ^ 1 holds the other head pair
            const float alpha_c = __shfl_xor_sync(0xffffffffu, alpha_a, 1);
            const float alpha_d = __shfl_xor_sync(0xffffffffu, alpha_b, 1);
            const float al[kGqa] = {ha == 0 ? alpha_a : alpha_c, ha == 0 ? alpha_b : alpha_d,
                                    ha == 0 ? alpha_c : alpha_a, ha == 0 ? alpha_d : alpha_b};
#pragma unroll
            for (int j = 0; j < kGqa; ++j) {
                acc[j].x *= al[j];
                acc[j].y *= al[j];
                acc[j].z *= al[j];
                acc[j].w *= al[j];
            }
            __syncwarp();
#pragma unroll 4
            for (int t = 0; t < kPageTokens; ++t) {
                const float4 pv = ld_shared_f32x4(pbuf + t * kGqa * 4);
                const uint2 vv = ld_shared_u32x2(vt + t * kRowBytes + (((lane >> 1) ^ (t & 7)) << 4) +
                                                 (lane & 1) * 8);
                const float2 v01 = half2_bits_to_float2(vv.x);
                const float2 v23 = half2_bits_to_float2(vv.y);
                const float pj[kGqa] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
                for (int j = 0; j < kGqa; ++j) {
                    acc[j].x = fmaf(pj[j], v01.x, acc[j].x);
                    acc[j].y = fmaf(pj[j], v01.y, acc[j].y);
                    acc[j].z = fmaf(pj[j], v23.x, acc[j].z);
                    acc[j].w = fmaf(pj[j], v23.y, acc[j].w);
                }
            }
        }
#else
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            o[mt][0] *= alpha_a;
            o[mt][1] *= alpha_b;
            o[mt][2] *= alpha_a;
            o[mt][3] *= alpha_b;
        }
        // ---- P^T tile in shared memory: [token][col], hi parts in cols 0-3,
        // F16 residuals in cols 4-7 (each lane writes its own column pair).
        const uint32_t w_lo = lo_side ? pack_half2(f16_residual(p0), f16_residual(p1))
                                      : pack_half2(p0, p1);
        const uint32_t w_hi = lo_side ? pack_half2(f16_residual(p2), f16_residual(p3))
                                      : pack_half2(p2, p3);
        st_shared_u32(pbuf + (lane >> 2) * 16 + (lane & 3) * 4, w_lo);
        st_shared_u32(pbuf + ((lane >> 2) + 8) * 16 + (lane & 3) * 4, w_hi);
        __syncwarp();
        uint32_t pb0, pb1;
        ldsm_x2_trans(pbuf + (lane & 15) * 16, pb0, pb1);

        // ---- O^T[dim][col] += V^T[dim][token] . P^T[token][col]
#pragma unroll
        for (int mt = 0; mt < 8; ++mt) {
            uint32_t a0, a1, a2, a3;
            const int chunk = 2 * mt + v_chunk_hi;
            ldsm_x4_trans(vt + v_row_off + ((chunk ^ r7) << 4), a0, a1, a2, a3);
            mma_16816(o[mt], a0, a1, a2, a3, pb0, pb1);
        }
#endif
        __syncwarp();
        if (lane == 0 && u + kAttnStages < u_end) {
            fence_proxy_async_smem();
            issue_unit(pool, layer, checked_page(pool, next_page, prod.e, err), prod.h, kt, bar,
                       policy);
            advance(batch, G, prod);
            if (u + kAttnStages + 1 < u_end) {
                next_page = batch.pages[prod.pbase + prod.i];
            }
        }
        advance(batch, G, cons);
    }
    // Let the next launch in the stream start its prologue while this CTA
    // finishes its tail.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    flush(true);
}

// ==================================================================== combine
// One CTA per (segment, query head of its group) for the segments whose
// partials the attention launch before it stored (segments held by one warp
// or one CTA were written there).  Up to kCombineWarps warps each merge a
// contiguous chunk of ceil(p / warps) partials -- eight loads in flight
// before their sums, the first eight issued with the (m, l) loads -- leave
// (o, m, l) in shared memory, and warp 0 merges
// those in warp order: a fixed summation order, so results do not depend on
// timing.  It waits for the attention grid (griddepcontrol.wait) and lets the
// next launch in the stream be scheduled at once.  One head's 128 dims (a
// float4 per lane) keep it small enough to share an SM with an attention CTA.
// In a KV-head split every CTA signals one arrival after its stores.
constexpr int kCombineWarps = 8;
constexpr int kCombineBatch = 8;

__global__ void __launch_bounds__(kCombineWarps * 32)
    combine_kernel(BatchView batch, int layer, const float *__restrict__ part_o,
                   const float *__restrict__ part_ml, float *__restrict__ out, Exchange xchg) {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    __shared__ float4 s_o[kCombineWarps][32];
    __shared__ float2 s_ml[kCombineWarps];
    const int seg = static_cast<int>(blockIdx.x) / kGqa;
    const int j = static_cast<int>(blockIdx.x) - seg * kGqa;  // query head within the group
    const int G = static_cast<int>(gridDim.x) / (kGqa * batch.n);
    // the plan was uploaded before the attention launch this kernel follows
    const int4 sg = batch.seg[seg];
    const int nparts = sg.y;
    if (nparts <= 1) {
        return;
    }
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int lane = threadIdx.x & 31;
    const int wid = threadIdx.x >> 5;
    const int want = (nparts + kCombineBatch - 1) / kCombineBatch;
    const int active = want < kCombineWarps ? want : kCombineWarps;
    const int chunk = (nparts + active - 1) / active;
    const int used = (nparts + chunk - 1) / chunk;  // warps with a non-empty chunk
    if (wid < used) {
        const int p0 = sg.x + wid * chunk;
        const int cnt = min(chunk, nparts - wid * chunk);
        const float2 *mlp = reinterpret_cast<const float2 *>(part_ml) + j;  // (m, l) of head j
        // this lane's float4 of head j in partial p0 + t
        const float4 *pob = reinterpret_cast<const float4 *>(part_o + static_cast<int64_t>(p0) * (kGqa * kHeadDim) +
                                                             j * kHeadDim) + lane;
        float4 ov[kCombineBatch];
        auto load_batch = [&](int t0) {
#pragma unroll
            for (int t = 0; t < kCombineBatch; ++t) {
                if (t0 + t < cnt) {
                    ov[t] = __ldcg(pob + static_cast<int64_t>(t0 + t) * (kGqa * kHeadDim / 4));
                }
            }
        };
        // the first batch of outputs goes out with the (m, l) loads: the
        // outputs do not depend on the weights
        load_batch(0);
        float mx = -INFINITY;
        float2 own = make_float2(-INFINITY, 0.f);  // (m, l) of partial p0 + lane
        for (int b = lane; b < cnt; b += 32) {
            const float2 ml = __ldcg(mlp + static_cast<int64_t>(p0 + b) * kGqa);
            if (b == lane) {
                own = ml;
            }
            mx = fmaxf(mx, ml.x);
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
        }
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        float den = 0.f;
        for (int b = 0; b < cnt; b += 32) {
            float w = 0.f;
            if (b + lane < cnt) {
                const float2 ml = b == 0 ? own : __ldcg(mlp + static_cast<int64_t>(p0 + b + lane) * kGqa);
                w = exp2f(ml.x - mx);
                den += w * ml.y;
            }
            const int cb = min(32, cnt - b);
            for (int t0 = 0; t0 < cb; t0 += kCombineBatch) {
                if (b + t0 > 0) {
                    load_batch(b + t0);
                }
#pragma unroll
                for (int t = 0; t < kCombineBatch; ++t) {
                    if (t0 + t < cb) {
                        const float wt = __shfl_sync(0xffffffffu, w, t0 + t);
                        acc.x += wt * ov[t].x;
                        acc.y += wt * ov[t].y;
                        acc.z += wt * ov[t].z;
                        acc.w += wt * ov[t].w;
                    }
                }
            }
        }
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) {
            den += __shfl_xor_sync(0xffffffffu, den, off);
        }
        s_o[wid][lane] = acc;
        if (lane == 0) {
            s_ml[wid] = make_float2(mx, den);
        }
    }
    __syncthreads();
    if (wid != 0) {
        return;
    }
    float mx = -INFINITY;
    for (int w = 0; w < used; ++w) {
        mx = fmaxf(mx, s_ml[w].x);
    }
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    float den = 0.f;
    for (int w = 0; w < used; ++w) {
        const float wt = exp2f(s_ml[w].x - mx);
        den += wt * s_ml[w].y;
        const float4 ov = s_o[w][lane];
        acc.x += wt * ov.x;
        acc.y += wt * ov.y;
        acc.z += wt * ov.z;
        acc.w += wt * ov.w;
    }
    const float inv = 1.f / den;
    const float4 res = make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
    const int e = seg / G;
    const int h = seg - e * G;
    const int n_dst = xchg.n_ranks == 0 ? 1 : xchg.n_ranks;
    for (int r = 0; r < n_dst; ++r) {
        float4 *ob = reinterpret_cast<float4 *>(out_slice(out, xchg, r, layer, e, h, G) + j * kHeadDim);
        ob[lane] = res;
    }
    signal_arrival(xchg, layer, lane);
}

// ================================================================ copy-on-write
// One block per (page pair, layer): copies the source page's K and V head
// blocks of that layer (2 * n_head_kv * 4 KiB, contiguous in the layer's slab)
// onto the destination page with 16-byte loads and stores.  All pending
// copies of a call go out in this one launch.
__global__ void __launch_bounds__(256) cow_copy_kernel(PoolView pool, const int2 *__restrict__ pairs,
                                                       int32_t n_pairs, DeviceError *err) {
    const int64_t item = blockIdx.x;
    const int64_t pair = item / pool.n_layers;
    const int layer = static_cast<int>(item - pair * pool.n_layers);
    if (pair >= n_pairs) {
        return;
    }
    const int2 pr = pairs[pair];
    if (pr.x < 0 || pr.x >= pool.n_pages || pr.y < 0 || pr.y >= pool.n_pages) {
        if (threadIdx.x == 0) {
            record_error(err, kErrBadIndex, kWhereCow, pr.x, pr.y);
        }
        return;
    }
    const int G = pool.n_head_kv;
    const uint4 *src = reinterpret_cast<const uint4 *>(
        pool.base + head_block_index(pr.x, layer, 0, 0, pool.n_pages, G) * kHeadBlockBytes);
    uint4 *dst = reinterpret_cast<uint4 *>(
        pool.base + head_block_index(pr.y, layer, 0, 0, pool.n_pages, G) * kHeadBlockBytes);
    const int n16 = 2 * G * kHeadBlockBytes / 16;
    for (int i = threadIdx.x; i < n16; i += blockDim.x) {
        dst[i] = __ldcs(src + i);
    }
}

// ===================================================================== gather
__global__ void gather_kernel(PoolView pool, const int32_t *__restrict__ slot_pages, int64_t pos0,
                              int64_t n, int layer, uint16_t *__restrict__ k_out,
                              uint16_t *__restrict__ v_out, DeviceError *err) {
    const int G = pool.n_head_kv;
    const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int64_t per_row = static_cast<int64_t>(G) * 16;
    if (idx >= n * per_row) {
        return;
    }
    const int64_t t = idx / per_row;
    const int rem = static_cast<int>(idx - t * per_row);
    const int h = rem >> 4;
    const int c = rem & 15;
    const int64_t pos = pos0 + t;
    const int64_t page = slot_pages[pos >> 4];
    if (page < 0 || page >= pool.n_pages) {
        record_error(err, kErrBadIndex, kWhereGather, static_cast<int>(page),
                     static_cast<int>(pos));
        return;
    }
    const int r = static_cast<int>(pos & 15);
    const int64_t within = r * kRowBytes + swizzled_chunk(r, c) * 16;
    const uint8_t *kb =
        pool.base + head_block_index(page, layer, 0, h, pool.n_pages, G) * kHeadBlockBytes;
    const uint8_t *vb =
        pool.base + head_block_index(page, layer, 1, h, pool.n_pages, G) * kHeadBlockBytes;
    const int64_t o = (t * G + h) * kHeadDim + c * 8;
    *reinterpret_cast<uint4 *>(k_out + o) = *reinterpret_cast<const uint4 *>(kb + within);
    *reinterpret_cast<uint4 *>(v_out + o) = *reinterpret_cast<const uint4 *>(vb + within);
}

}  // namespace

size_t attention_smem_bytes(bool cta_merge, bool cluster) {
    return static_cast<size_t>(kAttnWarps) * kWarpSmem + (cta_merge ? kCtaSmem : 0) +
           (cluster ? kClusterSmem : 0);
}

// The shared-memory opt-in (and, for the cluster variant, sizes up to 16) of
// one attention kernel, once per device.
template <bool kAppend, bool kCtaMerge, bool kCluster>
void configure_attention(int dev) {
    static bool configured[64] = {};
    if (dev >= 0 && dev < 64 && configured[dev]) {
        return;
    }
    auto kern = attention_kernel<kAppend, kCtaMerge, kCluster>;
    cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         static_cast<int>(attention_smem_bytes(kCtaMerge, kCluster)));
    if (kCluster) {
        cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    }
    if (dev >= 0 && dev < 64) {
        configured[dev] = true;
    }
}

int attention_cluster_fit(int csize) {
    static std::mutex mu;
    static int cache[64][kMaxCluster + 1] = {};
    if (csize < 2 || csize > kMaxCluster) {
        return 0;
    }
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        return 0;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev][csize] != 0) {
        return cache[dev][csize] > 0 ? cache[dev][csize] : 0;
    }
    configure_attention<true, true, true>(dev);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(csize));
    cfg.blockDim = dim3(kAttnWarps * 32);
    cfg.dynamicSmemBytes = attention_smem_bytes(true, true);
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = static_cast<unsigned>(csize);
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, attention_kernel<true, true, true>, &cfg) != cudaSuccess) {
        n = 0;
    }
    (void)cudaGetLastError();
    cache[dev][csize] = n > 0 ? n : -1;
    return n > 0 ? n : 0;
}

void launch_append(const PoolView &pool, const RopeView &rope, const BatchView &batch, int layer,
                   const float *k, const float *v, bool apply_rope, DeviceError *err,
                   cudaStream_t stream) {
    const int64_t warps = static_cast<int64_t>(batch.n) * pool.n_head_kv;
    const int blocks = static_cast<int>((warps + 3) / 4);
    if (apply_rope) {
        append_kernel<true, false><<<blocks, 128, 0, stream>>>(pool, rope, batch, nullptr, 0,
                                                               batch.n, layer, k, v, err);
    } else {
        append_kernel<false, false><<<blocks, 128, 0, stream>>>(pool, rope, batch, nullptr, 0,
                                                                batch.n, layer, k, v, err);
    }
}

void launch_append_range(const PoolView &pool, const RopeView &rope, const int32_t *range_pages,
                         int64_t pos0, int64_t n_tokens, int layer, const float *k, const float *v,
                         bool apply_rope, DeviceError *err, cudaStream_t stream) {
    const int64_t warps = n_tokens * pool.n_head_kv;
    const int blocks = static_cast<int>((warps + 3) / 4);
    BatchView none{};
    if (apply_rope) {
        append_kernel<true, true><<<blocks, 128, 0, stream>>>(pool, rope, none, range_pages, pos0,
                                                              n_tokens, layer, k, v, err);
    } else {
        append_kernel<false, true><<<blocks, 128, 0, stream>>>(pool, rope, none, range_pages,
                                                               pos0, n_tokens, layer, k, v, err);
    }
}

template <bool kAppend, bool kCtaMerge, bool kCluster>
void launch_attention_t(const PoolView &pool, const RopeView &rope, const BatchView &batch,
                        int layer, const float *q, const float *k_new, const float *v_new,
                        float *part_o, float *part_ml, int32_t *counters, float *out,
                        const Exchange &xchg, float scale_log2, DeviceError *err,
                        bool overlap_previous, cudaStream_t stream) {
    int dev = 0;
    cudaGetDevice(&dev);
    configure_attention<kAppend, kCtaMerge, kCluster>(dev);
    const int grid = (batch.n_warps + kAttnWarps - 1) / kAttnWarps;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kAttnWarps * 32);
    cfg.dynamicSmemBytes = attention_smem_bytes(kCtaMerge, kCluster);
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int n_attr = 0;
    if (overlap_previous) {
        attr[n_attr].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[n_attr].val.programmaticStreamSerializationAllowed = 1;
        ++n_attr;
    }
    if (kCluster) {
        attr[n_attr].id = cudaLaunchAttributeClusterDimension;
        attr[n_attr].val.clusterDim.x = static_cast<unsigned>(batch.cluster);
        attr[n_attr].val.clusterDim.y = 1;
        attr[n_attr].val.clusterDim.z = 1;
        ++n_attr;
    }
    cfg.attrs = attr;
    cfg.numAttrs = static_cast<unsigned>(n_attr);
    cudaLaunchKernelEx(&cfg, attention_kernel<kAppend, kCtaMerge, kCluster>, pool, rope, batch, layer, q,
                       k_new, v_new, part_o, part_ml, counters, out, xchg, scale_log2, err);
    if (batch.combine && batch.split_segments > 0) {
        cudaLaunchConfig_t cc = {};
        cc.gridDim = dim3(static_cast<unsigned>(batch.n * pool.n_head_kv * kGqa));
        cc.blockDim = dim3(kCombineWarps * 32);
        cc.stream = stream;
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cc.attrs = attr;
        cc.numAttrs = 1;
        cudaLaunchKernelEx(&cc, combine_kernel, batch, layer, part_o, part_ml, out, xchg);
    }
}

void launch_attention(const PoolView &pool, const RopeView &rope, const BatchView &batch, int layer,
                      const float *q, const float *k_new, const float *v_new, float *part_o,
                      float *part_ml, int32_t *counters, float *out, const Exchange &xchg,
                      float scale_log2, DeviceError *err, bool overlap_previous,
                      cudaStream_t stream) {
    const bool append = k_new != nullptr && v_new != nullptr;
    if (!append) {
        k_new = v_new = nullptr;
    }
    if (append && batch.cluster > 0) {
        launch_attention_t<true, true, true>(pool, rope, batch, layer, q, k_new, v_new, part_o, part_ml,
                                             counters, out, xchg, scale_log2, err, overlap_previous, stream);
    } else if (append && batch.cta_merge) {
        launch_attention_t<true, true, false>(pool, rope, batch, layer, q, k_new, v_new, part_o, part_ml,
                                              counters, out, xchg, scale_log2, err, overlap_previous, stream);
    } else if (append) {
        launch_attention_t<true, false, false>(pool, rope, batch, layer, q, k_new, v_new, part_o, part_ml,
                                               counters, out, xchg, scale_log2, err, overlap_previous, stream);
    } else if (batch.cluster > 0) {
        launch_attention_t<false, true, true>(pool, rope, batch, layer, q, k_new, v_new, part_o, part_ml,
                                              counters, out, xchg, scale_log2, err, overlap_previous, stream);
    } else if (batch.cta_merge) {
        launch_attention_t<false, true, false>(pool, rope, batch, layer, q, k_new, v_new, part_o, part_ml,
                                               counters, out, xchg, scale_log2, err, overlap_previous, stream);
    } else {
        launch_attention_t<false, false, false>(pool, rope, batch, layer, q, k_new, v_new, part_o, part_ml,
                                                counters, out, xchg, scale_log2, err, overlap_previous, stream);
    }
}

// =================================================================== split wait
__global__ void split_wait_kernel(const uint32_t *flag, uint32_t target, DeviceError *err) {
    // The next decode launch may start its prologue (plan and page reads of
    // its own layer) while this wait spins; its griddepcontrol.wait still
    // holds everything else until the arrivals are complete.
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const long long t0 = clock64();
    const volatile uint32_t *f = flag;
    while (static_cast<int32_t>(*f - target) < 0) {
        if (clock64() - t0 > kWaitBudgetCycles) {
            record_error(err, kErrTimeout, kWhereSplitWait, static_cast<int>(*f),
                         static_cast<int>(target));
            return;
        }
        __nanosleep(32);
    }
    __threadfence_system();
}

// Launched as a dependent of the decode launch before it: it may start while
// that kernel's tail still runs.  It completes only when every slice of the
// layer has arrived, and on every rank a slice's arrival comes after all reads
// of that (slot, head)'s partials and the reset of its counters, so the next
// decode launch (which waits for this one) never races the previous one.
void launch_split_wait(const uint32_t *flag, uint32_t target, DeviceError *err,
                       cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(1);
    cfg.blockDim = dim3(1);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, split_wait_kernel, flag, target, err);
}

void launch_cow_copy(const PoolView &pool, const int32_t *pairs, int32_t n_pairs, DeviceError *err,
                     cudaStream_t stream) {
    const int64_t blocks = static_cast<int64_t>(n_pairs) * pool.n_layers;
    if (blocks <= 0) {
        return;
    }
    cow_copy_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(
        pool, reinterpret_cast<const int2 *>(pairs), n_pairs, err);
}

void launch_gather(const PoolView &pool, const int32_t *slot_pages, int64_t pos0, int64_t n,
                   int layer, uint16_t *k_out, uint16_t *v_out, DeviceError *err,
                   cudaStream_t stream) {
    const int64_t threads = n * pool.n_head_kv * 16;
    const int blocks = static_cast<int>((threads + 255) / 256);
    gather_kernel<<<blocks, 256, 0, stream>>>(pool, slot_pages, pos0, n, layer, k_out, v_out, err);
}

}  // namespace hkv
