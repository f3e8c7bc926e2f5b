/*
 * hkv_oracle_graph.c -- the reference's GGML-CPU decode-attention graph for
 * one layer, restated op by op, used as the TIMED CPU BASELINE.
 *
 * TEST / MEASUREMENT INFRASTRUCTURE ONLY (bench.py's cpu_baseline leg and
 * `--impl reference` arm, and tests/).  The product never calls it.
 *
 * Follows run_kv_decode_graph_all_layers_with_backend_cache_ex
 * (src/higgs_pipeline.cpp:5629-5786) for one layer and one slot at a time,
 * the way the reference's single CUDA-executor/CPU backend serialises
 * requests (:4819-4825), with each graph op spread over all threads the way
 * ggml's CPU backend splits an op's rows across its thread pool:
 *   1. neox_rope_bf16_cache on q and k              (:5734-5735, :489-506)
 *   2. ggml_set_inplace of k_cur / v_cur at row past (:5748-5749), F32 cache
 *      ne=[head_dim, kv_heads, capacity] (:1161-1162)
 *   3. view rows [0, past] and repeat_kv_3d: materialise K and V to all query
 *      heads, [total][n_head][head_dim]           (:5750-5753, :441-456)
 *   4. kq = mul_mat(k4, q4)                        (:5764-5766)
 *   5. kq = scale(kq, 1/sqrt(head_dim))            (:5767)
 *   6. soft_max over the key axis                  (:5775)
 *   7. v_for_mm = cont(permute(v, 1,2,0,3))        (:5783), [n_head][head_dim][total]
 *   8. kqv = mul_mat(v_for_mm, kq)                 (:5784)
 *   9. permute + cont_2d to head-major [n_head*head_dim] (:5785-5786)
 * The RoPE helper comes from hkv_oracle.c (compiled without FMA contraction);
 * this file may be compiled with vectorising flags since ggml's own F32 dot
 * products are SIMD with reassociated partial sums.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

void hkvo_rope_neox(const float *x, int64_t n_head, int64_t head_dim,
                    const float *cos_row, const float *sin_row, float *y);

static float dot_f32(const float *a, const float *b, int64_t n) {
    float acc[16] = {0};
    int64_t i = 0;
    for (; i + 16 <= n; i += 16) {
        for (int k = 0; k < 16; ++k) {
            acc[k] += a[i + k] * b[i + k];
        }
    }
    float s = 0.0f;
    for (int k = 0; k < 16; ++k) {
        s += acc[k];
    }
    for (; i < n; ++i) {
        s += a[i] * b[i];
    }
    return s;
}

/* One layer of decode for n slots, each slot processed as one ggml graph.
 * q_pre [n][n_head][D], k_pre / v_new [n][n_head_kv][D] (F32, pre-RoPE q, k).
 * k_cache / v_cache: F32 [rows][n_head_kv][D]; slot e's cache starts at row
 *   row_off[e]; past[e] is the row the new token is written to; the slot then
 *   attends rows [0, past[e]].
 * cos_tab / sin_tab: [context][D/2] BF16-rounded tables.
 * work: caller scratch of hkvo_graph_work_floats() floats (reused across
 *   calls so the timed loop does no allocation or first-touch faulting).
 * out [n][n_head*D]. */
void hkvo_graph_decode_layer(int64_t n, int64_t n_head, int64_t n_head_kv, int64_t head_dim,
                             const float *q_pre, const float *k_pre, const float *v_new,
                             float *k_cache, float *v_cache, const int64_t *row_off,
                             const int32_t *past, const float *cos_tab, const float *sin_tab,
                             float scale, float *work, float *out) {
    const int64_t D = head_dim;
    const int64_t H = n_head;
    const int64_t G = n_head_kv;
    const int64_t R = H / G;
    const int64_t half = D / 2;
    int64_t max_total = 1;
    for (int64_t e = 0; e < n; ++e) {
        if ((int64_t)past[e] + 1 > max_total) {
            max_total = (int64_t)past[e] + 1;
        }
    }
    float *k4 = work;                         /* [total][H][D] */
    float *v4 = k4 + max_total * H * D;       /* [total][H][D] */
    float *vt = v4 + max_total * H * D;       /* [H][D][total] */
    float *kq = vt + max_total * H * D;       /* [H][total] */
    float *q = kq + H * max_total;            /* [H][D] roped */
    float *kqv = q + H * D;                   /* [H][D] */
    float *kr = kqv + H * D;                  /* [G][D] roped */

    for (int64_t e = 0; e < n; ++e) {
        const int64_t p = past[e];
        const int64_t total = p + 1;
        const float *cr = cos_tab + p * half;
        const float *sr = sin_tab + p * half;
        float *kc = k_cache + row_off[e] * G * D;
        float *vc = v_cache + row_off[e] * G * D;
        /* 1. RoPE */
        hkvo_rope_neox(q_pre + e * H * D, H, D, cr, sr, q);
        hkvo_rope_neox(k_pre + e * G * D, G, D, cr, sr, kr);
        /* 2. set_inplace */
        memcpy(kc + p * G * D, kr, (size_t)(G * D) * sizeof(float));
        memcpy(vc + p * G * D, v_new + e * G * D, (size_t)(G * D) * sizeof(float));
        /* 3. repeat_kv_3d (materialised) */
#pragma omp parallel for schedule(static)
        for (int64_t j = 0; j < total; ++j) {
            for (int64_t h = 0; h < H; ++h) {
                memcpy(k4 + (j * H + h) * D, kc + (j * G + h / R) * D, (size_t)D * sizeof(float));
                memcpy(v4 + (j * H + h) * D, vc + (j * G + h / R) * D, (size_t)D * sizeof(float));
            }
        }
        /* 4. kq = mul_mat(k4, q4) */
#pragma omp parallel for collapse(2) schedule(static)
        for (int64_t h = 0; h < H; ++h) {
            for (int64_t j = 0; j < total; ++j) {
                kq[h * total + j] = dot_f32(k4 + (j * H + h) * D, q + h * D, D);
            }
        }
        /* 5. scale */
#pragma omp parallel for schedule(static)
        for (int64_t i = 0; i < H * total; ++i) {
            kq[i] *= scale;
        }
        /* 6. soft_max */
#pragma omp parallel for schedule(static)
        for (int64_t h = 0; h < H; ++h) {
            float *row = kq + h * total;
            float mx = -INFINITY;
            for (int64_t j = 0; j < total; ++j) {
                mx = row[j] > mx ? row[j] : mx;
            }
            double sum = 0.0;
            for (int64_t j = 0; j < total; ++j) {
                row[j] = expf(row[j] - mx);
                sum += row[j];
            }
            const float inv = (float)(1.0 / sum);
            for (int64_t j = 0; j < total; ++j) {
                row[j] *= inv;
            }
        }
        /* 7. v_for_mm = cont(permute(v4, 1, 2, 0, 3)) -> [H][D][total] */
#pragma omp parallel for collapse(2) schedule(static)
        for (int64_t h = 0; h < H; ++h) {
            for (int64_t d = 0; d < D; ++d) {
                float *dst = vt + (h * D + d) * total;
                for (int64_t j = 0; j < total; ++j) {
                    dst[j] = v4[(j * H + h) * D + d];
                }
            }
        }
        /* 8. kqv = mul_mat(v_for_mm, kq) */
#pragma omp parallel for collapse(2) schedule(static)
        for (int64_t h = 0; h < H; ++h) {
            for (int64_t d = 0; d < D; ++d) {
                kqv[h * D + d] = dot_f32(vt + (h * D + d) * total, kq + h * total, total);
            }
        }
        /* 9. permute + cont_2d: head-major output */
        memcpy(out + e * H * D, kqv, (size_t)(H * D) * sizeof(float));
    }
}

/* Scratch floats hkvo_graph_decode_layer needs for a given max total. */
int64_t hkvo_graph_work_floats(int64_t max_total, int64_t n_head, int64_t n_head_kv, int64_t head_dim) {
    return 3 * max_total * n_head * head_dim + n_head * max_total + 2 * n_head * head_dim +
           n_head_kv * head_dim;
}
