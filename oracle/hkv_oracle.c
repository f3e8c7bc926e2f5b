/*
 * hkv_oracle.c -- CPU restatement of the reference's KV-cache decode path.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product (libhkv.so, the package's
 * host code) links, loads or calls this file.  It is used by tests/ as the
 * parity reference, by __graft_entry__.smoke() to check one tiny GPU run,
 * and by bench.py as the timed CPU baseline / reference arm.
 *
 * Reference: bluryar/higgs-audio.cpp, src/higgs_pipeline.cpp.  The reference's
 * arithmetic lives in the ggml submodule (ggml-org/ggml, README.md:32 pins
 * v0.15.3), which is absent from the reference checkout, so the reference
 * cannot be compiled here.  Pinning status:
 *   * K/V append (ggml_set_inplace, :5748-5749): PINNED by the known-answer
 *     pattern of self_check_backend_kv_cache_write (:6969-6986), replayed by
 *     tests/test_oracle.py and tests/test_gpu_parity.py.
 *   * cache layout / offsets (:1115-1120, :1137-1142): PINNED by the
 *     front/back known-answer writes of self_check_kv_cache (:5206-5227).
 *   * BF16 RoPE table (:471-487): the reference's own table code is compiled
 *     from its source by oracle/ref_rope_table.sh into oracle/_ref/ (when the
 *     reference checkout is present) and compared bit for bit.
 *   * NEOX RoPE (:489-506) and the attention chain (:5750-5786): parity
 *     UNPINNED -- the reference's decode self-checks only test shape and
 *     finiteness (:5350-5359, :7017-7023).  This file restates the graph op
 *     by op; ggml's internal rounding points are restated from the published
 *     upstream ggml algorithm.
 *
 * Compile with -ffp-contract=off: the reference's RoPE is three separate ggml
 * ops (mul, mul, sub/add), each rounded to F32, never a fused multiply-add.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ---------------------------------------------------------------- bf16 --
 * ggml_fp32_to_bf16 / ggml_bf16_to_fp32 as used by bf16_rne_to_f32
 * (src/higgs_pipeline.cpp:471-473): round to nearest even on the top 16 bits,
 * NaN forced quiet (upstream ggml's published conversion). */
static uint16_t bf16_bits(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) {
        return (uint16_t)((u >> 16) | 64u);
    }
    return (uint16_t)((u + (0x7fffu + ((u >> 16) & 1u))) >> 16);
}

float hkvo_bf16_round(float x) {
    uint32_t u = (uint32_t)bf16_bits(x) << 16;
    float out;
    memcpy(&out, &u, 4);
    return out;
}

/* make_bf16_rope_table (src/higgs_pipeline.cpp:475-487):
 *   freq_i  = 1 / powf(base, (2i) / key_length)      (float pow overload)
 *   angle   = (float)pos * freq_i
 *   table   = bf16_rne(cos/sin(angle)) stored as F32, row-major [pos][half]. */
void hkvo_rope_table(int64_t context_length, int64_t key_length, float base,
                     float *cos_tab, float *sin_tab) {
    const int64_t half = key_length / 2;
    for (int64_t pos = 0; pos < context_length; ++pos) {
        for (int64_t i = 0; i < half; ++i) {
            const float dim = (float)(i * 2);
            const float freq = 1.0f / powf(base, dim / (float)key_length);
            const float angle = (float)pos * freq;
            cos_tab[pos * half + i] = hkvo_bf16_round(cosf(angle));
            sin_tab[pos * half + i] = hkvo_bf16_round(sinf(angle));
        }
    }
}

/* ---------------------------------------------------------------- f16 --
 * IEEE binary32 -> binary16, round to nearest even (the conversion an F16
 * ggml cache and CUDA's __float2half_rn perform).  NaN maps to 0x7e00|sign. */
uint16_t hkvo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t a = x & 0x7fffffffu;
    if (a > 0x7f800000u) {
        return (uint16_t)(sign | 0x7e00u);
    }
    if (a >= 0x477ff000u) { /* >= 65520 rounds to infinity */
        return (uint16_t)(sign | 0x7c00u);
    }
    if (a >= 0x38800000u) { /* normal half */
        const uint32_t r = a + 0xfffu + ((a >> 13) & 1u) - (112u << 23);
        return (uint16_t)(sign | (r >> 13));
    }
    if (a < 0x33000000u) { /* below half of the smallest subnormal */
        return (uint16_t)sign;
    }
    const uint32_t e = a >> 23;
    const uint32_t m = (a & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e; /* 14..24 */
    uint32_t q = m >> shift;
    const uint32_t rem = m & ((1u << shift) - 1u);
    const uint32_t halfway = 1u << (shift - 1u);
    if (rem > halfway || (rem == halfway && (q & 1u))) {
        ++q;
    }
    return (uint16_t)(sign | q);
}

float hkvo_f16_to_f32(uint16_t h) {
    const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = ((uint32_t)h >> 10) & 0x1fu;
    uint32_t m = (uint32_t)h & 0x3ffu;
    uint32_t bits;
    if (e == 0x1fu) {
        bits = sign | 0x7f800000u | (m << 13);
    } else if (e != 0) {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    } else if (m == 0) {
        bits = sign;
    } else {
        e = 113u;
        while ((m & 0x400u) == 0) {
            m <<= 1;
            --e;
        }
        bits = sign | (e << 23) | ((m & 0x3ffu) << 13);
    }
    float out;
    memcpy(&out, &bits, 4);
    return out;
}

void hkvo_f32_to_f16_array(const float *src, uint16_t *dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        dst[i] = hkvo_f32_to_f16(src[i]);
    }
}

void hkvo_f16_to_f32_array(const uint16_t *src, float *dst, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
        dst[i] = hkvo_f16_to_f32(src[i]);
    }
}

/* ---------------------------------------------------------------- RoPE --
 * neox_rope_bf16_cache (src/higgs_pipeline.cpp:489-506) for one token:
 *   x0 = x[:, :half], x1 = x[:, half:]
 *   y0 = (x0*cos) - (x1*sin);  y1 = (x0*sin) + (x1*cos)
 * each product and each sum rounded to F32 separately (ggml_mul, ggml_sub,
 * ggml_add are distinct graph nodes).  x, y: [n_head][head_dim]. */
void hkvo_rope_neox(const float *x, int64_t n_head, int64_t head_dim,
                    const float *cos_row, const float *sin_row, float *y) {
    const int64_t half = head_dim / 2;
    for (int64_t h = 0; h < n_head; ++h) {
        const float *xh = x + h * head_dim;
        float *yh = y + h * head_dim;
        for (int64_t i = 0; i < half; ++i) {
            const float c = cos_row[i];
            const float s = sin_row[i];
            const float x0 = xh[i];
            const float x1 = xh[i + half];
            const float a = x0 * c;
            const float b = x1 * s;
            const float d = x0 * s;
            const float e = x1 * c;
            yh[i] = a - b;
            yh[i + half] = d + e;
        }
    }
}

/* RoPE + F16 store of n rows: the content the paged cache must hold after an
 * append of pre-RoPE k and raw v (ggml_set_inplace of the roped k_cur / raw
 * v_cur, :5734-5749), then F32->F16 RNE for the F16 cache.
 * k, v: [n][n_head_kv][head_dim] F32; pos: [n]; tables [ctx][head_dim/2].
 * k_out, v_out: [n][n_head_kv][head_dim] F16 bits.  rope=0 copies k raw. */
void hkvo_append_rows(int64_t n, int64_t n_head_kv, int64_t head_dim,
                      const float *k, const float *v, const int32_t *pos,
                      const float *cos_tab, const float *sin_tab, int rope,
                      uint16_t *k_out, uint16_t *v_out) {
    const int64_t half = head_dim / 2;
    const int64_t row = n_head_kv * head_dim;
    float *tmp = (float *)malloc((size_t)row * sizeof(float));
    for (int64_t t = 0; t < n; ++t) {
        if (rope) {
            hkvo_rope_neox(k + t * row, n_head_kv, head_dim, cos_tab + (int64_t)pos[t] * half,
                           sin_tab + (int64_t)pos[t] * half, tmp);
        } else {
            memcpy(tmp, k + t * row, (size_t)row * sizeof(float));
        }
        hkvo_f32_to_f16_array(tmp, k_out + t * row, row);
        hkvo_f32_to_f16_array(v + t * row, v_out + t * row, row);
    }
    free(tmp);
}

/* ----------------------------------------------------------- attention --
 * GQA decode attention over logical F16 caches (the chain at
 * src/higgs_pipeline.cpp:5750-5786 for one new token):
 *   head h reads KV head h / (n_head / n_head_kv)       (repeat_kv_3d, :441-456)
 *   s_j = (q_h . k_j) * scale      scale applied after the dot (:5764-5767)
 *   p   = softmax_j(s)             no mask: rows [0, n_tok) only (:5775)
 *   o_h = sum_j p_j v_j            head-major output o[h*D + d] (:5783-5786)
 * q: roped query [n][n_head][head_dim] F32.
 * k_all / v_all: logical caches, slot e's rows start at row_off[e], each row
 *   [n_head_kv][head_dim] F16 bits; slot e attends n_tok[e] rows.
 * mode 0 ("exact"): F16 K/V widened exactly, double accumulation throughout.
 * mode 1 ("ggml_f16"): upstream ggml CPU semantics for an F16 src0 mul_mat:
 *   q rounded to F16 (vec_dot_type of F16), softmax probabilities rounded to
 *   F16 before PV, F32 softmax; accumulations carried in double here.
 * out: [n][n_head*head_dim] F32. */
void hkvo_decode_attn(int mode, int64_t n, int64_t n_head, int64_t n_head_kv,
                      int64_t head_dim, const float *q, const uint16_t *k_all,
                      const uint16_t *v_all, const int64_t *row_off, const int32_t *n_tok,
                      float scale, float *out) {
    const int64_t rep = n_head / n_head_kv;
    const int64_t kv_row = n_head_kv * head_dim;
#pragma omp parallel for collapse(2) schedule(dynamic)
    for (int64_t e = 0; e < n; ++e) {
        for (int64_t h = 0; h < n_head; ++h) {
            const int64_t L = n_tok[e];
            const int64_t g = h / rep;
            const float *qh = q + (e * n_head + h) * head_dim;
            float *oh = out + e * n_head * head_dim + h * head_dim;
            double *s = (double *)malloc((size_t)(L > 0 ? L : 1) * sizeof(double));
            double *acc = (double *)calloc((size_t)head_dim, sizeof(double));
            float *qv = (float *)malloc((size_t)head_dim * sizeof(float));
            for (int64_t d = 0; d < head_dim; ++d) {
                qv[d] = mode == 1 ? hkvo_f16_to_f32(hkvo_f32_to_f16(qh[d])) : qh[d];
            }
            double mx = -INFINITY;
            for (int64_t j = 0; j < L; ++j) {
                const uint16_t *kr = k_all + (row_off[e] + j) * kv_row + g * head_dim;
                double dot = 0.0;
                for (int64_t d = 0; d < head_dim; ++d) {
                    dot += (double)qv[d] * (double)hkvo_f16_to_f32(kr[d]);
                }
                double sj;
                if (mode == 1) {
                    sj = (double)((float)dot * scale);
                } else {
                    sj = dot * (double)scale;
                }
                s[j] = sj;
                if (sj > mx) {
                    mx = sj;
                }
            }
            double l = 0.0;
            for (int64_t j = 0; j < L; ++j) {
                double p;
                if (mode == 1) {
                    p = (double)expf((float)(s[j] - mx));
                } else {
                    p = exp(s[j] - mx);
                }
                s[j] = p;
                l += p;
            }
            const double inv = l > 0.0 ? 1.0 / l : 0.0;
            const float inv_f = (float)inv;
            for (int64_t j = 0; j < L; ++j) {
                double p;
                if (mode == 1) {
                    p = (double)hkvo_f16_to_f32(hkvo_f32_to_f16((float)s[j] * inv_f));
                } else {
                    p = s[j] * inv;
                }
                const uint16_t *vr = v_all + (row_off[e] + j) * kv_row + g * head_dim;
                for (int64_t d = 0; d < head_dim; ++d) {
                    acc[d] += p * (double)hkvo_f16_to_f32(vr[d]);
                }
            }
            for (int64_t d = 0; d < head_dim; ++d) {
                oh[d] = (float)acc[d];
            }
            free(qv);
            free(acc);
            free(s);
        }
    }
}

int hkvo_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

void hkvo_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) {
        omp_set_num_threads(n);
    }
#else
    (void)n;
#endif
}
