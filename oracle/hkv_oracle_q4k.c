/* hkv_oracle_q4k.c -- CPU restatement of the Q4_K matrix-vector path of the
 * reference's backbone (TEST INFRASTRUCTURE, never the product).
 *
 * The reference runs its projections as mul_mat_f32(weight, activation)
 * (src/higgs_pipeline.cpp:465-469) over GGUF weights; with Q4_K weights the
 * GGML CPU backend quantises the F32 activation row to Q8_K and takes the
 * Q4_K x Q8_K dot product per weight row.  Those steps live in ggml v0.15.3
 * (the reference's vendor/ggml submodule, absent from the checkout); this file
 * restates ggml's published definitions:
 *   - block_q4_K: 256 weights in 144 bytes = f16 d, f16 dmin, 12 bytes of
 *     packed 6-bit (scale, min) pairs for 8 sub-blocks of 32, 128 bytes of
 *     4-bit quants (sub-block 2j in the low nibbles of bytes 32j..32j+31,
 *     sub-block 2j+1 in the high nibbles); w = d*sc*q - dmin*m.
 *   - block_q8_K: 256 activations in 292 bytes = f32 d, 256 int8, 16 int16
 *     sums of 16-element groups; quantised with iscale = -127/max where max
 *     is the element of largest magnitude (first one on ties), q =
 *     min(127, round-half-even(iscale*x)), d = 1/iscale.
 *   - the dot product (ggml's generic vec_dot_q4_K_q8_K): per block, 8
 *     int32 lanes accumulate scale * (q4 * q8) over 8-element groups, then
 *     sums[l] += (d4 * d8) * lane[l]; the mins enter as
 *     -(dmin4 * d8) * sum_j(bsum_j * m_{j/2}); the 8 lanes are added last.
 *   - rms_norm (ggml CPU): sum of x*x in double, mean = (float)(sum / n),
 *     scale = 1/sqrtf(mean + eps), y = x * scale; then y * weight (ggml_mul).
 *   - silu (scalar form): x / (1 + expf(-x)).
 * Pinning: the Q4_K decoding is checked against gguf.quants.dequantize
 * (gguf 0.19.0, installed) on random blocks; the Q8_K quantiser and the dot
 * product are checked against float64 dot products of the decoded blocks
 * (tests/test_oracle_q4k.py).  ggml itself cannot be built here.
 *
 * Compiled with -ffp-contract=off (oracle/Makefile, exact flags).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define QK 256
#define Q4K_BYTES 144
#define Q8K_BYTES 292

float hkvo_f16_to_f32(uint16_t h);

static void unpack_scale_min(const uint8_t *s, int j, int *sc, int *m) {
    if (j < 4) {
        *sc = s[j] & 63;
        *m = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0F) | ((s[j - 4] >> 6) << 4);
        *m = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

static float load_f16(const uint8_t *p) {
    uint16_t h;
    memcpy(&h, p, 2);
    return hkvo_f16_to_f32(h);
}

/* Decodes n_blocks Q4_K blocks into 256 * n_blocks floats. */
void hkvo_q4k_dequant(const uint8_t *blocks, int64_t n_blocks, float *out) {
    for (int64_t b = 0; b < n_blocks; ++b) {
        const uint8_t *blk = blocks + b * Q4K_BYTES;
        const float d = load_f16(blk);
        const float dmin = load_f16(blk + 2);
        const uint8_t *sc = blk + 4;
        const uint8_t *qs = blk + 16;
        float *y = out + b * QK;
        for (int pair = 0; pair < 4; ++pair) {
            int s0, m0, s1, m1;
            unpack_scale_min(sc, 2 * pair, &s0, &m0);
            unpack_scale_min(sc, 2 * pair + 1, &s1, &m1);
            const float d0 = d * (float)s0, mm0 = dmin * (float)m0;
            const float d1 = d * (float)s1, mm1 = dmin * (float)m1;
            const uint8_t *q = qs + 32 * pair;
            for (int l = 0; l < 32; ++l) {
                y[64 * pair + l] = d0 * (float)(q[l] & 0x0F) - mm0;
            }
            for (int l = 0; l < 32; ++l) {
                y[64 * pair + 32 + l] = d1 * (float)(q[l] >> 4) - mm1;
            }
        }
    }
}

static int round_half_even(float v) { return (int)nearbyintf(v); }

/* Quantises k floats (k % 256 == 0) into k / 256 Q8_K blocks. */
void hkvo_q8k_quantize(const float *x, int64_t k, uint8_t *out) {
    for (int64_t b = 0; b < k / QK; ++b) {
        const float *xb = x + b * QK;
        uint8_t *blk = out + b * Q8K_BYTES;
        float amax = 0.0f, max = 0.0f;
        for (int j = 0; j < QK; ++j) {
            const float ax = fabsf(xb[j]);
            if (ax > amax) {
                amax = ax;
                max = xb[j];
            }
        }
        int8_t qs[QK];
        int16_t bsums[16];
        float d = 0.0f;
        if (amax == 0.0f) {
            memset(qs, 0, sizeof(qs));
            memset(bsums, 0, sizeof(bsums));
        } else {
            const float iscale = -127.0f / max;
            for (int j = 0; j < QK; ++j) {
                const int v = round_half_even(iscale * xb[j]);
                qs[j] = (int8_t)(v < 127 ? v : 127);
            }
            for (int g = 0; g < 16; ++g) {
                int s = 0;
                for (int i = 0; i < 16; ++i) {
                    s += qs[16 * g + i];
                }
                bsums[g] = (int16_t)s;
            }
            d = 1.0f / iscale;
        }
        memcpy(blk, &d, 4);
        memcpy(blk + 4, qs, QK);
        memcpy(blk + 4 + QK, bsums, sizeof(bsums));
    }
}

/* Dot product of one Q4_K row with a Q8_K vector, n_blocks blocks each. */
float hkvo_q4k_dot_q8k(const uint8_t *w, const uint8_t *a, int64_t n_blocks) {
    float sums[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    float sumf = 0.0f;
    for (int64_t b = 0; b < n_blocks; ++b) {
        const uint8_t *wb = w + b * Q4K_BYTES;
        const uint8_t *ab = a + b * Q8K_BYTES;
        float d8;
        memcpy(&d8, ab, 4);
        const int8_t *q8 = (const int8_t *)(ab + 4);
        int16_t bsums[16];
        memcpy(bsums, ab + 4 + QK, sizeof(bsums));
        int8_t q4[QK];
        for (int pair = 0; pair < 4; ++pair) {
            const uint8_t *q = wb + 16 + 32 * pair;
            for (int l = 0; l < 32; ++l) {
                q4[64 * pair + l] = (int8_t)(q[l] & 0x0F);
                q4[64 * pair + 32 + l] = (int8_t)(q[l] >> 4);
            }
        }
        int scale[8], mins[8];
        for (int j = 0; j < 8; ++j) {
            unpack_scale_min(wb + 4, j, &scale[j], &mins[j]);
        }
        int summs = 0;
        for (int g = 0; g < 16; ++g) {
            summs += bsums[g] * mins[g / 2];
        }
        int32_t lane[8] = {0, 0, 0, 0, 0, 0, 0, 0};
        for (int j = 0; j < 8; ++j) {  /* sub-block of 32 = 4 groups of 8 */
            for (int g = 0; g < 4; ++g) {
                const int base = 32 * j + 8 * g;
                for (int l = 0; l < 8; ++l) {
                    const int16_t p = (int16_t)(q8[base + l] * q4[base + l]);
                    lane[l] += scale[j] * p;
                }
            }
        }
        const float d = load_f16(wb) * d8;
        for (int l = 0; l < 8; ++l) {
            sums[l] += d * (float)lane[l];
        }
        const float dmin = load_f16(wb + 2) * d8;
        sumf -= dmin * (float)summs;
    }
    for (int l = 0; l < 8; ++l) {
        sumf += sums[l];
    }
    return sumf;
}

/* y[r] = W[r] . x for n_vec activation vectors: x is [n_vec][cols] F32,
 * W is [rows][cols/256] Q4_K blocks, y is [n_vec][rows]. */
void hkvo_q4k_gemv(const uint8_t *w, int64_t rows, int64_t cols, const float *x,
                   int64_t n_vec, float *y, uint8_t *q8_scratch) {
    const int64_t nb = cols / QK;
    for (int64_t e = 0; e < n_vec; ++e) {
        hkvo_q8k_quantize(x + e * cols, cols, q8_scratch + e * nb * Q8K_BYTES);
    }
#pragma omp parallel for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
        for (int64_t e = 0; e < n_vec; ++e) {
            y[e * rows + r] = hkvo_q4k_dot_q8k(w + r * nb * Q4K_BYTES,
                                               q8_scratch + e * nb * Q8K_BYTES, nb);
        }
    }
}

/* ggml rms_norm followed by ggml_mul with a weight row (weight may be NULL):
 * n_rows rows of n floats. */
void hkvo_rms_norm_mul(const float *x, int64_t n_rows, int64_t n, float eps, const float *weight,
                       float *y) {
    for (int64_t r = 0; r < n_rows; ++r) {
        const float *xr = x + r * n;
        float *yr = y + r * n;
        double sum = 0.0;
        for (int64_t i = 0; i < n; ++i) {
            sum += (double)(xr[i] * xr[i]);
        }
        const float mean = (float)(sum / (double)n);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int64_t i = 0; i < n; ++i) {
            const float v = xr[i] * scale;
            yr[i] = weight != NULL ? v * weight[i] : v;
        }
    }
}

/* silu(gate) * up, elementwise. */
void hkvo_silu_mul(const float *gate, const float *up, int64_t n, float *y) {
    for (int64_t i = 0; i < n; ++i) {
        const float g = gate[i];
        y[i] = (g / (1.0f + expf(-g))) * up[i];
    }
}
