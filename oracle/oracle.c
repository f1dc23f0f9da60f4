/*
 * oracle.c — CPU restatement of the reference's quantised-linear arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (see oracle.h).  Compiled with -ffp-contract=off
 * so every fp32 operation rounds exactly where the restated shader rounds.
 * Each function cites the reference shader lines it follows; the dequant
 * formulas are the shaders' own, and every dequantised value is exactly
 * representable in fp32, so evaluation order cannot change a result.
 */
#include "oracle.h"
#include "../include/ggml_blocks.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

float oracle_half_to_float(uint16_t h) {
    _Float16 v;
    memcpy(&v, &h, 2);
    return (float)v;
}

uint16_t oracle_float_to_half(float f) {
    _Float16 v = (_Float16)f;
    uint16_t h;
    memcpy(&h, &v, 2);
    return h;
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static inline float rdh(const uint8_t *p) { return oracle_half_to_float(rd16(p)); }

/* kernels/dequant_q4_0.glsl:24-36 : y[j] = d*(q&15) + (-8d), y[j+16] = d*(q>>4) + (-8d) */
static void dq_q4_0(const uint8_t *src, float *dst, int64_t nb) {
    for (int64_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = src + ib * 18;
        float d = rdh(b);
        float dm = -8.0f * d;
        for (int j = 0; j < 16; ++j) {
            unsigned q = b[2 + j];
            dst[ib * 32 + j] = d * (float)(q & 0xFu) + dm;
            dst[ib * 32 + j + 16] = d * (float)(q >> 4) + dm;
        }
    }
}

/* kernels/dequant_q4_1.glsl:24-36 : y = d*q + m */
static void dq_q4_1(const uint8_t *src, float *dst, int64_t nb) {
    for (int64_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = src + ib * 20;
        float d = rdh(b), m = rdh(b + 2);
        for (int j = 0; j < 16; ++j) {
            unsigned q = b[4 + j];
            dst[ib * 32 + j] = d * (float)(q & 0xFu) + m;
            dst[ib * 32 + j + 16] = d * (float)(q >> 4) + m;
        }
    }
}

/* kernels/dequant_q5_0.glsl:26-46 : 5th bit from the 32-bit qh word */
static void dq_q5_0(const uint8_t *src, float *dst, int64_t nb) {
    for (int64_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = src + ib * 22;
        float d = rdh(b);
        float dm = -16.0f * d;
        uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
        for (int j = 0; j < 16; ++j) {
            unsigned q = b[6 + j];
            unsigned xh0 = ((qh >> (j + 0)) << 4) & 0x10u;
            unsigned xh1 = ((qh >> (j + 12))) & 0x10u;
            float x0 = (float)((q & 0xFu) | xh0);
            float x1 = (float)((q >> 4) | xh1);
            dst[ib * 32 + j] = x0 * d + dm;
            dst[ib * 32 + j + 16] = x1 * d + dm;
        }
    }
}

/* kernels/dequant_q8_0.glsl:23-27 : y = d*q */
static void dq_q8_0(const uint8_t *src, float *dst, int64_t nb) {
    for (int64_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = src + ib * 34;
        float d = rdh(b);
        for (int j = 0; j < 32; ++j) dst[ib * 32 + j] = d * (float)(int8_t)b[2 + j];
    }
}

/* kernels/dequant_q8_1.glsl:26-31 : y = d*q, the s field is not read */
static void dq_q8_1(const uint8_t *src, float *dst, int64_t nb) {
    for (int64_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = src + ib * 36;
        float d = rdh(b);
        for (int j = 0; j < 32; ++j) dst[ib * 32 + j] = d * (float)(int8_t)b[4 + j];
    }
}

/* kernels/dequant_q4_k.glsl:16-24 (get_scale_min_k4), shared by Q4_K and Q5_K */
static void scale_min_k4(int j, const uint8_t *s, float *sc, float *mn) {
    if (j < 4) {
        *sc = (float)(s[j] & 63u);
        *mn = (float)(s[j + 4] & 63u);
    } else {
        *sc = (float)((s[j + 4] & 0xFu) | ((s[j - 4] >> 6) << 4));
        *mn = (float)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

/* kernels/dequant_q4_k.glsl:34-57 : y = (d*sc)*q - dmin*m per 32-value sub-block */
static void dq_q4_k(const uint8_t *src, float *dst, int64_t nb) {
    for (int64_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = src + ib * 144;
        float dall = rdh(b), dmin = rdh(b + 2);
        const uint8_t *sc = b + 4, *qs = b + 16;
        for (int il = 0; il < 4; ++il) {
            float sc0, m0, sc1, m1;
            scale_min_k4(2 * il, sc, &sc0, &m0);
            scale_min_k4(2 * il + 1, sc, &sc1, &m1);
            float d0 = dall * sc0, min0 = dmin * m0;
            float d1 = dall * sc1, min1 = dmin * m1;
            for (int l = 0; l < 32; ++l) {
                unsigned q = qs[32 * il + l];
                dst[ib * 256 + 64 * il + l] = d0 * (float)(q & 0xFu) - min0;
                dst[ib * 256 + 64 * il + l + 32] = d1 * (float)(q >> 4) - min1;
            }
        }
    }
}

/* kernels/dequant_q5_k.glsl:37-74 : Q4_K plus a 5th bit from qh[l] bit (2il / 2il+1) */
static void dq_q5_k(const uint8_t *src, float *dst, int64_t nb) {
    for (int64_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = src + ib * 176;
        float dall = rdh(b), dmin = rdh(b + 2);
        const uint8_t *sc = b + 4, *qh = b + 16, *qs = b + 48;
        for (int il = 0; il < 4; ++il) {
            float sc0, m0, sc1, m1;
            scale_min_k4(2 * il, sc, &sc0, &m0);
            scale_min_k4(2 * il + 1, sc, &sc1, &m1);
            float d0 = dall * sc0, min0 = dmin * m0;
            float d1 = dall * sc1, min1 = dmin * m1;
            unsigned hm0 = 1u << (2 * il), hm1 = hm0 << 1;
            for (int l = 0; l < 32; ++l) {
                unsigned q = qs[32 * il + l], h = qh[l];
                dst[ib * 256 + 64 * il + l] = d0 * (float)((q & 0xFu) + ((h & hm0) ? 16u : 0u)) - min0;
                dst[ib * 256 + 64 * il + l + 32] = d1 * (float)((q >> 4) + ((h & hm1) ? 16u : 0u)) - min1;
            }
        }
    }
}

/* kernels/dequant_q6_k.glsl:28-58 : y = d * float(sc * (q6 - 32)) */
static void dq_q6_k(const uint8_t *src, float *dst, int64_t nb) {
    for (int64_t ib = 0; ib < nb; ++ib) {
        const uint8_t *b = src + ib * 210;
        const uint8_t *ql = b, *qh = b + 128;
        const int8_t *scales = (const int8_t *)(b + 192);
        float d = rdh(b + 208);
        for (int ip = 0; ip < 2; ++ip) {
            for (int il = 0; il < 32; ++il) {
                int is = 8 * ip + il / 16;
                unsigned qhb = qh[32 * ip + il];
                unsigned ql0 = ql[64 * ip + il], ql32 = ql[64 * ip + il + 32];
                int v0 = (int)((ql0 & 0xFu) | (((qhb >> 0) & 3u) << 4)) - 32;
                int v32 = (int)((ql32 & 0xFu) | (((qhb >> 2) & 3u) << 4)) - 32;
                int v64 = (int)((ql0 >> 4) | (((qhb >> 4) & 3u) << 4)) - 32;
                int v96 = (int)((ql32 >> 4) | (((qhb >> 6) & 3u) << 4)) - 32;
                float *o = dst + ib * 256 + 128 * ip + il;
                o[0] = d * (float)(scales[is + 0] * v0);
                o[32] = d * (float)(scales[is + 2] * v32);
                o[64] = d * (float)(scales[is + 4] * v64);
                o[96] = d * (float)(scales[is + 6] * v96);
            }
        }
    }
}

int oracle_dequant(int qtype, const void *src, float *dst, int64_t nb) {
    const uint8_t *s = (const uint8_t *)src;
    switch (qtype) {
    case VKF_DEQUANT_Q4_0: dq_q4_0(s, dst, nb); return 0;
    case VKF_DEQUANT_Q4_1: dq_q4_1(s, dst, nb); return 0;
    case VKF_DEQUANT_Q5_0: dq_q5_0(s, dst, nb); return 0;
    case VKF_DEQUANT_Q8_0: dq_q8_0(s, dst, nb); return 0;
    case VKF_DEQUANT_Q8_1: dq_q8_1(s, dst, nb); return 0;
    case VKF_DEQUANT_Q4_K: dq_q4_k(s, dst, nb); return 0;
    case VKF_DEQUANT_Q5_K: dq_q5_k(s, dst, nb); return 0;
    case VKF_DEQUANT_Q6_K: dq_q6_k(s, dst, nb); return 0;
    default: return -1;
    }
}

void oracle_quantize_q8_1(const float *x, void *dst, int64_t n) {
    uint8_t *out = (uint8_t *)dst;
    for (int64_t ib = 0; ib < n / 32; ++ib) {
        const float *xb = x + ib * 32;
        uint8_t *b = out + ib * 36;
        float amax = 0.0f;
        for (int j = 0; j < 32; ++j) {
            float a = fabsf(xb[j]);
            amax = a > amax ? a : amax;
        }
        float d = amax / 127.0f;
        int sum = 0;
        for (int j = 0; j < 32; ++j) {
            int q = 0;
            if (d != 0.0f) {
                q = (int)roundf(xb[j] / d);
                q = q < -127 ? -127 : (q > 127 ? 127 : q);
            }
            b[4 + j] = (uint8_t)(int8_t)q;
            sum += q;
        }
        uint16_t hd = oracle_float_to_half(d);
        uint16_t hs = oracle_float_to_half(d * (float)sum);
        b[0] = (uint8_t)(hd & 0xFF); b[1] = (uint8_t)(hd >> 8);
        b[2] = (uint8_t)(hs & 0xFF); b[3] = (uint8_t)(hs >> 8);
    }
}

/* kernels/linear_int8.glsl:33-46 (Abramowitz & Stegun 7.1.26 erf) and
 * linear_fp16.glsl:23-36 (silu / relu / gelu_erf). */
static float erf_as(float x) {
    float t = 1.0f / (1.0f + 0.3275911f * fabsf(x));
    float y = 1.0f - ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t * expf(-x * x);
    return x >= 0.0f ? y : -y;
}

float oracle_activation(int act, float x) {
    switch (act) {
    case 1: return x * (1.0f / (1.0f + expf(-x)));
    case 2: return x > 0.0f ? x : 0.0f;
    case 3: return 0.5f * x * (1.0f + erf_as(x * 0.70710678118654f));
    default: return x;
    }
}

/* kernels/linear_int8.glsl:31-46: the int8 shader nests its erf polynomial
 * differently from linear_fp16.glsl and takes sign(x) * val. */
static float gelu_int8_shader(float x) {
    float z = x * 0.70710678f;
    float t = 1.0f / (1.0f + 0.3275911f * fabsf(z));
    float poly = t * (0.254829592f + t * (-0.284496736f + t * (1.421413741f + t * (-1.453152027f + t * 1.061405429f))));
    float val = 1.0f - poly * expf(-z * z);
    float sg = z > 0.0f ? 1.0f : (z < 0.0f ? -1.0f : 0.0f);
    return 0.5f * x * (1.0f + sg * val);
}

void oracle_linear_int8_shader(const uint16_t *a, const int8_t *w, const float *w_scale,
                               float act_scale, int act, int M, int N, int K, uint16_t *out) {
    for (int m = 0; m < M; ++m)
        for (int n = 0; n < N; ++n) {
            int acc = 0;
            for (int k = 0; k < K; ++k) {
                float xf = oracle_half_to_float(a[(size_t)m * K + k]);
                int q = (int)roundf(xf / act_scale);
                q = q < -127 ? -127 : (q > 127 ? 127 : q);
                acc += q * (int)w[(size_t)n * K + k];
            }
            float r = (float)acc * w_scale[n];
            r = act == 3 ? gelu_int8_shader(r) : oracle_activation(act, r);
            out[(size_t)m * N + n] = oracle_float_to_half(r);
        }
}

void oracle_linear_int8(const int8_t *x, const int8_t *w, const float *sx, const float *sw,
                        const uint16_t *bias, int act, int M, int N, int K,
                        int32_t *acc_out, uint16_t *out, int nthreads) {
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int m = 0; m < M; ++m) {
        const int8_t *xr = x + (size_t)m * K;
        for (int n = 0; n < N; ++n) {
            const int8_t *wr = w + (size_t)n * K;
            int32_t acc = 0;
            for (int k = 0; k < K; ++k) acc += (int32_t)xr[k] * (int32_t)wr[k];
            if (acc_out) acc_out[(size_t)m * N + n] = acc;
            if (out) {
                float v = (float)acc * sx[m];
                v = v * sw[n];
                if (bias) v = v + oracle_half_to_float(bias[n]);
                v = oracle_activation(act, v);
                out[(size_t)m * N + n] = oracle_float_to_half(v);
            }
        }
    }
}

void oracle_linear_fp16_shader(const uint16_t *a, const uint16_t *b, int act,
                               int M, int N, int K, uint16_t *out) {
    for (int row = 0; row < M; ++row)
        for (int col = 0; col < N; ++col) {
            float acc = 0.0f;
            for (int k = 0; k < K; ++k)
                acc += oracle_half_to_float(a[(size_t)row * K + k]) * oracle_half_to_float(b[(size_t)k * N + col]);
            out[(size_t)row * N + col] = oracle_float_to_half(oracle_activation(act, acc));
        }
}

int oracle_quant_linear(int wtype, const void *w, int xtype, const void *x,
                        int ytype, void *y, int M, int N, int K, int nthreads) {
    int qk = vkf_qtype_block_values(wtype);
    if (K % qk != 0 || K % 32 != 0) return -1;
    int64_t nb_row = K / qk;
    size_t row_bytes = (size_t)nb_row * vkf_qtype_block_bytes(wtype);
    float *wf = (float *)malloc((size_t)N * K * sizeof(float));
    float *xf = (float *)malloc((size_t)M * K * sizeof(float));
    if (!wf || !xf) { free(wf); free(xf); return -2; }
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#endif
    /* Step 1 (hip_runtime_shim.cpp:1130-1151): dequantise W to an fp32 buffer. */
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int n = 0; n < N; ++n)
        oracle_dequant(wtype, (const uint8_t *)w + (size_t)n * row_bytes, wf + (size_t)n * K, nb_row);
    /* Step 1b (:1155-1158): activations to fp32 (Q8_1 decode, or fp16 widen). */
    if (xtype == 1) {
        for (int m = 0; m < M; ++m)
            oracle_dequant(VKF_DEQUANT_Q8_1, (const uint8_t *)x + (size_t)m * (K / 32) * 36, xf + (size_t)m * K, K / 32);
    } else {
        const uint16_t *xh = (const uint16_t *)x;
        for (size_t i = 0; i < (size_t)M * K; ++i) xf[i] = oracle_half_to_float(xh[i]);
    }
    /* Step 2 (:1161-1166, linear_fp16_fp32out.glsl:45-47): k-serial fp32 dot products. */
#ifdef _OPENMP
#pragma omp parallel for schedule(static) num_threads(nthreads)
#endif
    for (int n = 0; n < N; ++n) {
        const float *wr = wf + (size_t)n * K;
        for (int m = 0; m < M; ++m) {
            const float *xr = xf + (size_t)m * K;
            float acc = 0.0f;
            for (int k = 0; k < K; ++k) acc += xr[k] * wr[k];
            if (ytype == 0) ((float *)y)[(size_t)m * N + n] = acc;
            else ((uint16_t *)y)[(size_t)m * N + n] = oracle_float_to_half(acc);
        }
    }
    free(wf);
    free(xf);
    return 0;
}

/* ---- the non-matmul kernels of the hipLaunchKernel table ---------------- */

/* kernels/elementwise_f32.glsl:20-26: erf by A&S 7.1.26 with sign(x). */
static float erf_ew(float x) {
    float t = 1.0f / (1.0f + 0.3275911f * fabsf(x));
    float p = t * (0.254829592f + t * (-0.284496736f + t * (1.421413741f + t * (-1.453152027f + t * 1.061405429f))));
    float s = x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
    return s * (1.0f - p * expf(-x * x));
}

static float clampf01(float v) { return v < 0.0f ? 0.0f : (v > 1.0f ? 1.0f : v); }

/* kernels/elementwise_f32.glsl:33-50 (op ids 0..14). */
float oracle_unary(int op, float x) {
    switch (op) {
    case 0: return x / (1.0f + expf(-x));
    case 1: return 0.5f * x * (1.0f + erf_ew(x * 0.7071067811865476f));
    case 2: return x < 0.0f ? 0.0f : x;  /* max(x, 0.0): -0 stays -0 */
    case 3: return tanhf(x);
    case 4: return x * (1.0f / (1.0f + expf(-1.702f * x)));
    case 5: return -x;
    case 6: return 1.0f / (1.0f + expf(-x));
    case 7: return x * x;
    case 8: return sqrtf(x);
    case 9: return expf(x);
    case 10: return logf(x);
    case 11: return fabsf(x);
    case 12: return x > 0.0f ? 1.0f : (x < 0.0f ? -1.0f : 0.0f);
    case 13: return clampf01((x + 3.0f) / 6.0f);
    case 14: return x * clampf01((x + 3.0f) / 6.0f);
    default: return x;
    }
}

void oracle_elementwise(int op, const float *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; ++i) y[i] = oracle_unary(op, x[i]);
}

/* kernels/scale_f32.glsl:17-19 */
void oracle_scale(const float *x, float *y, int64_t n, float scale, float bias) {
    for (int64_t i = 0; i < n; ++i) y[i] = scale * x[i] + bias;
}

/* kernels/binop_f32.glsl:19-31 (src1 broadcast as i % src1_n; x / 0 = 0) */
void oracle_binop(int op, const float *a, const float *b, float *y, int64_t n, int64_t bn) {
    for (int64_t i = 0; i < n; ++i) {
        float u = a[i], v = b[i % bn];
        y[i] = op == 0 ? u + v : op == 1 ? u * v : op == 2 ? u - v : op == 3 ? (v != 0.0f ? u / v : 0.0f) : u;
    }
}

/* kernels/rms_norm_f32.glsl:23-57: y = x * inversesqrt(sum(x^2)/N + eps).
 * The shader sums per thread, then per subgroup, then across subgroups;
 * this sums in double, so agreement is to fp32 rounding, not bit for bit. */
void oracle_rms_norm_f32(const float *x, float *y, int M, int N, float eps) {
    for (int m = 0; m < M; ++m) {
        double s = 0.0;
        for (int c = 0; c < N; ++c) s += (double)x[(int64_t)m * N + c] * x[(int64_t)m * N + c];
        float r = (float)(1.0 / sqrt(s / N + (double)eps));
        for (int c = 0; c < N; ++c) y[(int64_t)m * N + c] = x[(int64_t)m * N + c] * r;
    }
}

/* kernels/rms_norm.glsl: fp16 x and gamma, y = fp16(x * rrms * gamma). */
void oracle_rms_norm_f16(const uint16_t *x, const uint16_t *g, uint16_t *y, int M, int N, float eps) {
    for (int m = 0; m < M; ++m) {
        double s = 0.0;
        for (int c = 0; c < N; ++c) {
            double v = oracle_half_to_float(x[(int64_t)m * N + c]);
            s += v * v;
        }
        float r = (float)(1.0 / sqrt(s / N + (double)eps));
        for (int c = 0; c < N; ++c)
            y[(int64_t)m * N + c] = oracle_float_to_half(oracle_half_to_float(x[(int64_t)m * N + c]) * r *
                                                         oracle_half_to_float(g[c]));
    }
}

/* kernels/softmax_online.glsl: y = exp(x - max) / sum(exp(x - max)) per row
 * (the shader's online (max, d) merge equals this up to rounding). */
void oracle_softmax(const float *x, float *y, int M, int N) {
    for (int m = 0; m < M; ++m) {
        const float *r = x + (int64_t)m * N;
        float mx = -1e38f;
        for (int c = 0; c < N; ++c) mx = r[c] > mx ? r[c] : mx;
        double d = 0.0;
        for (int c = 0; c < N; ++c) d += exp((double)r[c] - mx);
        for (int c = 0; c < N; ++c) y[(int64_t)m * N + c] = (float)(exp((double)r[c] - mx) / d);
    }
}

/* kernels/rope_neox.glsl:28-61 over every row and pair (rows [seq][head]). */
void oracle_rope_neox(const float *x, const int32_t *pos, float *y, int ne0, int ne1, int n_dims, int n_seqs,
                      float theta_scale, float freq_scale) {
    int half = ne0 / 2;
    for (int row = 0; row < ne1 * n_seqs; ++row)
        for (int j = 0; j < half; ++j) {
            int64_t b = (int64_t)row * ne0;
            float x0 = x[b + j], x1 = x[b + j + half];
            if (2 * j >= n_dims) {
                y[b + j] = x0;
                y[b + j + half] = x1;
                continue;
            }
            float theta = (float)pos[row / ne1] * powf(theta_scale, (float)j) * freq_scale;
            float c = cosf(theta), s = sinf(theta);
            y[b + j] = x0 * c - x1 * s;
            y[b + j + half] = x0 * s + x1 * c;
        }
}

/* kernels/embedding.glsl:16-31: out[b] = weight[idx[b]], zeros out of range
 * (esize 2: fp16 table and output; 4: fp32). */
void oracle_embedding(const void *w, int esize, const int32_t *idx, void *out, int V, int D, int B) {
    for (int b = 0; b < B; ++b) {
        int r = idx[b];
        for (int c = 0; c < D; ++c) {
            uint8_t *o = (uint8_t *)out + ((int64_t)b * D + c) * esize;
            if (r < 0 || r >= V) memset(o, 0, esize);
            else memcpy(o, (const uint8_t *)w + ((int64_t)r * D + c) * esize, esize);
        }
    }
}
