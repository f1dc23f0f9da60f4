/*
 * oracle.h — CPU restatement of the reference's quantised-linear arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker for the CUDA path:
 * only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load
 * it.  The product libraries under vkflame_b200/ never link or call it.
 *
 * Every function names the reference shader lines it restates.  The
 * restatement is pinned against the reference shaders themselves: the
 * recipe in oracle/build_ref.py compiles the GLSL main() bodies as C++
 * (oracle/_ref/) and tests/golden/ holds vectors produced by that build.
 */
#ifndef VKFLAME_ORACLE_H
#define VKFLAME_ORACLE_H

#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* fp16 <-> fp32, IEEE round-to-nearest-even (unpackHalf2x16 / float16_t()). */
float oracle_half_to_float(uint16_t h);
uint16_t oracle_float_to_half(float f);

/* Dequantise nb blocks of type qtype (VKF_DEQUANT_*) to fp32.
 * nb counts blocks of the format (32 or 256 values each).
 * Restates kernels/dequant_{q4_0,q4_1,q5_0,q8_0,q8_1,q4_k,q5_k,q6_k}.glsl. */
int oracle_dequant(int qtype, const void *src, float *dst, int64_t nb);

/* fp32 -> Q8_1, n values (n % 32 == 0).  No reference counterpart (the
 * reference only decodes Q8_1, kernels/dequant_q8_1.glsl); convention:
 * amax = max|x|, d = amax/127, q = clamp(round_half_away(x/d)), s = d*sum(q),
 * d and s stored as fp16. */
void oracle_quantize_q8_1(const float *x, void *dst, int64_t n);

/* kernels/linear_int8.glsl:48-101 exactly as written: fp16 A [MxK] is
 * quantised with act_scale inside the loop, W is int8 [NxK], result is
 * fp16(act(float(acc) * w_scale[n])).  act: 0 none, 1 silu, 2 relu, 3 gelu_erf. */
void oracle_linear_int8_shader(const uint16_t *a, const int8_t *w, const float *w_scale,
                               float act_scale, int act, int M, int N, int K,
                               uint16_t *out);

/* The int8 linear the boundary exposes (config: int8 X with per-row scale sx,
 * int8 W [NxK] with per-channel scale sw, optional fp16 bias).
 * acc[m,n] = sum_k X[m,k]*W[n,k] (int32, the linear_int8.glsl:54-90 loop);
 * out = fp16(act(((float)acc * sx[m]) * sw[n] + bias[n])), each op rounded
 * separately in fp32 (no contraction).  acc_out and/or out may be NULL. */
void oracle_linear_int8(const int8_t *x, const int8_t *w, const float *sx, const float *sw,
                        const uint16_t *bias, int act, int M, int N, int K,
                        int32_t *acc_out, uint16_t *out, int nthreads);

/* kernels/linear_fp16.glsl:38-51: fp16 A [MxK] x fp16 B [KxN], fp32
 * accumulation in k order, fp16 output after act. */
void oracle_linear_fp16_shader(const uint16_t *a, const uint16_t *b, int act,
                               int M, int N, int K, uint16_t *out);

/* The reference's quantised mul_mat sequence (shim/hip_runtime_shim.cpp:1129-1166)
 * as intended: dequantise W [N rows x K] to fp32, take fp16 X [MxK] (xtype 0)
 * or Q8_1 X (xtype 1) to fp32, then a k-serial fp32 dot product per output
 * (linear_fp16_fp32out.glsl:45-47 with B read as W^T).  Output fp32 (ytype 0)
 * or fp16 (ytype 1).  OpenMP over output rows with nthreads threads.
 * This is the timed CPU baseline. */
int oracle_quant_linear(int wtype, const void *w, int xtype, const void *x,
                        int ytype, void *y, int M, int N, int K, int nthreads);

/* Activation as the reference shaders define it (linear_fp16.glsl:23-36). */
float oracle_activation(int act, float x);

/* The non-matmul kernels of the hipLaunchKernel name table (fp32 unless
 * stated); each restates the shader it names. */
float oracle_unary(int op, float x);                                       /* elementwise_f32.glsl */
void oracle_elementwise(int op, const float *x, float *y, int64_t n);
void oracle_scale(const float *x, float *y, int64_t n, float scale, float bias);      /* scale_f32.glsl */
void oracle_binop(int op, const float *a, const float *b, float *y, int64_t n, int64_t bn); /* binop_f32.glsl */
void oracle_rms_norm_f32(const float *x, float *y, int M, int N, float eps);         /* rms_norm_f32.glsl */
void oracle_rms_norm_f16(const uint16_t *x, const uint16_t *g, uint16_t *y, int M, int N, float eps); /* rms_norm.glsl */
void oracle_softmax(const float *x, float *y, int M, int N);                         /* softmax_online.glsl */
void oracle_rope_neox(const float *x, const int32_t *pos, float *y, int ne0, int ne1, int n_dims, int n_seqs,
                      float theta_scale, float freq_scale);                          /* rope_neox.glsl */
void oracle_embedding(const void *w, int esize, const int32_t *idx, void *out, int V, int D, int B); /* embedding.glsl */

#ifdef __cplusplus
}
#endif
#endif
