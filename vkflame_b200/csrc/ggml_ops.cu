// ggml_ops.cu — the non-matmul kernels of the hipLaunchKernel name table:
// unary element-wise ops, scale, binary ops, RMS norms, softmax, neox RoPE,
// embedding / get_rows.  fp32 unless stated.
//
// Each restates the reference's compute shader of the same name
// (kernels/elementwise_f32.glsl, scale_f32.glsl, binop_f32.glsl,
// rms_norm_f32.glsl, rms_norm.glsl, softmax_online.glsl, rope_neox.glsl,
// embedding.glsl) as a CUDA kernel: the arithmetic per element is the
// shader's; the work split is this GPU's (grid-stride loops over 148 SMs,
// 16-byte vector accesses where the pointers allow, one CTA per row with
// warp-shuffle reductions for the row ops).  All are HBM-bound.  The
// transcendental functions are CUDA's own (expf, tanhf, logf, sqrtf, sinf,
// cosf, powf, rsqrtf), where the shaders used GLSL's.

#include "rt_internal.h"

#include <cuda_fp16.h>

#include <algorithm>

namespace vkf {
namespace ops {

constexpr int NT = 256;

// GELU's erf as the reference defines it (elementwise_f32.glsl:20-26):
// Abramowitz & Stegun formula 7.1.26 (|error| <= 1.5e-7), a published
// rational approximation with five coefficients.
__device__ __forceinline__ float erf_as(float x) {
    const float t = 1.0f / (1.0f + 0.3275911f * fabsf(x));
    const float p = t * (0.254829592f + t * (-0.284496736f + t * (1.421413741f + t * (-1.453152027f + t * 1.061405429f))));
    const float s = x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);
    return s * (1.0f - p * expf(-x * x));
}

// Op ids of VKF_EW_* (runtime/dispatch.h:24-38, elementwise_f32.glsl:33-50).
__device__ __forceinline__ float unary(float x, unsigned op) {
    switch (op) {
    case 0: return x / (1.0f + expf(-x));                                  // silu
    case 1: return 0.5f * x * (1.0f + erf_as(x * 0.7071067811865476f));    // gelu (erf)
    case 2: return fmaxf(x, 0.0f);                                          // relu
    case 3: return tanhf(x);                                                // tanh
    case 4: return x * (1.0f / (1.0f + expf(-1.702f * x)));                 // gelu_quick
    case 5: return -x;                                                      // neg
    case 6: return 1.0f / (1.0f + expf(-x));                                // sigmoid
    case 7: return x * x;                                                   // sqr
    case 8: return sqrtf(x);                                                // sqrt
    case 9: return expf(x);                                                 // exp
    case 10: return logf(x);                                                // log
    case 11: return fabsf(x);                                               // abs
    case 12: return x > 0.f ? 1.f : (x < 0.f ? -1.f : 0.f);                 // sgn
    case 13: return fminf(fmaxf((x + 3.0f) / 6.0f, 0.f), 1.f);              // hardsigmoid
    case 14: return x * fminf(fmaxf((x + 3.0f) / 6.0f, 0.f), 1.f);          // hardswish
    default: return x;
    }
}

__device__ __forceinline__ float binop(float a, float b, unsigned op) {
    switch (op) {
    case 0: return a + b;
    case 1: return a * b;
    case 2: return a - b;
    case 3: return b != 0.f ? a / b : 0.f;  // binop_f32.glsl:27: division by zero gives 0
    default: return a;
    }
}

// kind 0: unary op; 1: scale * x + bias.  float4 body when 16-byte aligned.
__global__ void __launch_bounds__(NT) map_kernel(const float *__restrict__ src, float *__restrict__ dst, uint64_t n,
                                                 unsigned op, int kind, float scale, float bias, int vec) {
    const uint64_t stride = (uint64_t)gridDim.x * NT;
    uint64_t i = (uint64_t)blockIdx.x * NT + threadIdx.x;
    // scale * x + bias as two roundings, as the shader states it (no fused multiply-add)
    auto f = [&](float x) { return kind == 0 ? unary(x, op) : __fadd_rn(__fmul_rn(scale, x), bias); };
    if (vec) {
        const uint64_t n4 = n / 4;
        for (uint64_t j = i; j < n4; j += stride) {
            float4 v = reinterpret_cast<const float4 *>(src)[j];
            v.x = f(v.x);
            v.y = f(v.y);
            v.z = f(v.z);
            v.w = f(v.w);
            reinterpret_cast<float4 *>(dst)[j] = v;
        }
        for (uint64_t j = n4 * 4 + i; j < n; j += stride) dst[j] = f(src[j]);
        return;
    }
    for (; i < n; i += stride) dst[i] = f(src[i]);
}

__global__ void __launch_bounds__(NT) binop_kernel(const float *__restrict__ a, const float *__restrict__ b,
                                                   float *__restrict__ d, uint64_t n, uint64_t bn, unsigned op) {
    const uint64_t stride = (uint64_t)gridDim.x * NT;
    for (uint64_t i = (uint64_t)blockIdx.x * NT + threadIdx.x; i < n; i += stride)
        d[i] = binop(a[i], b[bn == n ? i : i % bn], op);
}

__device__ __forceinline__ float block_sum(float v, float *red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5;
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float t = 0.f;
    if (threadIdx.x == 0) {
        for (int i = 0; i < NT / 32; ++i) t += red[i];
        red[NT / 32] = t;
    }
    __syncthreads();
    return red[NT / 32];
}

// rms_norm_f32.glsl: y = x * inversesqrt(sum(x^2) / N + eps), one CTA per row.
__global__ void __launch_bounds__(NT) rms_norm_f32_kernel(const float *__restrict__ x, float *__restrict__ y, int N,
                                                          float eps) {
    __shared__ float red[NT / 32 + 1];
    const float *xr = x + (int64_t)blockIdx.x * N;
    float *yr = y + (int64_t)blockIdx.x * N;
    float s = 0.f;
    for (int c = threadIdx.x; c < N; c += NT) s = fmaf(xr[c], xr[c], s);
    const float r = rsqrtf(block_sum(s, red) / (float)N + eps);
    for (int c = threadIdx.x; c < N; c += NT) yr[c] = xr[c] * r;
}

// rms_norm.glsl: fp16 x and gamma, y = fp16(x * rrms * gamma).
__global__ void __launch_bounds__(NT) rms_norm_f16_kernel(const __half *__restrict__ x, const __half *__restrict__ g,
                                                          __half *__restrict__ y, int N, float eps) {
    __shared__ float red[NT / 32 + 1];
    const __half *xr = x + (int64_t)blockIdx.x * N;
    __half *yr = y + (int64_t)blockIdx.x * N;
    float s = 0.f;
    for (int c = threadIdx.x; c < N; c += NT) {
        const float v = __half2float(xr[c]);
        s = fmaf(v, v, s);
    }
    const float r = rsqrtf(block_sum(s, red) / (float)N + eps);
    for (int c = threadIdx.x; c < N; c += NT) yr[c] = __float2half_rn(__half2float(xr[c]) * r * __half2float(g[c]));
}

// softmax_online.glsl: per row, running (max, denominator) pairs merged
// across threads; y = exp(x - max) / d.
__device__ __forceinline__ void merge(float &m, float &d, float mb, float db) {
    const float mn = fmaxf(m, mb);
    d = d * expf(m - mn) + db * expf(mb - mn);
    m = mn;
}

__global__ void __launch_bounds__(NT) softmax_kernel(const float *__restrict__ x, float *__restrict__ y, int N) {
    __shared__ float sm[NT / 32], sd[NT / 32], fin[2];
    const float *xr = x + (int64_t)blockIdx.x * N;
    float *yr = y + (int64_t)blockIdx.x * N;
    float m = -1e38f, d = 0.f;
    for (int c = threadIdx.x; c < N; c += NT) {
        const float v = xr[c];
        const float mn = fmaxf(m, v);
        d = d * expf(m - mn) + expf(v - mn);
        m = mn;
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) merge(m, d, __shfl_xor_sync(0xffffffffu, m, o), __shfl_xor_sync(0xffffffffu, d, o));
    if ((threadIdx.x & 31) == 0) {
        sm[threadIdx.x >> 5] = m;
        sd[threadIdx.x >> 5] = d;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float gm = sm[0], gd = sd[0];
        for (int w = 1; w < NT / 32; ++w) merge(gm, gd, sm[w], sd[w]);
        fin[0] = gm;
        fin[1] = gd;
    }
    __syncthreads();
    const float gm = fin[0], gd = fin[1];
    for (int c = threadIdx.x; c < N; c += NT) yr[c] = expf(xr[c] - gm) / gd;
}

// rope_neox.glsl: element j pairs with j + ne0/2 of the same row; rows are
// [seq][head]; theta = pos[seq] * theta_scale^j * freq_scale for 2j < n_dims,
// pass-through beyond.  One thread per (row, pair).
__global__ void __launch_bounds__(NT) rope_neox_kernel(const float *__restrict__ src, const int *__restrict__ pos,
                                                       float *__restrict__ dst, int ne0, int ne1, int n_dims,
                                                       int rows, float theta_scale, float freq_scale) {
    const int half = ne0 / 2;
    const int64_t total = (int64_t)rows * half;
    for (int64_t e = (int64_t)blockIdx.x * NT + threadIdx.x; e < total; e += (int64_t)gridDim.x * NT) {
        const int row = (int)(e / half), j = (int)(e - (int64_t)row * half);
        const int64_t b = (int64_t)row * ne0;
        const float x0 = src[b + j], x1 = src[b + j + half];
        if (2 * j >= n_dims) {
            dst[b + j] = x0;
            dst[b + j + half] = x1;
            continue;
        }
        const float theta = (float)pos[row / ne1] * powf(theta_scale, (float)j) * freq_scale;
        const float c = cosf(theta), s = sinf(theta);
        dst[b + j] = x0 * c - x1 * s;
        dst[b + j + half] = x0 * s + x1 * c;
    }
}

// embedding.glsl: out[b][:] = weight[idx[b]][:], zeros for an index outside
// [0, V).  T_in -> T_out: fp16 -> fp16 (the shader), fp32 -> fp32 and
// fp16 -> fp32 (ggml get_rows into an fp32 destination).
template <typename TI, typename TO>
__global__ void __launch_bounds__(NT) rows_kernel(const TI *__restrict__ w, const int *__restrict__ idx,
                                                  TO *__restrict__ out, int V, int D, int B) {
    const int64_t total = (int64_t)B * D;
    for (int64_t e = (int64_t)blockIdx.x * NT + threadIdx.x; e < total; e += (int64_t)gridDim.x * NT) {
        const int b = (int)(e / D), c = (int)(e - (int64_t)b * D);
        const int r = idx[b];
        float v = 0.f;
        if (r >= 0 && r < V) {
            if constexpr (sizeof(TI) == 2) v = __half2float(w[(int64_t)r * D + c]);
            else v = w[(int64_t)r * D + c];
        }
        if constexpr (sizeof(TO) == 2) out[e] = __float2half_rn(v);
        else out[e] = v;
    }
}

static int grid_for(uint64_t work) {
    static int sms = 0;
    if (!sms) {
        DeviceState *ds = device_state();
        sms = ds ? ds->sm_count : 148;
    }
    return (int)std::max<uint64_t>(1, std::min<uint64_t>((work + NT - 1) / NT, (uint64_t)sms * 8));
}

static thread_local cudaStream_t t_stream = nullptr;

}  // namespace ops

cudaStream_t ops_stream() { return ops::t_stream; }

int ops_unary(const float *src, float *dst, uint64_t n, unsigned op, cudaStream_t st) {
    if (n == 0) return VKF_OK;
    if (!src || !dst || op > 14) return VKF_ERR_INVALID;
    const int vec = (((uintptr_t)src | (uintptr_t)dst) & 15) == 0;
    ops::map_kernel<<<ops::grid_for(vec ? n / 4 : n), ops::NT, 0, st>>>(src, dst, n, op, 0, 0.f, 0.f, vec);
    return check_launch();
}

int ops_scale(const float *src, float *dst, uint64_t n, float scale, float bias, cudaStream_t st) {
    if (n == 0) return VKF_OK;
    if (!src || !dst) return VKF_ERR_INVALID;
    const int vec = (((uintptr_t)src | (uintptr_t)dst) & 15) == 0;
    ops::map_kernel<<<ops::grid_for(vec ? n / 4 : n), ops::NT, 0, st>>>(src, dst, n, 0, 1, scale, bias, vec);
    return check_launch();
}

int ops_binop(const float *a, const float *b, float *d, uint64_t n, uint64_t bn, unsigned op, cudaStream_t st) {
    if (n == 0) return VKF_OK;
    if (!a || !b || !d || bn == 0 || op > 3) return VKF_ERR_INVALID;
    ops::binop_kernel<<<ops::grid_for(n), ops::NT, 0, st>>>(a, b, d, n, bn, op);
    return check_launch();
}

int ops_rms_norm_f32(const float *x, float *y, int M, int N, float eps, cudaStream_t st) {
    if (M <= 0 || N <= 0) return M == 0 ? VKF_OK : VKF_ERR_INVALID;
    if (!x || !y) return VKF_ERR_INVALID;
    ops::rms_norm_f32_kernel<<<M, ops::NT, 0, st>>>(x, y, N, eps);
    return check_launch();
}

int ops_rms_norm_f16(const void *x, const void *g, void *y, int M, int N, float eps, cudaStream_t st) {
    if (M <= 0 || N <= 0) return M == 0 ? VKF_OK : VKF_ERR_INVALID;
    if (!x || !g || !y) return VKF_ERR_INVALID;
    ops::rms_norm_f16_kernel<<<M, ops::NT, 0, st>>>((const __half *)x, (const __half *)g, (__half *)y, N, eps);
    return check_launch();
}

int ops_softmax(const float *x, float *y, int M, int N, cudaStream_t st) {
    if (M <= 0 || N <= 0) return M == 0 ? VKF_OK : VKF_ERR_INVALID;
    if (!x || !y) return VKF_ERR_INVALID;
    ops::softmax_kernel<<<M, ops::NT, 0, st>>>(x, y, N);
    return check_launch();
}

int ops_rope_neox(const float *src, const int *pos, float *dst, int ne0, int ne1, int n_dims, int n_seqs,
                  float theta_scale, float freq_scale, cudaStream_t st) {
    if (ne0 <= 0 || ne1 <= 0 || n_seqs <= 0 || ne0 % 2 || n_dims < 0) return VKF_ERR_INVALID;
    if (!src || !pos || !dst) return VKF_ERR_INVALID;
    const int rows = ne1 * n_seqs;
    ops::rope_neox_kernel<<<ops::grid_for((uint64_t)rows * (ne0 / 2)), ops::NT, 0, st>>>(
        src, pos, dst, ne0, ne1, n_dims, rows, theta_scale, freq_scale);
    return check_launch();
}

// wt/ot: 0 fp16, 1 fp32.
int ops_rows(const void *w, int wt, const int *idx, void *out, int ot, int V, int D, int B, cudaStream_t st) {
    if (B == 0 || D == 0) return VKF_OK;
    if (!w || !idx || !out || V < 0 || D < 0 || B < 0) return VKF_ERR_INVALID;
    const int g = ops::grid_for((uint64_t)B * D);
    if (wt == 0 && ot == 0) ops::rows_kernel<__half, __half><<<g, ops::NT, 0, st>>>((const __half *)w, idx, (__half *)out, V, D, B);
    else if (wt == 1 && ot == 1) ops::rows_kernel<float, float><<<g, ops::NT, 0, st>>>((const float *)w, idx, (float *)out, V, D, B);
    else if (wt == 0 && ot == 1) ops::rows_kernel<__half, float><<<g, ops::NT, 0, st>>>((const __half *)w, idx, (float *)out, V, D, B);
    else return VKF_ERR_UNSUPPORTED;
    return check_launch();
}

}  // namespace vkf

using namespace vkf;

// ---- C ABI: the reference's dispatch entry points (runtime/dispatch.h:60-125) ----
// They carry no stream argument; they launch on the calling thread's stream
// set by vkflame_set_stream (default: the legacy default stream).

extern "C" int vkflame_set_stream(void *stream) {
    ops::t_stream = (cudaStream_t)stream;
    return set_status(VKF_OK);
}

extern "C" void *vkflame_get_stream(void) { return (void *)ops::t_stream; }

extern "C" int vkflame_dispatch_elementwise_f32(void *ctx, const void *src, void *dst, uint32_t n, uint32_t op) {
    (void)ctx;
    return set_status(ops_unary((const float *)src, (float *)dst, n, op, ops::t_stream));
}

extern "C" int vkflame_dispatch_scale_f32(void *ctx, const void *src, void *dst, uint32_t n, float scale, float bias) {
    (void)ctx;
    return set_status(ops_scale((const float *)src, (float *)dst, n, scale, bias, ops::t_stream));
}

extern "C" int vkflame_dispatch_binop_f32(void *ctx, const void *src0, const void *src1, void *dst, uint32_t n,
                                          uint32_t src1_n, uint32_t op) {
    (void)ctx;
    return set_status(ops_binop((const float *)src0, (const float *)src1, (float *)dst, n, src1_n, op, ops::t_stream));
}

extern "C" int vkflame_dispatch_rms_norm_f32(void *ctx, const void *src, void *dst, uint32_t M, uint32_t N, float eps) {
    (void)ctx;
    return set_status(ops_rms_norm_f32((const float *)src, (float *)dst, (int)M, (int)N, eps, ops::t_stream));
}

extern "C" int vkflame_dispatch_rms_norm(void *ctx, const void *X, const void *gamma, void *Y, int M, int N, float eps) {
    (void)ctx;
    return set_status(ops_rms_norm_f16(X, gamma, Y, M, N, eps, ops::t_stream));
}

extern "C" int vkflame_dispatch_softmax(void *ctx, const void *X, void *Y, int M, int N) {
    (void)ctx;
    return set_status(ops_softmax((const float *)X, (float *)Y, M, N, ops::t_stream));
}

extern "C" int vkflame_dispatch_rope_neox(void *ctx, const void *src, const void *pos, void *dst, uint32_t ne0,
                                          uint32_t ne1, uint32_t n_dims, uint32_t n_seqs, float theta_scale,
                                          float freq_scale, uint32_t p0, uint32_t p1) {
    (void)ctx;
    (void)p0;
    (void)p1;
    return set_status(ops_rope_neox((const float *)src, (const int *)pos, (float *)dst, (int)ne0, (int)ne1, (int)n_dims,
                                    (int)n_seqs, theta_scale, freq_scale, ops::t_stream));
}

extern "C" int vkflame_dispatch_embedding(void *ctx, const void *weight, const void *indices, void *out, int V, int D,
                                          int B) {
    (void)ctx;
    return set_status(ops_rows(weight, 0, (const int *)indices, out, 0, V, D, B, ops::t_stream));
}

/* get_rows into an fp32 destination (ggml get_rows_f32 / get_rows_f16). */
extern "C" int vkflame_get_rows(const void *weight, int weight_f32, const void *indices, float *out, int V, int D,
                                int B, void *stream) {
    return set_status(ops_rows(weight, weight_f32 ? 1 : 0, (const int *)indices, out, 1, V, D, B, (cudaStream_t)stream));
}
