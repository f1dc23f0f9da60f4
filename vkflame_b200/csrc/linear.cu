// linear.cu — kernel selection for the quantised linear entry points.
//
// Replaces the reference's quantised mul_mat chain (shim/hip_runtime_shim.cpp:
// 1129-1166: dequant W -> fp32 temp, dequant X -> fp32 temp, naive GEMM,
// two allocations and three synchronous submits per call) with one fused
// kernel launch on the caller's stream.

#include "rt_internal.h"

#include <cuda_fp16.h>

#include <cstdlib>

namespace vkf {
int gemv_launch(int wtype, const void *W, const void *X, int64_t ldx_bytes, void *Y, int y_f16, int64_t ldy, int M,
                int N, int K, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap, int prefetch,
                const vkf_gather_t *g = nullptr);
size_t gemv_ws_floats(int sms);
size_t gemv_counters(int N);
int gemv_cols_per_launch(int K);
int q8_1_to_f16(const void *src, void *dst, int M, int K, int64_t ldb, int64_t ldo, cudaStream_t stream);
int dequant_launch(const void *src, void *dst, uint64_t nb, int qtype, cudaStream_t stream, bool f16out);
int gemm_i8_tn(const int8_t *A, int64_t lda, const int8_t *B, int64_t ldb, int M, int N, int K, const float *sx,
               const float *sw, const void *bias, void *Y, int64_t ldy, int32_t *acc_out, int64_t ldacc, int act,
               cudaStream_t stream, int y_f16 = 1);
int gemm_tf32_tn(const float *A, int64_t lda, const float *B, int64_t ldb, int M, int N, int K, float alpha,
                 float beta, const void *C, int64_t ldc, int c_f16, const void *bias, int act, void *Y, int64_t ldy,
                 int y_f16, cudaStream_t stream);
int gemm_f16_tn(const void *A, int64_t lda, const void *B, int64_t ldb, int M, int N, int K, float alpha, float beta,
                const void *C, int64_t ldc, int c_f16, const void *bias, int act, void *Y, int64_t ldy, int y_f16,
                cudaStream_t stream);
bool qgemm_supported(int wtype, const void *W, int K);
size_t qgemm_ws_bytes(int wtype, int M, int N, int K);
int qgemm_launch(int wtype, const void *W, const void *X, int64_t ldx, void *Y, int y_f16, int64_t ldy, int M, int N,
                 int K, float *ws, int prefetch, cudaStream_t stream);
int transpose(const void *src, int64_t lds, void *dst, int64_t ldd, int rows, int cols, int esize,
              cudaStream_t stream);

// M above which quantised linears take the tensor-core GEMM instead of the
// decode GEMV (overridable with VKFLAME_GEMV_MAX_M for A/B comparisons).
static int gemv_max_m() {
    static const int v = [] {
        const char *e = getenv("VKFLAME_GEMV_MAX_M");
        return e ? atoi(e) : 8;
    }();
    return v;
}

static size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// VKFLAME_FUSED_PREFILL=0 routes prefill through widen-then-GEMM (A/B runs).
static bool fused_prefill_enabled() {
    static const bool on = [] {
        const char *e = getenv("VKFLAME_FUSED_PREFILL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Prefill path.  X reaches the GEMM as fp16 rows at 16-byte aligned
// addresses (Q8_1 activations widened, misaligned rows staged: M*K*2 bytes,
// small next to W).  Q4_0 / Q8_0 / Q4_K / Q5_K with K a multiple of 256 take
// the fused-dequant tcgen05 GEMM (W read once as packed blocks); otherwise W
// is widened to fp16 (one rounding per weight) and the f16 tcgen05 GEMM runs.
static int quant_linear_gemm(const void *W, int wtype, const void *X, int xtype, void *Y, int ytype, int M, int N,
                             int K, int64_t ldx, int64_t ldy, cudaStream_t stream, unsigned flags) {
    if (((size_t)K * 2) % 16) return VKF_ERR_UNSUPPORTED;
    const bool fused = fused_prefill_enabled() && qgemm_supported(wtype, W, K);
    // Staged X, then the widened W (widen path) or the split-tile partials
    // (fused path): one request, since growing the arena drops its contents.
    const size_t xbytes = align256((size_t)M * K * 2);
    const size_t wbytes = fused ? align256(qgemm_ws_bytes(wtype, M, N, K)) : align256((size_t)N * K * 2);
    const bool stage_x = xtype == VKF_X_Q8_1 || ((uintptr_t)X & 15) || (ldx * 2) % 16;
    uint8_t *scr = (uint8_t *)stream_scratch(stream, (stage_x ? xbytes : 0) + wbytes);
    if (!scr) return VKF_ERR_NOMEM;
    const void *xf = X;
    int64_t lda = ldx;
    if (stage_x) {
        int rc = VKF_OK;
        if (xtype == VKF_X_Q8_1) rc = q8_1_to_f16(X, scr, M, K, ldx, K, stream);
        else if (cudaMemcpy2DAsync(scr, (size_t)K * 2, X, ldx * 2, (size_t)K * 2, M, cudaMemcpyDeviceToDevice,
                                   stream) != cudaSuccess)
            rc = VKF_ERR_CUDA;
        if (rc) return rc;
        xf = scr;
        lda = K;
    }
    uint8_t *wf = scr + (stage_x ? xbytes : 0);
    if (fused)
        return qgemm_launch(wtype, W, xf, lda, Y, ytype == VKF_Y_F16, ldy, M, N, K, (float *)wf,
                            (flags & VKF_FLAG_STATIC_WEIGHTS) ? 1 : 0, stream);
    int rc = dequant_launch(W, wf, (uint64_t)N * K / vkf_qtype_block_values(wtype), wtype, stream, true);
    if (rc) return rc;
    return gemm_f16_tn(xf, lda, wf, K, M, N, K, 1.0f, 0.0f, nullptr, 0, 0, nullptr, 0, Y, ldy,
                       ytype == VKF_Y_F16, stream);
}

static bool gemv_format(int wtype) {
    return wtype == VKF_DEQUANT_Q4_0 || wtype == VKF_DEQUANT_Q8_0 || wtype == VKF_DEQUANT_Q4_K ||
           wtype == VKF_DEQUANT_Q5_K || wtype == VKF_DEQUANT_Q6_K;
}

// Decode path for M <= 8 (and, until the tensor-core GEMM covers a format,
// for larger M in column groups).
static int quant_linear_gemv(const void *W, int wtype, const void *X, int xtype, void *Y, int ytype, int M, int N,
                             int K, int64_t ldx, int64_t ldy, cudaStream_t stream, unsigned flags) {
    DeviceState *ds = device_state();
    if (!ds) return VKF_ERR_NO_DEVICE;
    // Activations must reach the kernel as fp16 rows at 16-byte aligned
    // addresses; anything else is staged once into scratch (M*K*2 bytes).
    const bool direct = xtype == VKF_X_F16 && ((uintptr_t)X & 15) == 0 && (ldx * 2) % 16 == 0;
    const int64_t ldx_st = ((int64_t)K * 2 + 15) / 16 * 16;  // staged row stride, bytes
    const size_t stage_bytes = direct ? 0 : (((size_t)M * ldx_st + 255) & ~size_t(255));
    const size_t ws_floats = gemv_ws_floats(ds->sm_count);
    uint8_t *scr = (uint8_t *)stream_scratch(stream, stage_bytes + ws_floats * sizeof(float));
    const size_t ncnt = gemv_counters(N);
    int *cnt = stream_counters(stream, ncnt);
    if (!scr || !cnt) return VKF_ERR_NOMEM;
    const void *xf = X;
    int64_t ldx_bytes = ldx * 2;
    if (!direct) {
        if (xtype == VKF_X_Q8_1) {
            int rc = q8_1_to_f16(X, scr, M, K, ldx, ldx_st / 2, stream);
            if (rc) return rc;
        } else {
            if (cudaMemcpy2DAsync(scr, ldx_st, X, ldx * 2, (size_t)K * 2, M, cudaMemcpyDeviceToDevice, stream) !=
                cudaSuccess)
                return VKF_ERR_CUDA;
        }
        xf = scr;
        ldx_bytes = ldx_st;
    }
    const int y_f16 = ytype == VKF_Y_F16;
    // Batch columns are processed in groups whose activations fit the
    // kernel's resident shared-memory budget (all 8 when K <= 4608).
    const int cols = gemv_cols_per_launch(K);
    for (int m0 = 0; m0 < M; m0 += cols) {
        const int mc = M - m0 < cols ? M - m0 : cols;
        const void *xm = (const uint8_t *)xf + m0 * ldx_bytes;
        void *ym = (uint8_t *)Y + (size_t)m0 * ldy * (y_f16 ? 2 : 4);
        int rc = gemv_launch(wtype, W, xm, ldx_bytes, ym, y_f16, ldy, mc, N, K, stream,
                             reinterpret_cast<float *>(scr + stage_bytes), ws_floats, cnt, ncnt,
                             (flags & VKF_FLAG_STATIC_WEIGHTS) ? 1 : 0);
        if (rc) return rc;
    }
    return VKF_OK;
}

// Formats with no fused decoder (Q4_1, Q5_0): widened to fp16 by their
// bit-exact dequant kernel, then the tensor-core GEMM, at every M (the
// reference's dequant + GEMM chain, shim/hip_runtime_shim.cpp:1129-1166,
// with one fp16 rounding of each weight).
static bool widen_format(int wtype) { return wtype == VKF_DEQUANT_Q4_1 || wtype == VKF_DEQUANT_Q5_0; }

int quant_linear(const void *W, int wtype, const void *X, int xtype, void *Y, int ytype, int M, int N, int K,
                 int64_t ldx, int64_t ldy, cudaStream_t stream, unsigned flags) {
    if (!gemv_format(wtype) && !widen_format(wtype)) return VKF_ERR_UNSUPPORTED;
    if (M < 0 || N < 0 || K < 0 || (xtype != VKF_X_F16 && xtype != VKF_X_Q8_1) ||
        (ytype != VKF_Y_F32 && ytype != VKF_Y_F16))
        return VKF_ERR_INVALID;
    if (M == 0 || N == 0) return VKF_OK;
    const int qk = vkf_qtype_block_values(wtype);
    if (K == 0 || K % qk || K % 32) return VKF_ERR_INVALID;
    if (ldy < N || (xtype == VKF_X_F16 && ldx < K) || (xtype == VKF_X_Q8_1 && ldx < K / 32)) return VKF_ERR_INVALID;
    const size_t row_bytes = (size_t)K / qk * vkf_qtype_block_bytes(wtype);
    const size_t xbytes = xtype == VKF_X_F16 ? ((size_t)(M - 1) * ldx + K) * 2 : ((size_t)(M - 1) * ldx + K / 32) * 36;
    const size_t ybytes = ((size_t)(M - 1) * ldy + N) * (ytype == VKF_Y_F16 ? 2 : 4);
    if (validate_device_range(W, row_bytes * N) || validate_device_range(X, xbytes) ||
        validate_device_range(Y, ybytes))
        return VKF_ERR_BADPTR;
    // Block alignment the decoders rely on: 32-bit words for Q4_K/Q5_K,
    // 16-bit elsewhere; fp16 / fp32 output element alignment.
    const uintptr_t wa = (uintptr_t)W;
    if ((wtype == VKF_DEQUANT_Q4_K || wtype == VKF_DEQUANT_Q5_K) ? (wa & 3) : (wa & 1)) return VKF_ERR_BADPTR;
    if ((uintptr_t)Y & (ytype == VKF_Y_F16 ? 1 : 3)) return VKF_ERR_BADPTR;
    if (xtype == VKF_X_F16 && ((uintptr_t)X & 1)) return VKF_ERR_BADPTR;
    if (M > gemv_max_m() || widen_format(wtype))
        return quant_linear_gemm(W, wtype, X, xtype, Y, ytype, M, N, K, ldx, ldy, stream, flags);
    return quant_linear_gemv(W, wtype, X, xtype, Y, ytype, M, N, K, ldx, ldy, stream, flags);
}

}  // namespace vkf

extern "C" int vkflame_quant_linear(const void *W, int wtype, const void *X, int xtype, void *Y, int ytype, int M,
                                    int N, int K, int64_t ldx, int64_t ldy, void *stream) {
    return vkf::set_status(vkf::quant_linear(W, wtype, X, xtype, Y, ytype, M, N, K, ldx, ldy, (cudaStream_t)stream, 0));
}

extern "C" int vkflame_quant_linear_ex(const void *W, int wtype, const void *X, int xtype, void *Y, int ytype, int M,
                                       int N, int K, int64_t ldx, int64_t ldy, unsigned flags, void *stream) {
    return vkf::set_status(
        vkf::quant_linear(W, wtype, X, xtype, Y, ytype, M, N, K, ldx, ldy, (cudaStream_t)stream, flags));
}


// ---- decode GEMV fused with the column all-gather ---------------------------

namespace vkf {

static int quant_linear_gather(const void *W, int wtype, const void *X, int ytype, int M, int N, int K, int64_t ldx,
                               int64_t ldy, unsigned flags, const vkf_gather_t *g, cudaStream_t stream) {
    (void)ldy;
    if (!gemv_format(wtype) || !g) return VKF_ERR_INVALID;
    if (g->world < 1 || g->world > VKF_MAX_RANKS || g->rank < 0 || g->rank >= g->world) return VKF_ERR_INVALID;
    if (M != 1 || N < 2 || N % 2 || K < 1 || ytype != VKF_Y_F16 || ldx < K) return VKF_ERR_INVALID;
    const int qk = vkf_qtype_block_values(wtype);
    if (K % qk || K % 32) return VKF_ERR_UNSUPPORTED;
    const int64_t ldx_bytes = g->x_gathered ? ldx * 4 : ldx * 2;  // gathered: 8-byte words of 2 values
    if (((uintptr_t)X & 15) || ldx_bytes % 16) return VKF_ERR_BADPTR;
    if (g->x_gathered && (ldx % 4 || g->x_stride % 16)) return VKF_ERR_BADPTR;
    for (int q = 0; q < g->world; ++q)
        if (!g->y_rank[q] || ((uintptr_t)g->y_rank[q] & 7)) return VKF_ERR_BADPTR;
    if (!g->epoch || !g->done || g->stride % 8) return VKF_ERR_BADPTR;
    const size_t row_bytes = (size_t)K / qk * vkf_qtype_block_bytes(wtype);
    if (validate_device_range(W, row_bytes * N)) return VKF_ERR_BADPTR;
    DeviceState *ds = device_state();
    if (!ds) return VKF_ERR_NO_DEVICE;
    const size_t ws_floats = gemv_ws_floats(ds->sm_count);
    float *ws = (float *)stream_scratch(stream, ws_floats * sizeof(float));
    const size_t ncnt = gemv_counters(N);
    int *cnt = stream_counters(stream, ncnt);
    if (!ws || !cnt) return VKF_ERR_NOMEM;
    return gemv_launch(wtype, W, X, ldx_bytes, g->y_rank[g->rank], 1, N, M, N, K, stream, ws, ws_floats, cnt, ncnt,
                       (flags & VKF_FLAG_STATIC_WEIGHTS) ? 1 : 0, g);
}

}  // namespace vkf

extern "C" int vkflame_quant_linear_gather(const void *W, int wtype, const void *X, int ytype, int M, int N, int K,
                                           int64_t ldx, int64_t ldy, unsigned flags, const vkf_gather_t *g,
                                           void *stream) {
    return vkf::set_status(
        vkf::quant_linear_gather(W, wtype, X, ytype, M, N, K, ldx, ldy, flags, g, (cudaStream_t)stream));
}

// ---- linear_int8 and the generic linear dispatcher --------------------------

namespace vkf {

int linear_int8(const int8_t *X, const int8_t *W, const float *sx, const float *sw, const void *bias, void *Y,
                int32_t *acc_out, int M, int N, int K, int act, cudaStream_t stream) {
    if (M < 0 || N < 0 || K < 0 || act < 0 || act > 3) return VKF_ERR_INVALID;
    if (M == 0 || N == 0) return VKF_OK;
    if (!Y && !acc_out) return VKF_ERR_INVALID;
    if (validate_device_range(X, (size_t)M * K) || validate_device_range(W, (size_t)N * K) ||
        (sx && validate_device_range(sx, (size_t)M * 4)) || (sw && validate_device_range(sw, (size_t)N * 4)) ||
        (bias && validate_device_range(bias, (size_t)N * 2)) || (Y && validate_device_range(Y, (size_t)M * N * 2)) ||
        (acc_out && validate_device_range(acc_out, (size_t)M * N * 4)))
        return VKF_ERR_BADPTR;
    const int8_t *xa = X, *wa = W;
    int64_t ld = K;
    if (K % 16 || ((uintptr_t)X & 15) || ((uintptr_t)W & 15)) {
        // TMA rows must start on 16-byte boundaries: pad K with zeros.
        const int64_t kp = (K + 15) / 16 * 16;
        uint8_t *scr = (uint8_t *)stream_scratch(stream, align256((size_t)M * kp) + align256((size_t)N * kp));
        if (!scr) return VKF_ERR_NOMEM;
        int8_t *xs = (int8_t *)scr, *ws = (int8_t *)(scr + align256((size_t)M * kp));
        if (cudaMemsetAsync(scr, 0, align256((size_t)M * kp) + align256((size_t)N * kp), stream) != cudaSuccess ||
            cudaMemcpy2DAsync(xs, kp, X, K, K, M, cudaMemcpyDeviceToDevice, stream) != cudaSuccess ||
            cudaMemcpy2DAsync(ws, kp, W, K, K, N, cudaMemcpyDeviceToDevice, stream) != cudaSuccess)
            return VKF_ERR_CUDA;
        xa = xs;
        wa = ws;
        ld = kp;
        K = (int)kp;
    }
    return gemm_i8_tn(xa, ld, wa, ld, M, N, K, sx, sw, bias, Y, N, acc_out, N, act, stream);
}

// runtime/dispatch.h:51-58 semantics, with the reference's ignored
// arguments implemented (runtime/dispatch.cpp:262-267): op(A) is M x K, op(B)
// is K x N, D = act(alpha * op(A) op(B) + beta * C), all row-major and packed.
int dispatch_linear(const void *A, const void *B, const void *C, void *D, int M, int N, int K, int dtype, int transA,
                    int transB, int act, const void *alpha, const void *beta, cudaStream_t stream) {
    if (M < 0 || N < 0 || K < 0 || act < 0 || act > 3) return VKF_ERR_INVALID;
    if (M == 0 || N == 0) return VKF_OK;
    if (!A || !B || !D) return VKF_ERR_BADPTR;
    const float al = alpha ? *(const float *)alpha : 1.0f, be = beta ? *(const float *)beta : 0.0f;
    int esize;
    switch (dtype) {
    case VKF_DTYPE_FP16:
    case VKF_DTYPE_FP16_FP32OUT: esize = 2; break;
    case VKF_DTYPE_INT8: esize = 1; break;
    case VKF_DTYPE_FP32: esize = 4; break;
    default: return VKF_ERR_UNSUPPORTED;  // bf16 inputs: not on this path
    }
    const int out_f16 = dtype == VKF_DTYPE_FP16 || dtype == VKF_DTYPE_INT8;
    if (validate_device_range(A, (size_t)M * K * esize) || validate_device_range(B, (size_t)K * N * esize) ||
        validate_device_range(D, (size_t)M * N * (out_f16 ? 2 : 4)) ||
        (C && be != 0.0f && validate_device_range(C, (size_t)M * N * (out_f16 ? 2 : 4))))
        return VKF_ERR_BADPTR;
    // Bring both operands to K-major (A: M x K, B: N x K), padding K to 16 bytes.
    const int64_t kp = ((int64_t)K * esize + 15) / 16 * 16 / esize;
    const bool a_ok = !transA && kp == K && ((uintptr_t)A & 15) == 0;
    const bool b_ok = transB && kp == K && ((uintptr_t)B & 15) == 0;
    const size_t abytes = a_ok ? 0 : align256((size_t)M * kp * esize), bbytes = b_ok ? 0 : align256((size_t)N * kp * esize);
    uint8_t *scr = nullptr;
    if (abytes + bbytes) {
        scr = (uint8_t *)stream_scratch(stream, abytes + bbytes);
        if (!scr) return VKF_ERR_NOMEM;
        if (kp != K && cudaMemsetAsync(scr, 0, abytes + bbytes, stream) != cudaSuccess) return VKF_ERR_CUDA;
    }
    const void *a = A, *b = B;
    int rc = VKF_OK;
    if (!a_ok) {
        rc = transA ? transpose(A, M, scr, kp, K, M, esize, stream)  // stored K x M
                    : (cudaMemcpy2DAsync(scr, kp * esize, A, (size_t)K * esize, (size_t)K * esize, M,
                                         cudaMemcpyDeviceToDevice, stream) == cudaSuccess ? VKF_OK : VKF_ERR_CUDA);
        a = scr;
    }
    if (rc) return rc;
    if (!b_ok) {
        rc = !transB ? transpose(B, N, scr + abytes, kp, K, N, esize, stream)  // stored K x N
                     : (cudaMemcpy2DAsync(scr + abytes, kp * esize, B, (size_t)K * esize, (size_t)K * esize, N,
                                          cudaMemcpyDeviceToDevice, stream) == cudaSuccess ? VKF_OK : VKF_ERR_CUDA);
        b = scr + abytes;
    }
    if (rc) return rc;
    if (dtype == VKF_DTYPE_FP32)
        return gemm_tf32_tn((const float *)a, kp, (const float *)b, kp, M, N, (int)kp, al, be, be != 0.0f ? C : nullptr,
                            N, 0, nullptr, act, D, N, 0, stream);
    if (dtype == VKF_DTYPE_INT8)
        return gemm_i8_tn((const int8_t *)a, kp, (const int8_t *)b, kp, M, N, (int)kp, nullptr, nullptr, nullptr, D, N,
                          nullptr, 0, act, stream);
    return gemm_f16_tn(a, kp, b, kp, M, N, (int)kp, al, be, be != 0.0f ? C : nullptr, N, out_f16, nullptr, act, D, N,
                       out_f16, stream);
}

}  // namespace vkf

extern "C" int vkflame_linear_int8(const int8_t *X, const int8_t *W, const float *sx, const float *sw,
                                   const void *bias, void *Y, int32_t *acc_out, int M, int N, int K, int activation,
                                   void *stream) {
    return vkf::set_status(vkf::linear_int8(X, W, sx, sw, bias, Y, acc_out, M, N, K, activation, (cudaStream_t)stream));
}

extern "C" int vkflame_dispatch_linear(void *ctx, const void *A, const void *B, const void *C, void *D, int M, int N,
                                       int K, int dtype, int transA, int transB, int activation, const void *alpha,
                                       const void *beta, void *stream) {
    (void)ctx;
    return vkf::set_status(vkf::dispatch_linear(A, B, C, D, M, N, K, dtype, transA, transB, activation, alpha, beta,
                                                (cudaStream_t)stream));
}
