// linear.cu — kernel selection for the quantised linear entry points.
//
// Replaces the reference's quantised mul_mat chain (shim/hip_runtime_shim.cpp:
// 1129-1166: dequant W -> fp32 temp, dequant X -> fp32 temp, naive GEMM,
// two allocations and three synchronous submits per call) with one fused
// kernel launch on the caller's stream.

#include "rt_internal.h"

#include <cuda_fp16.h>

namespace vkf {
int gemv_launch(int wtype, const void *W, const void *X, int64_t ldx_bytes, void *Y, int y_f16, int64_t ldy, int M,
                int N, int K, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap, int prefetch);
size_t gemv_ws_floats(int sms);
size_t gemv_counters(int N);
int gemv_cols_per_launch(int K);
int q8_1_to_f16(const void *src, void *dst, int M, int K, int64_t ldb, int64_t ldo, cudaStream_t stream);

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

int quant_linear(const void *W, int wtype, const void *X, int xtype, void *Y, int ytype, int M, int N, int K,
                 int64_t ldx, int64_t ldy, cudaStream_t stream, unsigned flags) {
    if (!gemv_format(wtype)) return VKF_ERR_UNSUPPORTED;
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

// Tensor-core GEMM entry points (tcgen05); filled in by gemm_tc.cu.
extern "C" int vkflame_linear_int8(const int8_t *X, const int8_t *W, const float *sx, const float *sw,
                                   const void *bias, void *Y, int32_t *acc_out, int M, int N, int K, int activation,
                                   void *stream) {
    (void)X; (void)W; (void)sx; (void)sw; (void)bias; (void)Y; (void)acc_out; (void)M; (void)N; (void)K;
    (void)activation; (void)stream;
    return vkf::set_status(VKF_ERR_UNSUPPORTED);
}

extern "C" int vkflame_dispatch_linear(void *ctx, const void *A, const void *B, const void *C, void *D, int M, int N,
                                       int K, int dtype, int transA, int transB, int activation, const void *alpha,
                                       const void *beta, void *stream) {
    (void)ctx; (void)A; (void)B; (void)C; (void)D; (void)M; (void)N; (void)K; (void)dtype; (void)transA;
    (void)transB; (void)activation; (void)alpha; (void)beta; (void)stream;
    return vkf::set_status(VKF_ERR_UNSUPPORTED);
}
