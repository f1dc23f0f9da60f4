// blas.cu — column-major BLAS GEMM on the tcgen05 kernels (the hipBLAS /
// hipBLASLt shims' back end).
//
//   C (m x n, col-major, ldc) = alpha * op(A) op(B) + beta * C
//
// The reference's shims swapped A<->B and m<->n and then ignored the
// transpose flags, leading dimensions, alpha and beta (shim/hipblas_shim.cpp:
// 101-110, runtime/dispatch.cpp:262-267).  Here they are honoured.  A
// column-major m x n C is a row-major n x m matrix R with row stride ldc, and
// R = op(B)^T op(A)^T, which the row-major "TN" kernels compute as
// D[j][i] = sum_k A''[j][k] B''[i][k] with A''[j][k] = op(B)(k, j) and
// B''[i][k] = op(A)(i, k).  With op(A) = A^T and op(B) = B (the usual
// X * W^T call) both operands are already K-major and no copy is made;
// otherwise the operand is transposed into scratch first.

#include "rt_internal.h"
#include "shim_api.h"

#include <cuda_fp16.h>

namespace vkf {

int gemm_i8_tn(const int8_t *A, int64_t lda, const int8_t *B, int64_t ldb, int M, int N, int K, const float *sx,
               const float *sw, const void *bias, void *Y, int64_t ldy, int32_t *acc_out, int64_t ldacc, int act,
               cudaStream_t stream, int y_f16);
int gemm_f16_tn(const void *A, int64_t lda, const void *B, int64_t ldb, int M, int N, int K, float alpha, float beta,
                const void *C, int64_t ldc, int c_f16, const void *bias, int act, void *Y, int64_t ldy, int y_f16,
                cudaStream_t stream);
int gemm_tf32_tn(const float *A, int64_t lda, const float *B, int64_t ldb, int M, int N, int K, float alpha,
                 float beta, const void *C, int64_t ldc, int c_f16, const void *bias, int act, void *Y, int64_t ldy,
                 int y_f16, cudaStream_t stream);
int transpose(const void *src, int64_t lds, void *dst, int64_t ldd, int rows, int cols, int esize,
              cudaStream_t stream);
int scale_c(void *C, int ctype, int64_t ldc, int m, int n, float beta, cudaStream_t stream);
int split_tf32(const float *src, int64_t lds, float *hi, float *lo, int64_t ldd, int rows, int k,
               cudaStream_t stream);


static int esize_of(int t) { return t == BT_F16 ? 2 : t == BT_I8 ? 1 : 4; }

// Makes a K-major copy (rows x k, row stride kp) of an operand when needed.
// kmajor: the operand is rows x k row-major with stride ld; otherwise it is
// k x rows row-major (stride ld) and is transposed.
static int prepare(const void *src, int64_t ld, int rows, int k, int es, bool kmajor, uint8_t *scr,
                   const void **out, int64_t *out_ld, cudaStream_t stream) {
    const int64_t kp = ((int64_t)k * es + 15) / 16 * 16 / es;
    if (kmajor && ((uintptr_t)src & 15) == 0 && (ld * es) % 16 == 0) {
        *out = src;
        *out_ld = ld;
        return VKF_OK;
    }
    *out = scr;
    *out_ld = kp;
    if (kmajor)
        return cudaMemcpy2DAsync(scr, kp * es, src, ld * es, (size_t)k * es, rows, cudaMemcpyDeviceToDevice, stream) ==
                       cudaSuccess
                   ? VKF_OK
                   : VKF_ERR_CUDA;
    return transpose(src, ld, scr, kp, k, rows, es, stream);
}

// Epilogue extras (hipBLASLt): scales per kernel row (= column of the
// column-major C) and per kernel column (= row of C), fp16 bias per kernel
// column, activation.  A row-major D = op(A) op(B) is the column-major
// D^T = op(B)^T op(A)^T, so for row-major callers kernel rows are D's rows.
int blas_gemm_ex(int transA, int transB, int m, int n, int k, float alpha, const void *A, int atype, int64_t lda,
                 const void *B, int btype, int64_t ldb, float beta, void *C, int ctype, int64_t ldc,
                 const float *row_scale, const float *col_scale, const void *bias, int act, cudaStream_t stream) {
    if (m < 0 || n < 0 || k < 0) return VKF_ERR_INVALID;
    if (m == 0 || n == 0) return VKF_OK;
    if (atype != btype || (atype != BT_F16 && atype != BT_F32 && atype != BT_I8)) return VKF_ERR_UNSUPPORTED;
    if (ctype != BT_F16 && ctype != BT_F32 && !(ctype == BT_I32 && atype == BT_I8)) return VKF_ERR_UNSUPPORTED;
    if (!C) return VKF_ERR_BADPTR;
    if (ldc < m) return VKF_ERR_INVALID;
    if (k == 0) return scale_c(C, ctype, ldc, m, n, beta, stream);  // hipBLAS: C = beta * C
    if (!A || !B) return VKF_ERR_BADPTR;
    if (lda < (transA ? k : m) || ldb < (transB ? n : k)) return VKF_ERR_INVALID;
    const int es = esize_of(atype);
    const int64_t kp = ((int64_t)k * es + 15) / 16 * 16 / es;
    // Staging regions: A'' (n rows, from B) first, then B'' (m rows, from A);
    // fp32 output from fp32 operands adds the tf32 hi/lo halves of both.
    const size_t a2bytes = ((size_t)n * kp * es + 255) & ~size_t(255);
    const size_t b2bytes = ((size_t)m * kp * es + 255) & ~size_t(255);
    const bool split = atype == BT_F32 && ctype == BT_F32;
    if (atype != BT_I8 && (row_scale || col_scale)) return VKF_ERR_UNSUPPORTED;
    if (atype == BT_I8 && (alpha != 1.0f || beta != 0.0f)) return VKF_ERR_UNSUPPORTED;
    uint8_t *scr = (uint8_t *)stream_scratch(stream, (a2bytes + b2bytes) * (split ? 3 : 1));
    if (!scr) return VKF_ERR_NOMEM;
    // A'' (n x k) from B: K-major iff op(B) = B (column-major k x n = row-major n x k).
    const void *a2, *b2;
    int64_t lda2, ldb2;
    int rc = prepare(B, ldb, n, k, es, !transB, scr, &a2, &lda2, stream);
    if (rc) return rc;
    // B'' (m x k) from A: K-major iff op(A) = A^T (column-major k x m = row-major m x k).
    rc = prepare(A, lda, m, k, es, transA, scr + a2bytes, &b2, &ldb2, stream);
    if (rc) return rc;
    if (split) {
        // fp32 GEMM as three tf32 products (hipblasSgemm callers expect fp32
        // accuracy, not tf32's 10-bit mantissa): x = hi + lo per operand,
        // C = a(lo_A' hi_B') + bC, then += a(hi_A' lo_B'), then += a(hi_A' hi_B')
        // with the epilogue (bias, activation) on the last pass; lo x lo
        // (~2^-22 relative) is dropped.
        float *ah = (float *)(scr + a2bytes + b2bytes), *al = (float *)((uint8_t *)ah + a2bytes);
        float *bh = (float *)((uint8_t *)al + a2bytes), *bl = (float *)((uint8_t *)bh + b2bytes);
        if (row_scale || col_scale) return VKF_ERR_UNSUPPORTED;
        if ((rc = split_tf32((const float *)a2, lda2, ah, al, kp, n, k, stream))) return rc;
        if ((rc = split_tf32((const float *)b2, ldb2, bh, bl, kp, m, k, stream))) return rc;
        if ((rc = gemm_tf32_tn(al, kp, bh, kp, n, m, k, alpha, beta, beta != 0.0f ? C : nullptr, ldc, 0, nullptr, 0,
                               C, ldc, 0, stream)))
            return rc;
        if ((rc = gemm_tf32_tn(ah, kp, bl, kp, n, m, k, alpha, 1.0f, C, ldc, 0, nullptr, 0, C, ldc, 0, stream)))
            return rc;
        return gemm_tf32_tn(ah, kp, bh, kp, n, m, k, alpha, 1.0f, C, ldc, 0, bias, act, C, ldc, 0, stream);
    }
    const int y_f16 = ctype == BT_F16;
    if (atype == BT_I8) {
        if (alpha != 1.0f || beta != 0.0f) return VKF_ERR_UNSUPPORTED;
        if (ctype == BT_I32)
            return gemm_i8_tn((const int8_t *)a2, lda2, (const int8_t *)b2, ldb2, n, m, k, nullptr, nullptr, nullptr,
                              nullptr, 0, (int32_t *)C, ldc, 0, stream, 0);
        return gemm_i8_tn((const int8_t *)a2, lda2, (const int8_t *)b2, ldb2, n, m, k, row_scale, col_scale, bias, C,
                          ldc, nullptr, 0, act, stream, y_f16);
    }
    if (row_scale || col_scale) return VKF_ERR_UNSUPPORTED;
    const void *cin = beta != 0.0f ? C : nullptr;
    if (atype == BT_F32)
        return gemm_tf32_tn((const float *)a2, lda2, (const float *)b2, ldb2, n, m, k, alpha, beta, cin, ldc, y_f16,
                            bias, act, C, ldc, y_f16, stream);
    return gemm_f16_tn(a2, lda2, b2, ldb2, n, m, k, alpha, beta, cin, ldc, y_f16, bias, act, C, ldc, y_f16, stream);
}

int blas_gemm(int transA, int transB, int m, int n, int k, float alpha, const void *A, int atype, int64_t lda,
              const void *B, int btype, int64_t ldb, float beta, void *C, int ctype, int64_t ldc, cudaStream_t stream) {
    return blas_gemm_ex(transA, transB, m, n, k, alpha, A, atype, lda, B, btype, ldb, beta, C, ctype, ldc, nullptr,
                        nullptr, nullptr, 0, stream);
}

}  // namespace vkf
