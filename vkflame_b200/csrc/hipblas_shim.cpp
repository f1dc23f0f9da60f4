// hipblas_shim.cpp — libhipblas.so.2: the hipBLAS drop-in over the B200
// tensor-core GEMMs of libvkflame_rt.so (include/vkflame_hipblas.h).
//
// Replaces shim/hipblas_shim.cpp of the reference, which forwarded every
// call to a Vulkan one-thread-per-output shader and ignored transposes,
// leading dimensions, alpha/beta and the handle's stream.

#include "../../include/vkflame_hipblas.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <vector>

#include "shim_api.h"

namespace {

struct Handle {
    cudaStream_t stream = nullptr;
};

int trans_of(int op) { return (op == HIPBLAS_OP_T || op == HIPBLAS_OP_C) ? 1 : (op == HIPBLAS_OP_N ? 0 : -1); }

hipblasStatus_t status_of(int vkf) {
    switch (vkf) {
    case VKF_OK: return HIPBLAS_STATUS_SUCCESS;
    case VKF_ERR_INVALID:
    case VKF_ERR_BADPTR: return HIPBLAS_STATUS_INVALID_VALUE;
    case VKF_ERR_UNSUPPORTED: return HIPBLAS_STATUS_NOT_SUPPORTED;
    case VKF_ERR_NOMEM: return HIPBLAS_STATUS_ALLOC_FAILED;
    case VKF_ERR_NO_DEVICE: return HIPBLAS_STATUS_ARCH_MISMATCH;
    default: return HIPBLAS_STATUS_EXECUTION_FAILED;
    }
}

int type_of(hipblasDatatype_t t) {
    switch (t) {
    case HIPBLAS_R_16F: return vkf::BT_F16;
    case HIPBLAS_R_32F: return vkf::BT_F32;
    case HIPBLAS_R_8I: return vkf::BT_I8;
    case HIPBLAS_R_32I: return vkf::BT_I32;
    default: return -1;
    }
}

int esize_of(hipblasDatatype_t t) { return t == HIPBLAS_R_16F ? 2 : t == HIPBLAS_R_8I ? 1 : 4; }

float half_to_float(const hipblasHalf *h) {
    __half v;
    *reinterpret_cast<unsigned short *>(&v) = *h;
    return __half2float(v);
}

// Scalar alpha/beta as the compute type: fp16 when computeType is R_16F.
float scalar(const void *p, hipblasComputeType_t ct, float dflt) {
    if (!p) return dflt;
    return ct == HIPBLAS_R_16F ? half_to_float((const hipblasHalf *)p) : *(const float *)p;
}

hipblasStatus_t gemm(void *handle, int transA, int transB, int m, int n, int k, float alpha, const void *A,
                     hipblasDatatype_t at, int lda, const void *B, hipblasDatatype_t bt, int ldb, float beta, void *C,
                     hipblasDatatype_t ct, int ldc) {
    if (!handle) return HIPBLAS_STATUS_NOT_INITIALIZED;
    const int ta = trans_of(transA), tb = trans_of(transB);
    const int a = type_of(at), b = type_of(bt), c = type_of(ct);
    if (ta < 0 || tb < 0 || a < 0 || b < 0 || c < 0) return HIPBLAS_STATUS_INVALID_VALUE;
    return status_of(vkf::blas_gemm(ta, tb, m, n, k, alpha, A, a, lda, B, b, ldb, beta, C, c, ldc,
                                    static_cast<Handle *>(handle)->stream));
}

// Pointer arrays of the batched calls: hipBLAS passes them in device memory;
// host arrays are accepted too.
std::vector<const void *> host_ptrs(const void *const *arr, int count) {
    std::vector<const void *> v(count > 0 ? count : 0);
    if (count <= 0) return v;
    cudaPointerAttributes attr;
    if (cudaPointerGetAttributes(&attr, arr) == cudaSuccess && attr.type == cudaMemoryTypeDevice) {
        cudaMemcpy(v.data(), arr, sizeof(void *) * count, cudaMemcpyDeviceToHost);
    } else {
        cudaGetLastError();
        for (int i = 0; i < count; ++i) v[i] = arr[i];
    }
    return v;
}

}  // namespace

extern "C" {

hipblasStatus_t hipblasCreate(void **handle) {
    if (!handle) return HIPBLAS_STATUS_INVALID_VALUE;
    if (vkflame_init() != VKF_OK) return HIPBLAS_STATUS_ARCH_MISMATCH;
    *handle = new Handle;
    return HIPBLAS_STATUS_SUCCESS;
}

hipblasStatus_t hipblasDestroy(void *handle) {
    delete static_cast<Handle *>(handle);
    return HIPBLAS_STATUS_SUCCESS;
}

hipblasStatus_t hipblasSetStream(void *handle, hipStream_t stream) {
    if (!handle) return HIPBLAS_STATUS_NOT_INITIALIZED;
    static_cast<Handle *>(handle)->stream = (cudaStream_t)stream;
    return HIPBLAS_STATUS_SUCCESS;
}

hipblasStatus_t hipblasGetStream(void *handle, hipStream_t *stream) {
    if (!handle || !stream) return HIPBLAS_STATUS_INVALID_VALUE;
    *stream = static_cast<Handle *>(handle)->stream;
    return HIPBLAS_STATUS_SUCCESS;
}

hipblasStatus_t hipblasSgemm(void *handle, int transA, int transB, int m, int n, int k, const float *alpha,
                             const float *A, int lda, const float *B, int ldb, const float *beta, float *C, int ldc) {
    return gemm(handle, transA, transB, m, n, k, alpha ? *alpha : 1.0f, A, HIPBLAS_R_32F, lda, B, HIPBLAS_R_32F, ldb,
                beta ? *beta : 0.0f, C, HIPBLAS_R_32F, ldc);
}

hipblasStatus_t hipblasHgemm(void *handle, int transA, int transB, int m, int n, int k, const hipblasHalf *alpha,
                             const hipblasHalf *A, int lda, const hipblasHalf *B, int ldb, const hipblasHalf *beta,
                             hipblasHalf *C, int ldc) {
    return gemm(handle, transA, transB, m, n, k, alpha ? half_to_float(alpha) : 1.0f, A, HIPBLAS_R_16F, lda, B,
                HIPBLAS_R_16F, ldb, beta ? half_to_float(beta) : 0.0f, C, HIPBLAS_R_16F, ldc);
}

hipblasStatus_t hipblasSgemmBatched(void *handle, int transA, int transB, int m, int n, int k, const float *alpha,
                                    const float *const A_array[], int lda, const float *const B_array[], int ldb,
                                    const float *beta, float *const C_array[], int ldc, int batch_count) {
    auto a = host_ptrs((const void *const *)A_array, batch_count), b = host_ptrs((const void *const *)B_array, batch_count),
         c = host_ptrs((const void *const *)C_array, batch_count);
    for (int i = 0; i < batch_count; ++i) {
        hipblasStatus_t s = hipblasSgemm(handle, transA, transB, m, n, k, alpha, (const float *)a[i], lda,
                                         (const float *)b[i], ldb, beta, (float *)c[i], ldc);
        if (s) return s;
    }
    return HIPBLAS_STATUS_SUCCESS;
}

hipblasStatus_t hipblasHgemmBatched(void *handle, int transA, int transB, int m, int n, int k,
                                    const hipblasHalf *alpha, const hipblasHalf *const A_array[], int lda,
                                    const hipblasHalf *const B_array[], int ldb, const hipblasHalf *beta,
                                    hipblasHalf *const C_array[], int ldc, int batch_count) {
    auto a = host_ptrs((const void *const *)A_array, batch_count), b = host_ptrs((const void *const *)B_array, batch_count),
         c = host_ptrs((const void *const *)C_array, batch_count);
    for (int i = 0; i < batch_count; ++i) {
        hipblasStatus_t s = hipblasHgemm(handle, transA, transB, m, n, k, alpha, (const hipblasHalf *)a[i], lda,
                                         (const hipblasHalf *)b[i], ldb, beta, (hipblasHalf *)c[i], ldc);
        if (s) return s;
    }
    return HIPBLAS_STATUS_SUCCESS;
}

hipblasStatus_t hipblasSgemmStridedBatched(void *handle, int transA, int transB, int m, int n, int k,
                                           const float *alpha, const float *A, int lda, long long strideA,
                                           const float *B, int ldb, long long strideB, const float *beta, float *C,
                                           int ldc, long long strideC, int batch_count) {
    for (int i = 0; i < batch_count; ++i) {
        hipblasStatus_t s = hipblasSgemm(handle, transA, transB, m, n, k, alpha, A + i * strideA, lda,
                                         B + i * strideB, ldb, beta, C + i * strideC, ldc);
        if (s) return s;
    }
    return HIPBLAS_STATUS_SUCCESS;
}

hipblasStatus_t hipblasHgemmStridedBatched(void *handle, int transA, int transB, int m, int n, int k,
                                           const hipblasHalf *alpha, const hipblasHalf *A, int lda,
                                           long long strideA, const hipblasHalf *B, int ldb, long long strideB,
                                           const hipblasHalf *beta, hipblasHalf *C, int ldc, long long strideC,
                                           int batch_count) {
    for (int i = 0; i < batch_count; ++i) {
        hipblasStatus_t s = hipblasHgemm(handle, transA, transB, m, n, k, alpha, A + i * strideA, lda,
                                         B + i * strideB, ldb, beta, C + i * strideC, ldc);
        if (s) return s;
    }
    return HIPBLAS_STATUS_SUCCESS;
}

hipblasStatus_t hipblasGemmEx(void *handle, int transA, int transB, int m, int n, int k, const void *alpha,
                              const void *A, hipblasDatatype_t aType, int lda, const void *B, hipblasDatatype_t bType,
                              int ldb, const void *beta, void *C, hipblasDatatype_t cType, int ldc,
                              hipblasComputeType_t computeType, hipblasGemmAlgo_t algo) {
    (void)algo;
    return gemm(handle, transA, transB, m, n, k, scalar(alpha, computeType, 1.0f), A, aType, lda, B, bType, ldb,
                scalar(beta, computeType, 0.0f), C, cType, ldc);
}

hipblasStatus_t hipblasGemmBatchedEx(void *handle, int transA, int transB, int m, int n, int k, const void *alpha,
                                     const void *const A_array[], hipblasDatatype_t aType, int lda,
                                     const void *const B_array[], hipblasDatatype_t bType, int ldb,
                                     const void *beta, void *const C_array[], hipblasDatatype_t cType, int ldc,
                                     int batch_count, hipblasComputeType_t computeType, hipblasGemmAlgo_t algo) {
    auto a = host_ptrs(A_array, batch_count), b = host_ptrs(B_array, batch_count),
         c = host_ptrs((const void *const *)C_array, batch_count);
    for (int i = 0; i < batch_count; ++i) {
        hipblasStatus_t s = hipblasGemmEx(handle, transA, transB, m, n, k, alpha, a[i], aType, lda, b[i], bType, ldb,
                                          beta, (void *)c[i], cType, ldc, computeType, algo);
        if (s) return s;
    }
    return HIPBLAS_STATUS_SUCCESS;
}

hipblasStatus_t hipblasGemmStridedBatchedEx(void *handle, int transA, int transB, int m, int n, int k,
                                            const void *alpha, const void *A, hipblasDatatype_t aType, int lda,
                                            long long strideA, const void *B, hipblasDatatype_t bType, int ldb,
                                            long long strideB, const void *beta, void *C, hipblasDatatype_t cType,
                                            int ldc, long long strideC, int batch_count,
                                            hipblasComputeType_t computeType, hipblasGemmAlgo_t algo) {
    const int ea = esize_of(aType), eb = esize_of(bType), ec = esize_of(cType);
    for (int i = 0; i < batch_count; ++i) {
        hipblasStatus_t s = hipblasGemmEx(handle, transA, transB, m, n, k, alpha, (const char *)A + i * strideA * ea,
                                          aType, lda, (const char *)B + i * strideB * eb, bType, ldb, beta,
                                          (char *)C + i * strideC * ec, cType, ldc, computeType, algo);
        if (s) return s;
    }
    return HIPBLAS_STATUS_SUCCESS;
}

hipblasStatus_t hipblasStrsmBatched(void *, int, int, int, int, int, int, const float *, const float *const[], int,
                                    float *const[], int, int) {
    return HIPBLAS_STATUS_NOT_SUPPORTED;
}

}  // extern "C"
