/*
 * vkflame_hipblas.h — exports of libhipblas.so.2 (the hipBLAS drop-in).
 *
 * Same names, signatures and constant values as the reference shim
 * (shim/hipblas_shim.cpp:10-37 constants, :52-363 functions).  Matrices are
 * column-major device pointers as in hipBLAS; unlike the reference, which
 * ignored them (shim/hipblas_shim.cpp:89-92, runtime/dispatch.cpp:262-267),
 * transpose flags, leading dimensions, alpha and beta are honoured.  GEMMs
 * run on the tcgen05 tensor-core kernels of libvkflame_rt.so: f16 x f16
 * (kind::f16, fp32 accumulate), f32 x f32 (kind::tf32), s8 x s8 (kind::i8,
 * exact int32 accumulate).
 */
#ifndef VKFLAME_HIPBLAS_H
#define VKFLAME_HIPBLAS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int hipblasStatus_t;
typedef void *hipStream_t;
typedef int hipblasDatatype_t;
typedef int hipblasComputeType_t;
typedef int hipblasGemmAlgo_t;
typedef unsigned short hipblasHalf;

#define HIPBLAS_STATUS_SUCCESS 0
#define HIPBLAS_STATUS_NOT_INITIALIZED 1
#define HIPBLAS_STATUS_ALLOC_FAILED 2
#define HIPBLAS_STATUS_INVALID_VALUE 3
#define HIPBLAS_STATUS_ARCH_MISMATCH 4
#define HIPBLAS_STATUS_MAPPING_ERROR 5
#define HIPBLAS_STATUS_EXECUTION_FAILED 6
#define HIPBLAS_STATUS_INTERNAL_ERROR 7
#define HIPBLAS_STATUS_NOT_SUPPORTED 8

#define HIPBLAS_OP_N 111
#define HIPBLAS_OP_T 112
#define HIPBLAS_OP_C 113

#define HIPBLAS_R_32F 0
#define HIPBLAS_R_64F 1
#define HIPBLAS_R_16F 2
#define HIPBLAS_R_8I 4
#define HIPBLAS_R_32I 10 /* extension: int32 C of an int8 GemmEx (the reference defines no int32 type) */
#define HIPBLAS_GEMM_DEFAULT 0

/* shim/hipblas_shim.cpp:52-80 */
hipblasStatus_t hipblasCreate(void **handle);
hipblasStatus_t hipblasDestroy(void *handle);
hipblasStatus_t hipblasSetStream(void *handle, hipStream_t stream);
hipblasStatus_t hipblasGetStream(void *handle, hipStream_t *stream);

/* shim/hipblas_shim.cpp:84-142 */
hipblasStatus_t hipblasSgemm(void *handle, int transA, int transB, int m, int n, int k, const float *alpha,
                             const float *A, int lda, const float *B, int ldb, const float *beta, float *C, int ldc);
hipblasStatus_t hipblasHgemm(void *handle, int transA, int transB, int m, int n, int k, const hipblasHalf *alpha,
                             const hipblasHalf *A, int lda, const hipblasHalf *B, int ldb, const hipblasHalf *beta,
                             hipblasHalf *C, int ldc);
/* shim/hipblas_shim.cpp:145-188 (pointer arrays may live in device or host memory) */
hipblasStatus_t hipblasSgemmBatched(void *handle, int transA, int transB, int m, int n, int k, const float *alpha,
                                    const float *const A_array[], int lda, const float *const B_array[], int ldb,
                                    const float *beta, float *const C_array[], int ldc, int batch_count);
hipblasStatus_t hipblasHgemmBatched(void *handle, int transA, int transB, int m, int n, int k,
                                    const hipblasHalf *alpha, const hipblasHalf *const A_array[], int lda,
                                    const hipblasHalf *const B_array[], int ldb, const hipblasHalf *beta,
                                    hipblasHalf *const C_array[], int ldc, int batch_count);
/* shim/hipblas_shim.cpp:191-245 (strides in elements) */
hipblasStatus_t hipblasSgemmStridedBatched(void *handle, int transA, int transB, int m, int n, int k,
                                           const float *alpha, const float *A, int lda, long long strideA,
                                           const float *B, int ldb, long long strideB, const float *beta, float *C,
                                           int ldc, long long strideC, int batch_count);
hipblasStatus_t hipblasHgemmStridedBatched(void *handle, int transA, int transB, int m, int n, int k,
                                           const hipblasHalf *alpha, const hipblasHalf *A, int lda,
                                           long long strideA, const hipblasHalf *B, int ldb, long long strideB,
                                           const hipblasHalf *beta, hipblasHalf *C, int ldc, long long strideC,
                                           int batch_count);
/* shim/hipblas_shim.cpp:251-290; alpha/beta are fp32 unless computeType is HIPBLAS_R_16F */
hipblasStatus_t hipblasGemmEx(void *handle, int transA, int transB, int m, int n, int k, const void *alpha,
                              const void *A, hipblasDatatype_t aType, int lda, const void *B, hipblasDatatype_t bType,
                              int ldb, const void *beta, void *C, hipblasDatatype_t cType, int ldc,
                              hipblasComputeType_t computeType, hipblasGemmAlgo_t algo);
/* shim/hipblas_shim.cpp:293-314 */
hipblasStatus_t hipblasGemmBatchedEx(void *handle, int transA, int transB, int m, int n, int k, const void *alpha,
                                     const void *const A_array[], hipblasDatatype_t aType, int lda,
                                     const void *const B_array[], hipblasDatatype_t bType, int ldb,
                                     const void *beta, void *const C_array[], hipblasDatatype_t cType, int ldc,
                                     int batch_count, hipblasComputeType_t computeType, hipblasGemmAlgo_t algo);
/* shim/hipblas_shim.cpp:317-349 */
hipblasStatus_t hipblasGemmStridedBatchedEx(void *handle, int transA, int transB, int m, int n, int k,
                                            const void *alpha, const void *A, hipblasDatatype_t aType, int lda,
                                            long long strideA, const void *B, hipblasDatatype_t bType, int ldb,
                                            long long strideB, const void *beta, void *C, hipblasDatatype_t cType,
                                            int ldc, long long strideC, int batch_count,
                                            hipblasComputeType_t computeType, hipblasGemmAlgo_t algo);
/* shim/hipblas_shim.cpp:354-363: not supported, as in the reference */
hipblasStatus_t hipblasStrsmBatched(void *handle, int side, int uplo, int transA, int diag, int m, int n,
                                    const float *alpha, const float *const A[], int lda, float *const B[], int ldb,
                                    int batch_count);

#ifdef __cplusplus
}
#endif
#endif
