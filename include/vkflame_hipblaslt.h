/*
 * vkflame_hipblaslt.h — exports of libhipblaslt.so.0 (the hipBLASLt drop-in).
 *
 * Names, signatures and constant values of the reference shim
 * (shim/hipblaslt_shim.cpp:12-58 constants, :104-426 functions).  As in the
 * reference, hipblasLtMatmul treats matrices as row-major (its comment at
 * shim/hipblaslt_shim.cpp:370): op(A) is M x K, op(B) is K x N, D is M x N,
 * leading dimensions from the layouts (default: the column count).  Unlike
 * the reference (defects at :254-262 / :418-423), BIAS_POINTER, the scale
 * pointers, transposes, alpha/beta, batch count and strided offsets are
 * honoured:
 *   D = act( alpha * op(A) op(B) [* a_scale[m] * b_scale[n]] + bias[n] ) + beta * C
 * a_scale / b_scale are per-row / per-column fp32 vectors (int8 inputs: the
 * linear_int8 per-row / per-channel scales); bias is fp16[N]; act from the
 * epilogue (RELU, GELU (erf form), SILU; BIAS adds the bias only).
 */
#ifndef VKFLAME_HIPBLASLT_H
#define VKFLAME_HIPBLASLT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int hipblasStatus_t;
typedef void *hipStream_t;

#define HIPBLASLT_MATRIX_LAYOUT_ROWS 0
#define HIPBLASLT_MATRIX_LAYOUT_COLS 1
#define HIPBLASLT_MATRIX_LAYOUT_LD 2
#define HIPBLASLT_MATRIX_LAYOUT_TYPE 3
#define HIPBLASLT_MATRIX_LAYOUT_BATCH_COUNT 4
#define HIPBLASLT_MATRIX_LAYOUT_STRIDED_BATCH_OFFSET 5

#define HIPBLASLT_MATMUL_DESC_TRANSA 0
#define HIPBLASLT_MATMUL_DESC_TRANSB 1
#define HIPBLASLT_MATMUL_DESC_COMPUTE_TYPE 2
#define HIPBLASLT_MATMUL_DESC_SCALE_TYPE 3
#define HIPBLASLT_MATMUL_DESC_POINTER_MODE 4
#define HIPBLASLT_MATMUL_DESC_EPILOGUE 5
#define HIPBLASLT_MATMUL_DESC_BIAS_POINTER 6
#define HIPBLASLT_MATMUL_DESC_A_SCALE_POINTER 7
#define HIPBLASLT_MATMUL_DESC_B_SCALE_POINTER 8
#define HIPBLASLT_MATMUL_DESC_D_SCALE_POINTER 9
#define HIPBLASLT_MATMUL_DESC_AMAX_D_POINTER 10

#define HIPBLASLT_EPILOGUE_DEFAULT 0
#define HIPBLASLT_EPILOGUE_RELU 1
#define HIPBLASLT_EPILOGUE_BIAS 2
#define HIPBLASLT_EPILOGUE_GELU 3
#define HIPBLASLT_EPILOGUE_SILU 4

#define HIPBLASLT_R_16F 0
#define HIPBLASLT_R_32F 1
#define HIPBLASLT_R_8I 2
#define HIPBLASLT_R_16B 3
#define HIPBLASLT_R_32I 4 /* extension: int32 D of an int8 matmul (the reference defines no int32 type) */

#define HIPBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES 0

/* shim/hipblaslt_shim.cpp:104-116 */
hipblasStatus_t hipblasLtCreate(void **lightHandle);
hipblasStatus_t hipblasLtDestroy(void *lightHandle);
/* :120-209 */
hipblasStatus_t hipblasLtMatrixLayoutCreate(void **matLayout, int type, uint64_t rows, uint64_t cols, int64_t ld);
hipblasStatus_t hipblasLtMatrixLayoutDestroy(void *matLayout);
hipblasStatus_t hipblasLtMatrixLayoutSetAttribute(void *matLayout, int attr, const void *buf, size_t sizeInBytes);
hipblasStatus_t hipblasLtMatrixLayoutGetAttribute(void *matLayout, int attr, void *buf, size_t sizeInBytes,
                                                  size_t *sizeWritten);
/* :213-292 */
hipblasStatus_t hipblasLtMatmulDescCreate(void **matmulDesc, int computeType, int scaleType);
hipblasStatus_t hipblasLtMatmulDescDestroy(void *matmulDesc);
hipblasStatus_t hipblasLtMatmulDescSetAttribute(void *matmulDesc, int attr, const void *buf, size_t sizeInBytes);
hipblasStatus_t hipblasLtMatmulDescGetAttribute(void *matmulDesc, int attr, void *buf, size_t sizeInBytes,
                                                size_t *sizeWritten);
/* :296-319 */
hipblasStatus_t hipblasLtMatmulPreferenceCreate(void **pref);
hipblasStatus_t hipblasLtMatmulPreferenceDestroy(void *pref);
hipblasStatus_t hipblasLtMatmulPreferenceSetAttribute(void *pref, int attr, const void *buf, size_t sizeInBytes);
/* :323-343: one algorithm, as in the reference */
hipblasStatus_t hipblasLtMatmulAlgoGetHeuristic(void *lightHandle, void *matmulDesc, void *Adesc, void *Bdesc,
                                                void *Cdesc, void *Ddesc, void *pref, int requestedAlgoCount,
                                                void *heuristicResultsArray, int *returnAlgoCount);
/* :347-426; alpha/beta are host fp32 scalars (NULL: 1 and 0); workspace is not used */
hipblasStatus_t hipblasLtMatmul(void *lightHandle, void *matmulDesc, const void *alpha, const void *A, void *Adesc,
                                const void *B, void *Bdesc, const void *beta, const void *C, void *Cdesc, void *D,
                                void *Ddesc, const void *algo, void *workspace, size_t workspaceSizeInBytes,
                                hipStream_t stream);

#ifdef __cplusplus
}
#endif
#endif
