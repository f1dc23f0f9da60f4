// shim_api.h — entry points of libvkflame_rt.so used by the drop-in shim
// libraries (internal: C++ linkage, not part of the public C ABI).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/vkflame_rt.h"

namespace vkf {
enum BlasType { BT_F16 = 0, BT_F32 = 1, BT_I8 = 2, BT_I32 = 3 };
int blas_gemm(int transA, int transB, int m, int n, int k, float alpha, const void *A, int atype, int64_t lda,
              const void *B, int btype, int64_t ldb, float beta, void *C, int ctype, int64_t ldc, cudaStream_t stream);
int blas_gemm_ex(int transA, int transB, int m, int n, int k, float alpha, const void *A, int atype, int64_t lda,
                 const void *B, int btype, int64_t ldb, float beta, void *C, int ctype, int64_t ldc,
                 const float *row_scale, const float *col_scale, const void *bias, int act, cudaStream_t stream);
}  // namespace vkf
