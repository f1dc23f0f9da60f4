// layout.cu — operand layout helpers for the tensor-core GEMM: a tiled
// transpose that brings MN-major operands (hipBLAS op(N) B, op(T) A) into the
// K-major layout the GEMM's TMA tiles read.

#include "rt_internal.h"

#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

namespace vkf {
namespace {

// dst[c * ldd + r] = src[r * lds + c] for r < rows, c < cols.
template <typename T>
__global__ void __launch_bounds__(256) transpose_kernel(const T *__restrict__ src, int64_t lds, T *__restrict__ dst,
                                                        int64_t ldd, int rows, int cols) {
    __shared__ T tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
    for (int i = ty; i < 32; i += 8) {
        const int r = r0 + i, c = c0 + tx;
        if (r < rows && c < cols) tile[i][tx] = src[(int64_t)r * lds + c];
    }
    __syncthreads();
    for (int i = ty; i < 32; i += 8) {
        const int c = c0 + i, r = r0 + tx;
        if (r < rows && c < cols) dst[(int64_t)c * ldd + r] = tile[tx][i];
    }
}

// C[j * ldc + i] = beta * C[j * ldc + i] for i < m, j < n (column-major);
// beta == 0 writes zeros without reading C (BLAS convention: NaNs in C do
// not propagate).
template <typename T>
__global__ void __launch_bounds__(256) scale_kernel(T *C, int64_t ldc, int m, int n, float beta) {
    const int64_t total = (int64_t)m * n;
    for (int64_t e = blockIdx.x * 256ll + threadIdx.x; e < total; e += (int64_t)gridDim.x * 256) {
        const int64_t j = e / m, i = e - j * m;
        T &c = C[j * ldc + i];
        if constexpr (std::is_same<T, __half>::value) c = beta == 0.f ? __float2half_rn(0.f) : __float2half_rn(beta * __half2float(c));
        else if constexpr (std::is_same<T, int32_t>::value) c = beta == 0.f ? 0 : __float2int_rn(beta * (float)c);
        else c = beta == 0.f ? 0.f : beta * c;
    }
}

// x = hi + lo with hi = x rounded to tf32 (10-bit mantissa, ties away) and
// lo = x - hi (exact in fp32); both K-major rows x k, row stride ldd.
__global__ void __launch_bounds__(256) split_tf32_kernel(const float *__restrict__ src, int64_t lds,
                                                         float *__restrict__ hi, float *__restrict__ lo, int64_t ldd,
                                                         int rows, int k) {
    const int64_t total = (int64_t)rows * k;
    for (int64_t e = blockIdx.x * 256ll + threadIdx.x; e < total; e += (int64_t)gridDim.x * 256) {
        const int64_t r = e / k, c = e - r * k;
        const float x = src[r * lds + c];
        uint32_t h;
        asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(x));
        const float hf = __uint_as_float(h);
        hi[r * ldd + c] = hf;
        lo[r * ldd + c] = x - hf;
    }
}

}  // namespace

int split_tf32(const float *src, int64_t lds, float *hi, float *lo, int64_t ldd, int rows, int k,
               cudaStream_t stream) {
    if (rows <= 0 || k <= 0) return VKF_OK;
    const int64_t total = (int64_t)rows * k;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
    split_tf32_kernel<<<grid, 256, 0, stream>>>(src, lds, hi, lo, ldd, rows, k);
    return check_launch();
}

// hipBLAS GEMM with k == 0: C = beta * C (column-major m x n, ldc).
int scale_c(void *C, int ctype, int64_t ldc, int m, int n, float beta, cudaStream_t stream) {
    if (beta == 1.0f || m <= 0 || n <= 0) return VKF_OK;
    const int64_t total = (int64_t)m * n;
    const int grid = (int)std::min<int64_t>((total + 255) / 256, 148 * 16);
    switch (ctype) {
    case 0: scale_kernel<__half><<<grid, 256, 0, stream>>>((__half *)C, ldc, m, n, beta); break;
    case 1: scale_kernel<float><<<grid, 256, 0, stream>>>((float *)C, ldc, m, n, beta); break;
    case 3: scale_kernel<int32_t><<<grid, 256, 0, stream>>>((int32_t *)C, ldc, m, n, beta); break;
    default: return VKF_ERR_UNSUPPORTED;
    }
    return check_launch();
}

int transpose(const void *src, int64_t lds, void *dst, int64_t ldd, int rows, int cols, int esize,
              cudaStream_t stream) {
    if (rows <= 0 || cols <= 0) return VKF_OK;
    dim3 grid((cols + 31) / 32, (rows + 31) / 32);
    switch (esize) {
    case 1: transpose_kernel<uint8_t><<<grid, 256, 0, stream>>>((const uint8_t *)src, lds, (uint8_t *)dst, ldd, rows, cols); break;
    case 2: transpose_kernel<uint16_t><<<grid, 256, 0, stream>>>((const uint16_t *)src, lds, (uint16_t *)dst, ldd, rows, cols); break;
    case 4: transpose_kernel<uint32_t><<<grid, 256, 0, stream>>>((const uint32_t *)src, lds, (uint32_t *)dst, ldd, rows, cols); break;
    default: return VKF_ERR_INVALID;
    }
    return check_launch();
}

}  // namespace vkf
