// layout.cu — operand layout helpers for the tensor-core GEMM: a tiled
// transpose that brings MN-major operands (hipBLAS op(N) B, op(T) A) into the
// K-major layout the GEMM's TMA tiles read.

#include "rt_internal.h"

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

}  // namespace

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
