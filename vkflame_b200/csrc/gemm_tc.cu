// gemm_tc.cu — tcgen05 tensor-core GEMM for prefill-sized linears (M >= 32).
//
//   D[m, n] = epilogue( sum_k A[m, k] * B[n, k] )       A: M x K, B: N x K (K-major)
//
// kind::i8 (s8 x s8 -> s32) serves linear_int8 (kernels/linear_int8.glsl,
// whose int32 accumulator this reproduces bit for bit); kind::f16 (f16 x f16
// -> f32) serves fp16 GEMMs and quantised-weight prefill (weights widened to
// fp16 first); kind::tf32 serves fp32 GEMMs.  The reference computes these with one thread per output and
// a K-serial loop (linear_int8.glsl:48-101, linear_fp16.glsl:38-51).
//
// One 128 x BN output tile per CTA, 192 threads:
//   warp 0       TMA producer: 2-D tiled loads (128-byte swizzle, no
//                multicast) of A and B K-blocks into an NS-deep ring;
//   warp 1       allocates the TMEM accumulator; one thread issues
//                tcgen05.mma (4 per 128-byte K-block) and commits each stage
//                back to the producer, and the finished tile to the epilogue;
//   warps 2..5   epilogue: tcgen05.ld of the accumulator (each warp owns the
//                32 TMEM lanes = tile rows of its warp rank), scaling, bias,
//                activation, store.
// Out-of-range rows and K are zero-filled by TMA, so any M, N, K work.

#include "tc_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

namespace vkf {
namespace gemm {

constexpr int BM = 128;
constexpr int BKB = 128;  // bytes of K per stage
constexpr int NT = 192;

struct Epi {
    void *Y;
    int64_t ldy;
    int y_f16;
    int32_t *acc_out;  // optional raw accumulators (i8), row stride ldacc
    int64_t ldacc;
    const float *sx;   // per-row scale (i8), optional
    const float *sw;   // per-column scale (i8), optional
    const __half *bias;
    int act;
    float alpha, beta;  // f16 path: alpha * acc + beta * C
    const void *C;
    int64_t ldc;
    int c_f16;
    unsigned *err;
};

__device__ __forceinline__ float erf_as(float x) {
    // Abramowitz & Stegun 7.1.26, the form the reference shaders use
    // (kernels/linear_fp16.glsl:23-28).
    const float t = 1.0f / (1.0f + 0.3275911f * fabsf(x));
    const float y =
        1.0f - ((((1.061405429f * t - 1.453152027f) * t + 1.421413741f) * t - 0.284496736f) * t + 0.254829592f) * t *
                   expf(-x * x);
    return x >= 0.0f ? y : -y;
}

__device__ __forceinline__ float activation(int act, float x) {
    switch (act) {
    case VKF_ACT_SILU: return x * (1.0f / (1.0f + expf(-x)));
    case VKF_ACT_RELU: return x > 0.0f ? x : 0.0f;
    case VKF_ACT_GELU_ERF: return 0.5f * x * (1.0f + erf_as(x * 0.70710678118654f));
    default: return x;
    }
}

template <int KIND, int BN, int NS>
__global__ void __launch_bounds__(NT, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N, int K,
                const __grid_constant__ Epi e) {
    constexpr bool I8 = KIND == tc::KIND_I8;
    constexpr int A_BYTES = BM * BKB, B_BYTES = BN * BKB, STAGE = A_BYTES + B_BYTES;
    constexpr int KE = I8 ? 128 : KIND == tc::KIND_TF32 ? 32 : 64;  // elements of K per stage
    constexpr uint32_t IDESC = tc::instr_desc(KIND, BM, BN);
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + NS * STAGE);
    uint64_t *empty = full + NS;
    uint64_t *accf = empty + NS;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(accf + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    const int KB = (K + KE - 1) / KE;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(accf, 1);
        fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tslot, BN);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem = *tslot;

    if (warp == 0 && lane == 0) {
        for (int kb = 0; kb < KB; ++kb) {
            const int s = kb % NS;
            if (kb >= NS && !mbar_wait(&empty[s], ((kb / NS) & 1) ^ 1, e.err)) break;
            mbar_arrive_expect_tx(&full[s], STAGE);
            uint8_t *st = smem + s * STAGE;
            tc::tma_load_2d(st, &tmA, kb * KE, m0, &full[s]);
            tc::tma_load_2d(st + A_BYTES, &tmB, kb * KE, n0, &full[s]);
        }
    } else if (warp == 1 && lane == 0) {
        for (int kb = 0; kb < KB; ++kb) {
            const int s = kb % NS;
            if (!mbar_wait(&full[s], (kb / NS) & 1, e.err)) break;
            tc::fence_after_sync();
            const uint32_t sa = smem_addr(smem + s * STAGE), sb = sa + A_BYTES;
#pragma unroll
            for (int kk = 0; kk < BKB / 32; ++kk)
                tc::mma<KIND>(tmem, tc::smem_desc_sw128(sa + kk * 32), tc::smem_desc_sw128(sb + kk * 32), IDESC,
                            (kb | kk) != 0);
            tc::commit(&empty[s]);
        }
        tc::commit(accf);
    } else if (warp >= 2) {
        // ---- epilogue ----
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        const int row = m0 + 32 * q + lane;
        const bool ok = mbar_wait(accf, 0, e.err);
        tc::fence_after_sync();
        float sxr = 1.0f;
        if (I8 && e.sx && row < M) sxr = e.sx[row];
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
            uint32_t r[32];
            tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 32 * c, r);
            if (!ok || row >= M) continue;
            const int col0 = n0 + 32 * c;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                const int col = col0 + j;
                if (col >= N) break;
                float v;
                if constexpr (I8) {
                    const int32_t acc = (int32_t)r[j];
                    if (e.acc_out) e.acc_out[(int64_t)row * e.ldacc + col] = acc;
                    v = (float)acc;
                    v = __fmul_rn(v, sxr);
                    if (e.sw) v = __fmul_rn(v, e.sw[col]);
                } else {
                    v = __fmul_rn(e.alpha, __uint_as_float(r[j]));
                    if (e.C && e.beta != 0.0f) {
                        const float cv = e.c_f16 ? __half2float(reinterpret_cast<const __half *>(e.C)[(int64_t)row * e.ldc + col])
                                                 : reinterpret_cast<const float *>(e.C)[(int64_t)row * e.ldc + col];
                        v = __fadd_rn(v, __fmul_rn(e.beta, cv));
                    }
                }
                if (e.bias) v = __fadd_rn(v, __half2float(e.bias[col]));
                v = activation(e.act, v);
                if (e.Y) {
                    if (e.y_f16) reinterpret_cast<__half *>(e.Y)[(int64_t)row * e.ldy + col] = __float2half_rn(v);
                    else reinterpret_cast<float *>(e.Y)[(int64_t)row * e.ldy + col] = v;
                }
            }
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_free(tmem, BN);
    }
}

// ---- host: tensor maps ------------------------------------------------------

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        cudaDriverEntryPointQueryResult q;
        void *p = nullptr;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    });
    return fn;
}

// Row-major [rows x cols] matrix of esize-byte elements, row stride ld
// elements; box = (box_cols x box_rows), 128-byte swizzle.
static bool make_map(CUtensorMap *m, const void *base, int esize, int64_t rows, int64_t cols, int64_t ld,
                     int box_cols, int box_rows) {
    const CUtensorMapDataType dt = esize == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                   : esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT32;
    auto fn = encode_fn();
    if (!fn) return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(m, dt, 2,
                    const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

template <int KIND, int BN, int NS>
static int launch(const void *A, int64_t lda, const void *B, int64_t ldb, int M, int N, int K, const Epi &e,
                  cudaStream_t stream) {
    const int esize = KIND == tc::KIND_I8 ? 1 : KIND == tc::KIND_TF32 ? 4 : 2, KE = BKB / esize;
    CUtensorMap ta, tb;
    if (!make_map(&ta, A, esize, M, K, lda, KE, BM) || !make_map(&tb, B, esize, N, K, ldb, KE, BN))
        return VKF_ERR_INVALID;
    const size_t smem = (size_t)NS * (BM + BN) * BKB + 1024 + 256;
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        cudaFuncSetAttribute(gemm_kernel<KIND, BN, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr[dev] = true;
    }
    dim3 grid((N + BN - 1) / BN, (M + BM - 1) / BM);
    gemm_kernel<KIND, BN, NS><<<grid, NT, smem, stream>>>(ta, tb, M, N, K, e);
    return check_launch();
}

}  // namespace gemm

// TMA requirements: 16-byte aligned bases and row strides.
static bool tma_ok(const void *p, int64_t ld, int esize) {
    return ((uintptr_t)p & 15) == 0 && (ld * esize) % 16 == 0;
}

// D = epilogue(A x B^T); A: M x K (lda), B: N x K (ldb), both int8.
int gemm_i8_tn(const int8_t *A, int64_t lda, const int8_t *B, int64_t ldb, int M, int N, int K, const float *sx,
               const float *sw, const void *bias, void *Y, int64_t ldy, int32_t *acc_out, int64_t ldacc, int act,
               cudaStream_t stream, int y_f16) {
    DeviceState *ds = device_state();
    if (!ds) return VKF_ERR_NO_DEVICE;
    if (!tma_ok(A, lda, 1) || !tma_ok(B, ldb, 1)) return VKF_ERR_BADPTR;
    gemm::Epi e{};
    e.Y = Y;
    e.ldy = ldy;
    e.y_f16 = y_f16;
    e.acc_out = acc_out;
    e.ldacc = ldacc;
    e.sx = sx;
    e.sw = sw;
    e.bias = (const __half *)bias;
    e.act = act;
    e.err = ds->d_error;
    return gemm::launch<tc::KIND_I8, 256, 4>(A, lda, B, ldb, M, N, K, e, stream);
}

// D = act(alpha * A x B^T + beta * C + bias); A: M x K f16, B: N x K f16.
int gemm_f16_tn(const void *A, int64_t lda, const void *B, int64_t ldb, int M, int N, int K, float alpha, float beta,
                const void *C, int64_t ldc, int c_f16, const void *bias, int act, void *Y, int64_t ldy, int y_f16,
                cudaStream_t stream) {
    DeviceState *ds = device_state();
    if (!ds) return VKF_ERR_NO_DEVICE;
    if (!tma_ok(A, lda, 2) || !tma_ok(B, ldb, 2)) return VKF_ERR_BADPTR;
    gemm::Epi e{};
    e.Y = Y;
    e.ldy = ldy;
    e.y_f16 = y_f16;
    e.alpha = alpha;
    e.beta = beta;
    e.C = C;
    e.ldc = ldc;
    e.c_f16 = c_f16;
    e.bias = (const __half *)bias;
    e.act = act;
    e.err = ds->d_error;
    return gemm::launch<tc::KIND_F16, 256, 4>(A, lda, B, ldb, M, N, K, e, stream);
}

// As gemm_f16_tn with fp32 operands (tensor-core tf32: 10-bit mantissa products, fp32 accumulation).
int gemm_tf32_tn(const float *A, int64_t lda, const float *B, int64_t ldb, int M, int N, int K, float alpha,
                 float beta, const void *C, int64_t ldc, int c_f16, const void *bias, int act, void *Y, int64_t ldy,
                 int y_f16, cudaStream_t stream) {
    DeviceState *ds = device_state();
    if (!ds) return VKF_ERR_NO_DEVICE;
    if (!tma_ok(A, lda, 4) || !tma_ok(B, ldb, 4)) return VKF_ERR_BADPTR;
    gemm::Epi e{};
    e.Y = Y;
    e.ldy = ldy;
    e.y_f16 = y_f16;
    e.alpha = alpha;
    e.beta = beta;
    e.C = C;
    e.ldc = ldc;
    e.c_f16 = c_f16;
    e.bias = (const __half *)bias;
    e.act = act;
    e.err = ds->d_error;
    return gemm::launch<tc::KIND_TF32, 256, 4>(A, lda, B, ldb, M, N, K, e, stream);
}

}  // namespace vkf
