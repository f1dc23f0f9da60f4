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
// Persistent CTAs (one per SM) over 128 x BN output tiles, 192 threads:
//   warp 0       TMA producer: 2-D tiled loads (128-byte swizzle, no
//                multicast) of A and B K-blocks into an NS-deep ring;
//   warp 1       allocates the double-buffered TMEM accumulator; one thread
//                issues tcgen05.mma (4 per 128-byte K-block), commits each
//                stage back to the producer and each finished tile to the
//                epilogue;
//   warps 2..5   epilogue: tcgen05.ld of the accumulator (each warp owns the
//                32 TMEM lanes = tile rows of its warp rank), scaling, bias,
//                activation, store.
// Out-of-range rows and K are zero-filled by TMA, so any M, N, K work.

#include "tc_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <climits>
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
    int vec;            // VEC_* bits
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

// Epi::vec bits: the operand's rows are 16-byte aligned (base and stride).
enum { VEC_Y = 1, VEC_ACC = 2, VEC_C = 4, VEC_SW = 8, VEC_BIAS = 16 };

__device__ __forceinline__ uint32_t h2_bits(float a, float b) {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t *>(&h);
}

// 32 values from p[col0 ..] (ncol valid, 1.0 / 0.0 past the end or when p is null).
__device__ __forceinline__ void load_f32_chunk(const float *p, int col0, int ncol, bool vec, float (&o)[32]) {
    if (!p) {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = 1.0f;
        return;
    }
    if (vec) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 t = __ldg(reinterpret_cast<const float4 *>(p + col0 + j));
            o[j] = t.x;
            o[j + 1] = t.y;
            o[j + 2] = t.z;
            o[j + 3] = t.w;
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = j < ncol ? p[col0 + j] : 1.0f;
    }
}

__device__ __forceinline__ void load_f16_chunk(const __half *p, int col0, int ncol, bool vec, float (&o)[32]) {
    if (vec) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
            const uint4 t = __ldg(reinterpret_cast<const uint4 *>(p + col0 + j));
            const uint32_t w[4] = {t.x, t.y, t.z, t.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[i]));
                o[j + 2 * i] = f.x;
                o[j + 2 * i + 1] = f.y;
            }
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) o[j] = j < ncol ? __half2float(p[col0 + j]) : 0.0f;
    }
}

// Persistent: one CTA per SM walks the output tiles (tile = m_tile + m_tiles *
// n_tile, so the M-tiles that share a B tile run on neighbouring CTAs at about
// the same time and B is read from DRAM once).  The TMEM accumulator is double
// buffered (2 x BN columns): the epilogue warps drain tile i while the MMA
// thread accumulates tile i + 1.
template <int KIND, int BN, int NS>
__global__ void __launch_bounds__(NT, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int M, int N, int K,
                const __grid_constant__ Epi e) {
    constexpr bool I8 = KIND == tc::KIND_I8;
    constexpr int A_BYTES = BM * BKB, B_BYTES = BN * BKB, STAGE = A_BYTES + B_BYTES;
    constexpr int KE = I8 ? 128 : KIND == tc::KIND_TF32 ? 32 : 64;  // elements of K per stage
    constexpr uint32_t IDESC = tc::instr_desc(KIND, BM, BN);
    constexpr uint32_t TCOLS = 2 * BN <= 32 ? 32 : 2 * BN <= 64 ? 64 : 2 * BN <= 128 ? 128 : 2 * BN <= 256 ? 256 : 512;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + NS * STAGE);
    uint64_t *empty = full + NS;
    uint64_t *acc_full = empty + NS;   // [2]: MMA -> epilogue
    uint64_t *acc_empty = acc_full + 2; // [2]: epilogue -> MMA (4 warps)
    uint32_t *tslot = reinterpret_cast<uint32_t *>(acc_empty + 2);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int m_tiles = (M + BM - 1) / BM, n_tiles = (N + BN - 1) / BN, tiles = m_tiles * n_tiles;
    const int KB = (K + KE - 1) / KE;

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&acc_full[b], 1);
            mbar_init(&acc_empty[b], 4);
        }
        fence_mbar_init();
    }
    if (warp == 1) tc::tmem_alloc(tslot, TCOLS);
    tc::fence_before_sync();
    __syncthreads();
    tc::fence_after_sync();
    const uint32_t tmem0 = *tslot;

    if (warp == 0 && lane == 0) {
        // ---- TMA producer: a continuous ring across the CTA's tiles ----
        int g = 0;  // global k-block counter
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x) {
            const int m0 = (tile % m_tiles) * BM, n0 = (tile / m_tiles) * BN;
            for (int kb = 0; kb < KB; ++kb, ++g) {
                const int s = g % NS;
                if (g >= NS && !(ok = mbar_wait(&empty[s], ((g / NS) & 1) ^ 1, e.err))) break;
                mbar_arrive_expect_tx(&full[s], STAGE);
                uint8_t *st = smem + s * STAGE;
                tc::tma_load_2d(st, &tmA, kb * KE, m0, &full[s]);
                tc::tma_load_2d(st + A_BYTES, &tmB, kb * KE, n0, &full[s]);
            }
        }
    } else if (warp == 1 && lane == 0) {
        // ---- MMA issuer ----
        int g = 0, it = 0;
        bool ok = true;
        for (int tile = blockIdx.x; tile < tiles && ok; tile += gridDim.x, ++it) {
            const int b = it & 1;
            // the epilogue must have drained this accumulator buffer (two tiles ago)
            if (it >= 2 && !(ok = mbar_wait(&acc_empty[b], ((it >> 1) & 1) ^ 1, e.err))) break;
            tc::fence_after_sync();
            const uint32_t tmem = tmem0 + b * BN;
            for (int kb = 0; kb < KB; ++kb, ++g) {
                const int s = g % NS;
                if (!(ok = mbar_wait(&full[s], (g / NS) & 1, e.err))) break;
                tc::fence_after_sync();
                const uint32_t sa = smem_addr(smem + s * STAGE), sb = sa + A_BYTES;
#pragma unroll
                for (int kk = 0; kk < BKB / 32; ++kk)
                    tc::mma<KIND>(tmem, tc::smem_desc_sw128(sa + kk * 32), tc::smem_desc_sw128(sb + kk * 32), IDESC,
                                  (kb | kk) != 0);
                tc::commit(&empty[s]);
            }
            tc::commit(&acc_full[b]);
        }
    } else if (warp >= 2) {
        // ---- epilogue ----
        const int q = warp & 3;  // TMEM lane quarter this warp may access
        int it = 0;
        for (int tile = blockIdx.x; tile < tiles; tile += gridDim.x, ++it) {
            const int b = it & 1;
            const int m0 = (tile % m_tiles) * BM, n0 = (tile / m_tiles) * BN;
            const int row = m0 + 32 * q + lane;
            const bool ok = mbar_wait(&acc_full[b], (it >> 1) & 1, e.err);
            tc::fence_after_sync();
            const uint32_t tmem = tmem0 + b * BN;
            float sxr = 1.0f;
            if (I8 && e.sx && row < M) sxr = e.sx[row];
#pragma unroll 1
            for (int c = 0; c < BN / 32; ++c) {
                uint32_t r[32];
                tc::tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + 32 * c, r);
                const int col0 = n0 + 32 * c;
                if (!ok || row >= M || col0 >= N) continue;
                // This thread owns 32 consecutive columns of one output row: with
                // 16-byte aligned rows every read and write below is a vector
                // access along the row; ragged or unaligned chunks go scalar.
                const bool full = col0 + 32 <= N;
                const int ncol = full ? 32 : N - col0;
                float v[32];
                if constexpr (I8) {
                    if (e.acc_out) {
                        int32_t *ap = e.acc_out + (int64_t)row * e.ldacc + col0;
                        if (full && (e.vec & VEC_ACC)) {
#pragma unroll
                            for (int j = 0; j < 32; j += 4)
                                *reinterpret_cast<uint4 *>(ap + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
                        } else {
#pragma unroll
                            for (int j = 0; j < 32; ++j)
                                if (j < ncol) ap[j] = (int32_t)r[j];
                        }
                    }
                    float swv[32];
                    load_f32_chunk(e.sw, col0, ncol, full && (e.vec & VEC_SW), swv);
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(__fmul_rn((float)(int32_t)r[j], sxr), swv[j]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(e.alpha, __uint_as_float(r[j]));
                    if (e.C && e.beta != 0.0f) {
                        float cv[32];
                        if (e.c_f16)
                            load_f16_chunk(reinterpret_cast<const __half *>(e.C) + (int64_t)row * e.ldc, col0, ncol,
                                           full && (e.vec & VEC_C), cv);
                        else
                            load_f32_chunk(reinterpret_cast<const float *>(e.C) + (int64_t)row * e.ldc, col0, ncol,
                                           full && (e.vec & VEC_C), cv);
#pragma unroll
                        for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], __fmul_rn(e.beta, cv[j]));
                    }
                }
                if (e.bias) {
                    float bv[32];
                    load_f16_chunk(e.bias, col0, ncol, full && (e.vec & VEC_BIAS), bv);
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __fadd_rn(v[j], bv[j]);
                }
                if (e.act) {
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = activation(e.act, v[j]);
                }
                if (!e.Y) continue;
                if (e.y_f16) {
                    __half *yp = reinterpret_cast<__half *>(e.Y) + (int64_t)row * e.ldy + col0;
                    if (full && (e.vec & VEC_Y)) {
#pragma unroll
                        for (int j = 0; j < 32; j += 8) {
                            uint4 o;
                            o.x = h2_bits(v[j], v[j + 1]);
                            o.y = h2_bits(v[j + 2], v[j + 3]);
                            o.z = h2_bits(v[j + 4], v[j + 5]);
                            o.w = h2_bits(v[j + 6], v[j + 7]);
                            *reinterpret_cast<uint4 *>(yp + j) = o;
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < ncol) yp[j] = __float2half_rn(v[j]);
                    }
                } else {
                    float *yp = reinterpret_cast<float *>(e.Y) + (int64_t)row * e.ldy + col0;
                    if (full && (e.vec & VEC_Y)) {
#pragma unroll
                        for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4 *>(yp + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < ncol) yp[j] = v[j];
                    }
                }
            }
            tc::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
            if (!ok) break;
        }
    }
    tc::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_free(tmem0, TCOLS);
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

}  // namespace gemm

bool make_kmajor_map(CUtensorMap *m, const void *base, int esize, int64_t rows, int64_t cols, int64_t ld,
                     int box_rows) {
    return gemm::make_map(m, base, esize, rows, cols, ld, gemm::BKB / esize, box_rows);
}

bool make_rowmajor_map(CUtensorMap *m, const void *base, int esize, int64_t rows, int64_t cols, int64_t ld,
                       int box_cols, int box_rows) {
    auto fn = gemm::encode_fn();
    if (!fn || ((uintptr_t)base & 15) || (ld * esize) % 16 || (box_cols * esize) % 16 || box_cols > 256 ||
        box_rows > 256)
        return false;
    cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)(ld * esize)};
    cuuint32_t box[2] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, esize == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2,
              const_cast<void *>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
              CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

bool make_byte_matrix_map(CUtensorMap *m, const void *base, int64_t rows, int64_t row_bytes, int box_bytes,
                          int box_rows) {
    auto fn = gemm::encode_fn();
    if (!fn || row_bytes % 16 || box_bytes % 8 || ((uintptr_t)base & 15) || box_bytes / 8 > 256 || box_rows > 256)
        return false;
    cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)rows};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(box_bytes / 8), (cuuint32_t)box_rows};
    cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void *>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace gemm {

static bool rows16(const void *p, int64_t ld, int esize) {
    return ((uintptr_t)p & 15) == 0 && (ld * esize) % 16 == 0;
}

template <int KIND, int BN, int NS>
static int launch(const void *A, int64_t lda, const void *B, int64_t ldb, int M, int N, int K, Epi e,
                  cudaStream_t stream) {
    e.vec = (e.Y && rows16(e.Y, e.ldy, e.y_f16 ? 2 : 4) ? VEC_Y : 0) |
            (e.acc_out && rows16(e.acc_out, e.ldacc, 4) ? VEC_ACC : 0) |
            (e.C && rows16(e.C, e.ldc, e.c_f16 ? 2 : 4) ? VEC_C : 0) | (e.sw && rows16(e.sw, 0, 4) ? VEC_SW : 0) |
            (e.bias && rows16(e.bias, 0, 2) ? VEC_BIAS : 0);
    const int esize = KIND == tc::KIND_I8 ? 1 : KIND == tc::KIND_TF32 ? 4 : 2, KE = BKB / esize;
    CUtensorMap ta, tb;
    if (!make_map(&ta, A, esize, M, K, lda, KE, BM) || !make_map(&tb, B, esize, N, K, ldb, KE, BN))
        return VKF_ERR_INVALID;
    const size_t smem = (size_t)NS * (BM + BN) * BKB + 1024 + 512;
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        cudaFuncSetAttribute(gemm_kernel<KIND, BN, NS>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        attr[dev] = true;
    }
    const int tiles = ((N + BN - 1) / BN) * ((M + BM - 1) / BM);
    DeviceState *ds = device_state();
    const int grid = std::max(1, std::min(tiles, ds ? ds->sm_count : 148));
    gemm_kernel<KIND, BN, NS><<<grid, NT, smem, stream>>>(ta, tb, M, N, K, e);
    return check_launch();
}

// Tile width: the persistent grid's time is about ceil(tiles / SMs) tile
// times, and a tile's time grows with its width, so pick the width that
// minimises ceil(tiles / SMs) * BN (wider on ties: fewer A re-reads).
template <int KIND>
static int launch_auto(const void *A, int64_t lda, const void *B, int64_t ldb, int M, int N, int K, const Epi &e,
                       cudaStream_t stream) {
    DeviceState *ds = device_state();
    const int sms = ds ? ds->sm_count : 148;
    const int widths[] = {256, 224, 192, 160, 128};
    int best = 256;
    int64_t best_cost = INT64_MAX;
    for (int bn : widths) {
        const int64_t tiles = (int64_t)((N + bn - 1) / bn) * ((M + BM - 1) / BM);
        const int64_t cost = ((tiles + sms - 1) / sms) * bn;
        if (cost < best_cost) {
            best_cost = cost;
            best = bn;
        }
    }
    switch (best) {
    case 224: return launch<KIND, 224, 4>(A, lda, B, ldb, M, N, K, e, stream);
    case 192: return launch<KIND, 192, 4>(A, lda, B, ldb, M, N, K, e, stream);
    case 160: return launch<KIND, 160, 4>(A, lda, B, ldb, M, N, K, e, stream);
    case 128: return launch<KIND, 128, 4>(A, lda, B, ldb, M, N, K, e, stream);
    default: return launch<KIND, 256, 4>(A, lda, B, ldb, M, N, K, e, stream);
    }
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
    return gemm::launch_auto<tc::KIND_I8>(A, lda, B, ldb, M, N, K, e, stream);
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
    return gemm::launch_auto<tc::KIND_F16>(A, lda, B, ldb, M, N, K, e, stream);
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
    return gemm::launch_auto<tc::KIND_TF32>(A, lda, B, ldb, M, N, K, e, stream);
}

}  // namespace vkf
