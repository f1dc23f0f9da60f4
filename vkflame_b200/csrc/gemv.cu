// gemv.cu — decode GEMV (M <= 8) over ggml block-quantised weights.
//
//   Y[m, n] = sum_k X[m, k] * dequant(W)[n, k]      X fp16, Y fp32 or fp16
//
// Replaces the reference's quantised mul_mat path, which dequantised the
// whole weight to a temporary fp32 buffer and ran a one-thread-per-output
// GEMM (shim/hip_runtime_shim.cpp:1102-1172, kernels/linear_fp16_fp32out.glsl).
// Here the packed blocks are read once from HBM and decoded in registers.
//
// Structure (per CTA, 160 threads):
//   warp 4      producer: one TMA bulk copy (cp.async.bulk) per weight row per
//               K-step into an NST-deep shared-memory ring, plus the K-step's
//               activations, completion tracked by mbarrier transaction bytes;
//               weights are marked L2 evict-first (streamed once).
//   warps 0..3  consumers: each owns 32 rows (two 16-row MMA groups) of the
//               128-row tile, decodes blocks into m16n8k16 fragments
//               (gemv_q.cuh) and accumulates in fp32 registers.  The MMA's
//               8-wide N dimension carries the M <= 8 batch columns.
// Scheduling is stream-K: the (tile, K-step) iteration space is split
// evenly over a grid sized to fill the GPU, so any N balances across all
// SMs.  A tile split between CTAs is finished by the last contributor,
// which sums the partials in CTA order (deterministic) from scratch memory.

#include "gemv_q.cuh"

#include <algorithm>

namespace vkf {
namespace gemv {

struct Args {
    const uint8_t *W;
    const uint8_t *X;  // fp16 activations, rows 16-byte aligned
    void *Y;
    int M, N, K;
    int64_t ldx_bytes;  // X row stride in bytes (multiple of 16)
    int64_t ldy;        // Y row stride in elements
    int64_t row_bytes;  // W row stride in bytes
    int T, S;           // tiles, K-steps per tile
    int64_t I;          // T * S
    int G;              // grid size
    float *ws;          // partial tiles: [G][2][1024] floats
    int *cnt;           // per-tile arrival counters (zero between launches)
    unsigned *err;
    int y_f16;
};

constexpr int NT = 160;
constexpr int PARTIAL_FLOATS = 4 * 2 * 32 * 4;  // warps x groups x lanes x 4

__device__ __forceinline__ int cta_of(int64_t i, const Args &a) { return (int)(((i + 1) * a.G - 1) / a.I); }
__device__ __forceinline__ int64_t first_iter(int c, const Args &a) { return (int64_t)c * a.I / a.G; }

__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

__device__ __forceinline__ void store_y(const Args &a, int m, int n, float v) {
    if (m < a.M && n < a.N) {
        if (a.y_f16) reinterpret_cast<__half *>(a.Y)[(int64_t)m * a.ldy + n] = __float2half_rn(v);
        else reinterpret_cast<float *>(a.Y)[(int64_t)m * a.ldy + n] = v;
    }
}

template <int QT, int NST>
__global__ void __launch_bounds__(NT, 2) gemv_kernel(const __grid_constant__ Args a) {
    using Gm = Geo<QT>;
    constexpr int QK = Fmt<QT>::QK, BB = Fmt<QT>::BB;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + NST * Gm::STAGE);
    uint64_t *empty = full + NST;
    int *flag = reinterpret_cast<int *>(empty + NST);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    const int64_t it0 = first_iter(cta, a), it1 = first_iter(cta + 1, a);

    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 4);
        }
        fence_mbar_init();
    }
    // Activation columns >= M are never copied: make them zero once.
    for (int s = 0; s < NST; ++s)
        for (int i = threadIdx.x; i < (8 - a.M) * (XP / 16); i += NT) {
            int col = a.M + i / (XP / 16);
            reinterpret_cast<uint4 *>(smem + s * Gm::STAGE + TILE_ROWS * Gm::RP + col * XP)[i % (XP / 16)] =
                make_uint4(0, 0, 0, 0);
        }
    __syncthreads();

    if (warp == 4) {
        // ---------------- producer ----------------
        const uint64_t pol_w = policy_evict_first(), pol_x = policy_evict_last();
        int n = 0;
        for (int64_t it = it0; it < it1; ++it, ++n) {
            const int s = n % NST;
            const uint32_t ph = (uint32_t)(n / NST) & 1u;
            if (n >= NST && !mbar_wait(&empty[s], ph ^ 1u, a.err)) break;
            const int tile = (int)(it / a.S), step = (int)(it % a.S);
            const int nval = min(KS, a.K - step * KS);
            const int wbytes = nval / QK * BB;
            uint8_t *st = smem + s * Gm::STAGE;
            uint32_t srow[4], ssz[4];
            const uint8_t *sbase[4];
            uint32_t mine = 0;
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int r = lane + 32 * i;
                const int row = tile * TILE_ROWS + r;
                ssz[i] = 0;
                srow[i] = r;
                if (row < a.N) {
                    const uint8_t *src = a.W + (int64_t)row * a.row_bytes + (int64_t)step * Gm::STEP_BYTES;
                    const uint32_t off = (uint32_t)((uintptr_t)src & 15);
                    sbase[i] = src - off;
                    ssz[i] = (off + wbytes + 15) & ~15u;
                    mine += ssz[i];
                }
            }
            uint32_t xsz = 0;
            const uint8_t *xsrc = nullptr;
            if (lane < a.M) {
                xsrc = a.X + (int64_t)lane * a.ldx_bytes + (int64_t)step * KS * 2;
                xsz = (nval * 2 + 15) & ~15u;
                mine += xsz;
            }
            uint32_t total = mine;
#pragma unroll
            for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
            if (lane == 0) mbar_arrive_expect_tx(&full[s], total);
            __syncwarp();
#pragma unroll
            for (int i = 0; i < 4; ++i)
                if (ssz[i]) bulk_g2s(st + srow[i] * Gm::RP, sbase[i], ssz[i], &full[s], pol_w);
            if (xsz) bulk_g2s(st + TILE_ROWS * Gm::RP + lane * XP, xsrc, xsz, &full[s], pol_x);
        }
        return;
    }

    // ---------------- consumers ----------------
    const int g = lane >> 2, t = lane & 3;
    float acc[2][4];
#pragma unroll
    for (int r = 0; r < 2; ++r) zero4(acc[r]);
    const int first_tile = (int)(it0 / a.S);
    // After a bounded wait gives up (error bit already set) the warp keeps
    // walking the same iterations without waiting or computing, so every
    // consumer warp still reaches the same named barriers.
    bool ok = true;
    int n = 0;
    for (int64_t it = it0; it < it1; ++it, ++n) {
        const int s = n % NST;
        const uint32_t ph = (uint32_t)(n / NST) & 1u;
        if (ok) ok = mbar_wait(&full[s], ph, a.err);
        const int tile = (int)(it / a.S), step = (int)(it % a.S);
        const int nval = min(KS, a.K - step * KS);
        const uint8_t *st = smem + s * Gm::STAGE;
        const uint8_t *xc = st + TILE_ROWS * Gm::RP + g * XP;
#pragma unroll
        for (int rg = 0; rg < 2; ++rg) {
            if (!ok) break;
            const int r_a = warp * 32 + rg * 16 + g, r_b = r_a + 8;
            const int64_t row_a = (int64_t)tile * TILE_ROWS + r_a, row_b = row_a + 8;
            const uintptr_t ga = (uintptr_t)a.W + row_a * a.row_bytes + (int64_t)step * Gm::STEP_BYTES;
            const uintptr_t gb = (uintptr_t)a.W + row_b * a.row_bytes + (int64_t)step * Gm::STEP_BYTES;
            Step<QT>::run(st + r_a * Gm::RP + (ga & 15), st + r_b * Gm::RP + (gb & 15), xc, t, nval / 32, acc[rg]);
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);

        if (step != a.S - 1 && it + 1 != it1) continue;

        // ---- tile epilogue ----
        const int64_t tb = (int64_t)tile * a.S;
        const bool whole = tb >= it0 && tb + a.S <= it1;
        float out[2][4];
        bool write = true;
        if (whole) {
#pragma unroll
            for (int r = 0; r < 2; ++r)
#pragma unroll
                for (int i = 0; i < 4; ++i) out[r][i] = acc[r][i];
        } else {
            const int slot = tile == first_tile ? 0 : 1;
            float *mine = a.ws + ((int64_t)cta * 2 + slot) * PARTIAL_FLOATS;
#pragma unroll
            for (int r = 0; r < 2; ++r)
                reinterpret_cast<float4 *>(mine)[(warp * 2 + r) * 32 + lane] =
                    make_float4(acc[r][0], acc[r][1], acc[r][2], acc[r][3]);
            __threadfence();
            consumer_bar();
            const int c_first = cta_of(tb, a), c_last = cta_of(tb + a.S - 1, a);
            if (threadIdx.x == 0) {
                int old = atomicAdd(&a.cnt[tile], 1);
                *flag = (old == c_last - c_first);
            }
            consumer_bar();
            write = *flag != 0;
            if (write) {
                __threadfence();
#pragma unroll
                for (int r = 0; r < 2; ++r) zero4(out[r]);
                for (int c = c_first; c <= c_last; ++c) {
                    const int cslot = (tile == (int)(first_iter(c, a) / a.S)) ? 0 : 1;
                    const float *p = a.ws + ((int64_t)c * 2 + cslot) * PARTIAL_FLOATS;
#pragma unroll
                    for (int r = 0; r < 2; ++r) {
                        float4 v = __ldcg(reinterpret_cast<const float4 *>(p) + (warp * 2 + r) * 32 + lane);
                        out[r][0] += v.x;
                        out[r][1] += v.y;
                        out[r][2] += v.z;
                        out[r][3] += v.w;
                    }
                }
                if (threadIdx.x == 0) atomicExch(&a.cnt[tile], 0);
            }
            consumer_bar();  // `flag` is reused by the next tile
        }
        if (write) {
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const int row = tile * TILE_ROWS + warp * 32 + r * 16 + g;
                store_y(a, 2 * t, row, out[r][0]);
                store_y(a, 2 * t + 1, row, out[r][1]);
                store_y(a, 2 * t, row + 8, out[r][2]);
                store_y(a, 2 * t + 1, row + 8, out[r][3]);
            }
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) zero4(acc[r]);
    }
}

template <int QT>
struct Launcher {
    static constexpr int NST = 4;
    static size_t smem_bytes() { return (size_t)NST * Geo<QT>::STAGE + 2 * NST * sizeof(uint64_t) + 16; }
    static int occupancy() {
        static int occ[64] = {0};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 64 && occ[dev]) return occ[dev];
        cudaFuncSetAttribute(gemv_kernel<QT, NST>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes());
        int o = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, gemv_kernel<QT, NST>, NT, smem_bytes());
        if (o < 1) o = 1;
        if (dev < 64) occ[dev] = o;
        return o;
    }
    static int launch(Args &a, int sms, cudaStream_t stream, void *scratch_override, size_t scratch_cap) {
        a.T = (a.N + TILE_ROWS - 1) / TILE_ROWS;
        a.S = (a.K + KS - 1) / KS;
        a.I = (int64_t)a.T * a.S;
        int64_t g = (int64_t)sms * occupancy();
        a.G = (int)std::min<int64_t>(g, a.I);
        size_t cnt_bytes = ((size_t)a.T * sizeof(int) + 255) & ~size_t(255);
        size_t need = cnt_bytes + (size_t)a.G * 2 * PARTIAL_FLOATS * sizeof(float);
        uint8_t *scr;
        if (scratch_override) {
            if (need > scratch_cap) return VKF_ERR_INVALID;
            scr = (uint8_t *)scratch_override;
        } else {
            scr = (uint8_t *)stream_scratch(stream, need);
            if (!scr) return VKF_ERR_NOMEM;
        }
        a.cnt = reinterpret_cast<int *>(scr);
        a.ws = reinterpret_cast<float *>(scr + cnt_bytes);
        gemv_kernel<QT, NST><<<a.G, NT, smem_bytes(), stream>>>(a);
        return check_launch();
    }
};

}  // namespace gemv

// Size of the scratch a GEMV call needs (counters + partial tiles).
size_t gemv_scratch_bytes(int N, int sms, int occ) {
    int T = (N + gemv::TILE_ROWS - 1) / gemv::TILE_ROWS;
    size_t cnt_bytes = ((size_t)T * sizeof(int) + 255) & ~size_t(255);
    return cnt_bytes + (size_t)sms * occ * 2 * gemv::PARTIAL_FLOATS * sizeof(float);
}

// X: fp16, rows 16-byte aligned (ldx_bytes multiple of 16).  Checked by caller.
int gemv_launch(int wtype, const void *W, const void *X, int64_t ldx_bytes, void *Y, int y_f16, int64_t ldy,
                int M, int N, int K, cudaStream_t stream, void *scratch, size_t scratch_cap) {
    DeviceState *ds = device_state();
    if (!ds) return VKF_ERR_NO_DEVICE;
    gemv::Args a{};
    a.W = (const uint8_t *)W;
    a.X = (const uint8_t *)X;
    a.Y = Y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.ldx_bytes = ldx_bytes;
    a.ldy = ldy;
    a.row_bytes = (int64_t)K / vkf_qtype_block_values(wtype) * vkf_qtype_block_bytes(wtype);
    a.err = ds->d_error;
    a.y_f16 = y_f16;
    const int sms = ds->sm_count;
    switch (wtype) {
    case VKF_DEQUANT_Q4_0: return gemv::Launcher<VKF_DEQUANT_Q4_0>::launch(a, sms, stream, scratch, scratch_cap);
    case VKF_DEQUANT_Q8_0: return gemv::Launcher<VKF_DEQUANT_Q8_0>::launch(a, sms, stream, scratch, scratch_cap);
    case VKF_DEQUANT_Q4_K: return gemv::Launcher<VKF_DEQUANT_Q4_K>::launch(a, sms, stream, scratch, scratch_cap);
    case VKF_DEQUANT_Q5_K: return gemv::Launcher<VKF_DEQUANT_Q5_K>::launch(a, sms, stream, scratch, scratch_cap);
    case VKF_DEQUANT_Q6_K: return gemv::Launcher<VKF_DEQUANT_Q6_K>::launch(a, sms, stream, scratch, scratch_cap);
    default: return VKF_ERR_UNSUPPORTED;
    }
}

}  // namespace vkf
