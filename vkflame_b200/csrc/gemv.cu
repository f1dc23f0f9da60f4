// gemv.cu — decode GEMV (M <= 8) over ggml block-quantised weights.
//
//   Y[m, n] = sum_k X[m, k] * dequant(W)[n, k]      X fp16, Y fp32 or fp16
//
// Replaces the reference's quantised mul_mat path, which dequantised the
// whole weight to a temporary fp32 buffer and ran a one-thread-per-output
// GEMM (shim/hip_runtime_shim.cpp:1102-1172, kernels/linear_fp16_fp32out.glsl).
// Here the packed blocks are read once from HBM and decoded in registers.
//
// Measured on B200 (copy microbenchmarks): streaming reads reach ~7.1 TB/s
// when each request run is kilobytes long, but a 128-row x 144..272-byte
// K-step (the natural MMA tile of a ggml row-major matrix) held DRAM to
// 2.6-4.4 TB/s.  The kernel therefore works on items of 16 rows x a K-range
// of up to ~3 KB of each row (the whole row for K = 5120 Q4_K):
//
//   warp CW       producer: one TMA bulk copy per row per item into an
//                 NST-deep ring, completion by mbarrier transaction bytes.
//   warps 0..CW-1 consumers: take the work units (one super-block, or eight
//                 32-value blocks, of the 16 rows) round-robin, decode them
//                 into m16n8k16 fragments (gemv_q.cuh: A = the 16 weight
//                 rows, N = the M <= 8 activation columns) and keep a per-warp
//                 fp32 accumulator; they never wait for each other, and the
//                 last warp to finish a row block reduces the CW partials.
//
// The activations X (M x K fp16) stay resident in shared memory for the whole
// CTA, stored permuted in fragment order; the fp32 sums of every 32-value
// sub-block (hi + lo fp16) are precomputed next to them for the K-quant
// min-term MMA.  Scheduling is stream-K over the (row block, K-range) items:
// the iteration space is split evenly over one or two CTAs per SM, a row block
// split between CTAs being finished by its last contributor, which sums the
// partials in CTA order (deterministic) from scratch memory.  Batch columns
// that do not fit the resident budget are processed in groups by the caller.
// Launches use programmatic dependent launch (griddepcontrol): a launch's
// prologue, and with static weights its weight streaming, overlaps the tail
// of the previous kernel on the stream.

#include "gemv_q.cuh"

#include <algorithm>
#include <cstdlib>

namespace vkf {
namespace gemv {

constexpr int CW = 8;                 // consumer warps
constexpr int NT = 32 * (CW + 1);
constexpr int NST = 3;                // ring depth
constexpr int ROW_BUDGET = 1600;      // max bytes of one row per item
constexpr int X_BUDGET = 80 * 1024;   // resident activations + sums
constexpr int SMEM_MAX = 227 * 1024;
// Two CTAs per SM when the activations are small: a CTA of the next launch
// on the stream can then stream its weights while this one drains.
constexpr int SMEM_HALF = 112 * 1024;
constexpr int X_HALF = 36 * 1024;
constexpr int ZERO_BYTES = 1024;      // zero activations / sums for columns >= M

struct Args {
    const uint8_t *W;
    const uint8_t *X;  // fp16, rows 16-byte aligned
    void *Y;
    int M, N, K;
    int64_t ldx_bytes, ldy, row_bytes;
    int units;         // 256-value units per row (the last may be partial for 32-value blocks)
    int upi;           // units per item (the last item of a row block may have fewer)
    int S;             // items per row block
    int T;             // row blocks of 16 rows
    int64_t I;         // T * S
    int G;             // grid
    int rpb;           // smem pitch of one row's bytes in a stage
    int xpr;           // smem pitch of one resident activation row
    int xsp;           // smem pitch of one column's sub-block sums
    int stage_bytes;
    float *ws;         // partials: [G][2][128] floats
    int *cnt;          // per-row-block arrival counters (zero between launches)
    unsigned *err;
    int y_f16;
    int prefetch;      // stream weights before the previous kernel on the stream completes
    int probe;         // debug (VKFLAME_GEMV_PROBE): 1 skips the decode (data path alone), 2 skips the
                       // copies and waits (decode alone, on whatever the ring holds)
};

__device__ __forceinline__ int cta_of(int64_t i, const Args &a) { return (int)(((i + 1) * a.G - 1) / a.I); }
__device__ __forceinline__ int64_t first_iter(int c, const Args &a) { return (int64_t)c * a.I / a.G; }
__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory"); }

__device__ __forceinline__ void store_y(const Args &a, int m, int n, float v) {
    if (m < a.M && n < a.N) {
        if (a.y_f16) reinterpret_cast<__half *>(a.Y)[(int64_t)m * a.ldy + n] = __float2half_rn(v);
        else reinterpret_cast<float *>(a.Y)[(int64_t)m * a.ldy + n] = v;
    }
}

template <int QT>
__global__ void __launch_bounds__(NT, 2) gemv_kernel(const __grid_constant__ Args a) {
    constexpr int QK = Fmt<QT>::QK, BB = Fmt<QT>::BB, PARTS = Fmt<QT>::PARTS;
    constexpr int UB = (256 / QK) * BB;  // bytes of one 256-value unit of a row
    constexpr bool KQ = QT == VKF_DEQUANT_Q4_K || QT == VKF_DEQUANT_Q5_K;  // has a min term
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *xs = smem;                                       // M x xpr, permuted fp16
    uint8_t *sums = xs + a.M * a.xpr;                         // M x xsp (K-quants)
    uint8_t *zero = sums + a.M * a.xsp;                       // ZERO_BYTES of zeros
    uint8_t *ring = zero + ZERO_BYTES;                        // NST x stage_bytes
    uint64_t *full = reinterpret_cast<uint64_t *>(ring + NST * a.stage_bytes);
    uint64_t *empty = full + NST;
    int *redcnt = reinterpret_cast<int *>(empty + NST);       // NST + 1 arrival counters
    float *red = reinterpret_cast<float *>(empty + NST + 2);  // (NST + 1) x CW x 32 x 4

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    const int64_t it0 = first_iter(cta, a), it1 = first_iter(cta + 1, a);
    // Programmatic dependent launch: let the next kernel on the stream start
    // its prologue now; everything this kernel reads or writes that another
    // kernel may touch (X, Y, the scratch) waits for the previous kernel.
    asm volatile("griddepcontrol.launch_dependents;");

    for (int i = threadIdx.x; i < ZERO_BYTES / 16; i += NT) reinterpret_cast<uint4 *>(zero)[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        for (int r = 0; r <= NST; ++r) redcnt[r] = 0;
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == CW) {
        // ---------------- producer ----------------
        // Weights that no kernel writes (a.prefetch) are streamed at once;
        // otherwise the producer too waits for the previous kernel.
        if (!a.prefetch) asm volatile("griddepcontrol.wait;" ::: "memory");
        if (a.probe >= 2) return;
        int n = 0;
        for (int64_t it = it0; it < it1; ++it, ++n) {
            const int s = n % NST;
            const uint32_t ph = (uint32_t)(n / NST) & 1u;
            if (n >= NST && !mbar_wait(&empty[s], ph ^ 1u, a.err)) break;
            const int tile = (int)(it / a.S), step = (int)(it - (int64_t)tile * a.S);
            const int u0 = step * a.upi, nu = min(a.upi, a.units - u0);
            // Bytes of this item's units in one row (a partial last unit of a
            // 32-value-block format holds only the blocks that exist), widened
            // to whole 16-byte granules: a 16-byte aligned granule never
            // crosses a page, so the few bytes read either side are mapped.
            const int64_t b0 = (int64_t)u0 * UB;
            const int64_t b1 = (int64_t)(u0 + nu) * UB < a.row_bytes ? (int64_t)(u0 + nu) * UB : a.row_bytes;
            const int row = tile * 16 + lane;
            uint32_t sz = 0;
            const uint8_t *src = nullptr;
            if (lane < 16 && row < a.N) {
                const uint8_t *p = a.W + (int64_t)row * a.row_bytes + b0;
                const uint32_t off = (uint32_t)((uintptr_t)p & 15);
                src = p - off;
                sz = (uint32_t)((off + (b1 - b0) + 15) & ~15);
            }
            uint32_t total = sz;
#pragma unroll
            for (int o = 16; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
            if (lane == 0) mbar_arrive_expect_tx(&full[s], total);
            __syncwarp();
            if (sz) bulk_g2s(ring + s * a.stage_bytes + lane * a.rpb, src, sz, &full[s]);
        }
        return;
    }

    // ---------------- consumers ----------------
    asm volatile("griddepcontrol.wait;" ::: "memory");
    // Resident activations, permuted (x0, x2, x1, x3) per group of four.
    // Loads are batched through registers (read-only path) so their
    // latencies overlap instead of serialising behind the shared stores.
    {
        const int groups = a.K / 4, total = a.M * groups;
        constexpr int B = 8;
        for (int i0 = threadIdx.x; i0 < total; i0 += B * CW * 32) {
            uint2 v[B];
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const int i = i0 + b * CW * 32;
                if (i < total) {
                    const int m = i / groups, q = i - m * groups;
                    v[b] = __ldg(reinterpret_cast<const uint2 *>(a.X + (int64_t)m * a.ldx_bytes) + q);
                }
            }
#pragma unroll
            for (int b = 0; b < B; ++b) {
                const int i = i0 + b * CW * 32;
                if (i < total) {
                    const int m = i / groups, q = i - m * groups;
                    *reinterpret_cast<uint2 *>(xs + m * a.xpr + q * 8) =
                        make_uint2(prmt(v[b].x, v[b].y, 0x5410), prmt(v[b].x, v[b].y, 0x7632));
                }
            }
        }
    }
    consumer_bar();
    if constexpr (KQ) {
        // fp32 sum of each 32-value sub-block, split hi + lo fp16, laid out as
        // the min MMA's B fragment: [super-block][t] = (hi 2t, 2t+1 | lo 2t, 2t+1)
        const int nsub = a.K / 32;
        for (int i = threadIdx.x; i < a.M * nsub; i += CW * 32) {
            const int m = i / nsub, j = i - m * nsub;
            const uint4 *xr = reinterpret_cast<const uint4 *>(xs + m * a.xpr + j * 64);
            float part[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 v = xr[c];
                const uint32_t w[4] = {v.x, v.y, v.z, v.w};
                float s2 = 0.f;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[e]));
                    s2 += f.x + f.y;
                }
                part[c] = s2;
            }
            const float sum = (part[0] + part[1]) + (part[2] + part[3]);
            const __half hi = __float2half_rn(sum);
            const __half lo = __float2half_rn(sum - __half2float(hi));
            __half *o = reinterpret_cast<__half *>(sums + m * a.xsp + (j / 8) * 32 + ((j % 8) / 2) * 8) + (j & 1);
            o[0] = hi;
            o[2] = lo;
        }
        consumer_bar();
    }

    const int g = lane >> 2, t = lane & 3;
    const uint8_t *xg = g < a.M ? xs + g * a.xpr : nullptr;
    const uint8_t *sg = g < a.M ? sums + g * a.xsp : nullptr;
    // After a bounded wait gives up (error bit already set) the warp keeps
    // walking the same iterations without waiting or computing, so every
    // consumer warp still reaches the same named barriers.
    bool ok = true;
    float acc[4];
    zero4(acc);
    const int first_tile = (int)(it0 / a.S);
    // Warps take the units of the CTA's item sequence round-robin (unit i of
    // the sequence goes to warp i mod CW), never waiting for each other: a
    // warp releases a ring slot when done with it, and at the end of a row
    // block leaves its partial in one of NST + 1 reduction buffers (a warp
    // can run at most NST items ahead); the last warp to arrive reduces.
    int ubase = 0;  // units of this CTA's earlier items, mod CW
    int tiles_done = 0;
    int n = 0;
    for (int64_t it = it0; it < it1; ++it, ++n) {
        const int s = n % NST;
        const uint32_t ph = (uint32_t)(n / NST) & 1u;
        if (ok && a.probe < 2) ok = mbar_wait(&full[s], ph, a.err);
        const int tile = (int)(it / a.S), step = (int)(it - (int64_t)tile * a.S);
        const int u0 = step * a.upi, nu = min(a.upi, a.units - u0);
        if (ok && (a.probe == 0 || a.probe == 2)) {
            const uint8_t *st = ring + s * a.stage_bytes;
            const int64_t row_a = (int64_t)tile * 16 + g, row_b = row_a + 8;
            const uintptr_t ga = (uintptr_t)a.W + row_a * a.row_bytes + (int64_t)u0 * UB;
            const uintptr_t gb = (uintptr_t)a.W + row_b * a.row_bytes + (int64_t)u0 * UB;
            const uint8_t *ra = st + g * a.rpb + (ga & 15), *rb = st + (g + 8) * a.rpb + (gb & 15);
            int u = warp - ubase;
            if (u < 0) u += CW;
            for (; u < nu; u += CW) {
                const int kv = (u0 + u) * 256;
                const int nblk = min(8, (a.K - kv) / 32);
                const uint8_t *xc = xg ? xg + kv * 2 : zero;
                const uint8_t *xsum = sg ? sg + (u0 + u) * 32 : zero;
                Step<QT>::run(ra + u * UB, rb + u * UB, xc, xsum, t, 0, nblk, acc);
            }
        }
        ubase = (ubase + nu) % CW;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);

        if (step != a.S - 1 && it + 1 != it1) continue;

        // ---- row-block epilogue: the last warp to arrive reduces ----
        const int rbuf = tiles_done % (NST + 1);
        ++tiles_done;
        float *rbase = red + rbuf * CW * 128;
        reinterpret_cast<float4 *>(rbase)[warp * 32 + lane] = make_float4(acc[0], acc[1], acc[2], acc[3]);
        zero4(acc);
        __threadfence_block();
        __syncwarp();
        int last = 0;
        if (lane == 0) last = atomicAdd(&redcnt[rbuf], 1) == CW - 1;
        last = __shfl_sync(0xffffffffu, last, 0);
        if (!last) continue;
        __threadfence_block();
        float o[4] = {0.f, 0.f, 0.f, 0.f};
        for (int w = 0; w < CW; ++w) {
            const float4 v = reinterpret_cast<const float4 *>(rbase)[w * 32 + lane];
            o[0] += v.x;
            o[1] += v.y;
            o[2] += v.z;
            o[3] += v.w;
        }
        __syncwarp();
        if (lane == 0) redcnt[rbuf] = 0;
        const int64_t tb = (int64_t)tile * a.S;
        const bool whole = tb >= it0 && tb + a.S <= it1;
        bool write = true;
        if (!whole) {
            const int slot = tile == first_tile ? 0 : 1;
            reinterpret_cast<float4 *>(a.ws + ((int64_t)cta * 2 + slot) * 128)[lane] = make_float4(o[0], o[1], o[2], o[3]);
            __threadfence();
            __syncwarp();
            const int c_first = cta_of(tb, a), c_last = cta_of(tb + a.S - 1, a);
            int fin = 0;
            if (lane == 0) fin = atomicAdd(&a.cnt[tile], 1) == c_last - c_first;
            fin = __shfl_sync(0xffffffffu, fin, 0);
            write = fin != 0;
            if (write) {
                __threadfence();
                zero4(o);
#pragma unroll 4
                for (int c = c_first; c <= c_last; ++c) {
                    const int cslot = (tile == (int)(first_iter(c, a) / a.S)) ? 0 : 1;
                    const float4 v =
                        __ldcg(reinterpret_cast<const float4 *>(a.ws + ((int64_t)c * 2 + cslot) * 128) + lane);
                    o[0] += v.x;
                    o[1] += v.y;
                    o[2] += v.z;
                    o[3] += v.w;
                }
                if (lane == 0) atomicExch(&a.cnt[tile], 0);
            }
        }
        if (write) {
            const int row = tile * 16 + g;
            store_y(a, 2 * t, row, o[0]);
            store_y(a, 2 * t + 1, row, o[1]);
            store_y(a, 2 * t, row + 8, o[2]);
            store_y(a, 2 * t + 1, row + 8, o[3]);
        }
    }
}

template <int QT>
struct Launcher {
    static constexpr int QK = Fmt<QT>::QK, BB = Fmt<QT>::BB;
    static constexpr int UB = (256 / QK) * BB;
    static constexpr bool KQ = QT == VKF_DEQUANT_Q4_K || QT == VKF_DEQUANT_Q5_K;
    static int launch(Args &a, int sms, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap) {
        a.units = (a.K + 255) / 256;
        a.xpr = ((a.K * 2 + 95) / 128) * 128 + 32;  // pitch = 8 banks mod 32: conflict-free fragment loads
        a.xsp = KQ ? ((a.K / 256) * 32 + 15) / 16 * 16 : 0;
        const int fixed = a.M * (a.xpr + a.xsp) + ZERO_BYTES + 2 * NST * 8 + 16 + (NST + 1) * CW * 32 * 16;
        const int budget = a.M * (a.xpr + a.xsp) <= X_HALF ? SMEM_HALF : SMEM_MAX;
        const int row_avail = (budget - fixed) / (NST * 16) - 32;  // room for padding and misalignment
        const int umax = std::min(ROW_BUDGET, row_avail) / UB;
        if (umax < 1) return VKF_ERR_UNSUPPORTED;
        a.S = (a.units + umax - 1) / umax;
        a.upi = (a.units + a.S - 1) / a.S;
        a.S = (a.units + a.upi - 1) / a.upi;
        a.T = (a.N + 15) / 16;
        a.I = (int64_t)a.T * a.S;
        const int ng = ((a.upi * UB + 15) / 16 + 1) | 1;  // odd granule count: rows 4 banks apart
        a.rpb = ng * 16;
        a.stage_bytes = 16 * a.rpb;
        const size_t smem = (size_t)fixed + NST * (size_t)a.stage_bytes;
        if (smem > (size_t)budget) return VKF_ERR_UNSUPPORTED;
        static bool attr_set[64] = {false};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 64 && !attr_set[dev]) {
            cudaFuncSetAttribute(gemv_kernel<QT>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX);
            attr_set[dev] = true;
        }
        a.G = (int)std::max<int64_t>(1, std::min<int64_t>((int64_t)sms * (budget == SMEM_HALF ? 2 : 1), a.I));
        if ((size_t)a.G * 2 * 128 > ws_cap || (size_t)a.T > cnt_cap) return VKF_ERR_INVALID;
        a.ws = ws;
        a.cnt = cnt;
        static const int probe = [] { const char *e = getenv("VKFLAME_GEMV_PROBE"); return e ? atoi(e) : 0; }();
        a.probe = probe;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(a.G);
        cfg.blockDim = dim3(NT);
        cfg.dynamicSmemBytes = smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        cudaLaunchKernelEx(&cfg, gemv_kernel<QT>, a);
        return check_launch();
    }
};

}  // namespace gemv

// Batch columns per launch so the resident activations fit the budget.
int gemv_cols_per_launch(int K) {
    const size_t per = (size_t)K * 2 + 160 + (size_t)K / 8;
    return (int)std::max<size_t>(1, std::min<size_t>(8, gemv::X_BUDGET / per));
}
size_t gemv_counters(int N) { return (size_t)(N + 15) / 16; }
size_t gemv_ws_floats(int sms) { return (size_t)sms * 2 * 2 * 128; }

// X: fp16, rows 16-byte aligned (ldx_bytes multiple of 16).  Checked by caller.
int gemv_launch(int wtype, const void *W, const void *X, int64_t ldx_bytes, void *Y, int y_f16, int64_t ldy, int M,
                int N, int K, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap, int prefetch) {
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
    a.prefetch = prefetch;
    const int sms = ds->sm_count;
    switch (wtype) {
    case VKF_DEQUANT_Q4_0: return gemv::Launcher<VKF_DEQUANT_Q4_0>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q8_0: return gemv::Launcher<VKF_DEQUANT_Q8_0>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q4_K: return gemv::Launcher<VKF_DEQUANT_Q4_K>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q5_K: return gemv::Launcher<VKF_DEQUANT_Q5_K>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q6_K: return gemv::Launcher<VKF_DEQUANT_Q6_K>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    default: return VKF_ERR_UNSUPPORTED;
    }
}

// Same launch with the SM count and the kernel error word supplied by the
// caller, so that nothing here allocates device memory (the allocation-free
// entry point in noalloc.cu).
int gemv_launch_raw(int wtype, const void *W, const void *X, int64_t ldx_bytes, void *Y, int y_f16, int64_t ldy,
                    int M, int N, int K, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap,
                    int sms, unsigned *err) {
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
    a.err = err;
    a.y_f16 = y_f16;
    a.prefetch = 0;
    switch (wtype) {
    case VKF_DEQUANT_Q4_0: return gemv::Launcher<VKF_DEQUANT_Q4_0>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q8_0: return gemv::Launcher<VKF_DEQUANT_Q8_0>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q4_K: return gemv::Launcher<VKF_DEQUANT_Q4_K>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q5_K: return gemv::Launcher<VKF_DEQUANT_Q5_K>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q6_K: return gemv::Launcher<VKF_DEQUANT_Q6_K>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    default: return VKF_ERR_UNSUPPORTED;
    }
}

}  // namespace vkf
