// gemv.cu — decode GEMV (M <= 8) over ggml block-quantised weights.
//
//   Y[m, n] = sum_k X[m, k] * dequant(W)[n, k]      X fp16, Y fp32 or fp16
//
// Replaces the reference's quantised mul_mat path, which dequantised the
// whole weight to a temporary fp32 buffer and ran a one-thread-per-output
// GEMM (shim/hip_runtime_shim.cpp:1102-1172, kernels/linear_fp16_fp32out.glsl).
// Here the packed blocks are read once from HBM and decoded in registers.
//
// Work items are 16 rows x a K-range of each row (a run of ~0.5-1.6 KB per
// row: short K-steps of many rows hold DRAM well below its streaming rate on
// B200).  One CTA per SM:
//
//   warp CW       producer: one TMA bulk copy per row per item into an
//                 NST-deep ring, completion by mbarrier transaction bytes;
//                 with static weights it starts before the previous kernel
//                 on the stream has finished (programmatic dependent launch).
//   warps 0..CW-1 consumers: take the 256-value units of the item sequence
//                 round-robin, decode them into m16n8k16 fragments
//                 (gemv_q.cuh) and keep a per-warp fp32 accumulator for the
//                 current row block.  At the end of a row block a warp parks
//                 its partial in the block's shared-memory slot and goes on;
//                 the last warp to arrive (one shared atomic per warp) sums
//                 the slot in warp order (deterministic) and stores Y.  No
//                 consumer ever waits for another.
//
// The activations stay resident in shared memory for the whole CTA, stored
// in the decode's fragment order, with the K-quant sub-block sums beside
// them; one pass over X builds both.  The (row block, K-range) items are
// split evenly over the CTAs; a row block cut between CTAs (at most the
// first and the last of each CTA) is finished by its last contributor, which
// sums the partials in CTA order from scratch memory.

#include "gemv_q.cuh"

#include <algorithm>
#include <cstdlib>

namespace vkf {
namespace gemv {

constexpr int NST_MAX = 8;            // ring depth cap
constexpr int ROW_BUDGET = 4400;      // max bytes of one row per item
constexpr int SMEM_MAX = 227 * 1024;
constexpr int X_BUDGET = 120 * 1024;  // resident activations + sums
constexpr int MAX_SLOTS = NST_MAX + 2; // per-warp row-block partial slots

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
    int I;             // T * S
    int G;             // grid
    int nst;           // ring depth
    int rpb;           // smem pitch of one row's bytes in a stage
    int stage_bytes;
    int xpr;           // smem pitch of one resident activation column
    int xsp;           // smem pitch of one column's sub-block sums
    int slots;         // partial slots (row blocks in flight)
    int off_sums, off_ring, off_red, off_bar;
    float *ws;         // partials of cut row blocks: [G][2][16 * M]
    int *cnt;          // per-row-block arrival counters (zero between launches)
    unsigned *err;
    int y_f16;
    int prefetch;      // stream weights before the previous kernel on the stream completes
};

__device__ __forceinline__ int first_item(int c, const Args &a) { return (int)((int64_t)c * a.I / a.G); }
__device__ __forceinline__ int cta_of_item(int i, const Args &a) {
    return (int)(((int64_t)(i + 1) * a.G - 1) / a.I);
}
template <int CW>
__device__ __forceinline__ void consumer_bar() {
    asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory");
}

__device__ __forceinline__ void store_y(const Args &a, int m, int n, float v) {
    if (a.y_f16) reinterpret_cast<__half *>(a.Y)[(int64_t)m * a.ldy + n] = __float2half_rn(v);
    else reinterpret_cast<float *>(a.Y)[(int64_t)m * a.ldy + n] = v;
}

// Resident activations: one thread per (column, 32-value sub-block) reads the
// 64 source bytes, stores them in fragment order (groups of four permuted
// (x0, x2, x1, x3); owned layout: swizzled granules) and, for the K-quants,
// their fp32 sum: split into hi + lo fp16 in the min-term MMA's B layout
// [super-block][t] = (hi 2t, hi 2t+1, lo 2t, lo 2t+1), or (M = 1 column
// form) as fp32 in the [super-block][t][2] order of the thread's sub-blocks.
template <bool OWN, bool KQ, bool COLS, int NTC>
__device__ __forceinline__ void load_activations(const Args &a, uint8_t *xs, uint8_t *sums) {
    const int nsb = a.K / 32, jobs = a.M * nsb;
    for (int j = threadIdx.x; j < jobs; j += NTC) {
        const int m = j / nsb, sb = j - m * nsb;
        const uint4 *src = reinterpret_cast<const uint4 *>(a.X + (int64_t)m * a.ldx_bytes + sb * 64);
        uint4 v[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) v[c] = __ldg(src + c);
        uint8_t *col = xs + m * a.xpr;
        const int v0 = sb * 32;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t w[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint32_t lo = w[2 * h], hi = w[2 * h + 1];  // values (x0 x1), (x2 x3)
                const uint2 p = make_uint2(prmt(lo, hi, 0x5410), prmt(lo, hi, 0x7632));
                const int v4 = v0 + 8 * c + 4 * h;  // first value of the group
                const int off = OWN ? (v4 >> 8) * 512 + owned_group_offset(v4 & 255) : v4 * 2;
                *reinterpret_cast<uint2 *>(col + off) = p;
            }
        }
        if constexpr (KQ) {
            float part[4];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t w[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
                float s2 = 0.f;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&w[e]));
                    s2 += f.x + f.y;
                }
                part[c] = s2;
            }
            const float sum = (part[0] + part[1]) + (part[2] + part[3]);
            if constexpr (COLS) {
                reinterpret_cast<float *>(sums + m * a.xsp + (sb / 8) * 32)[m1_sum_slot(sb % 8)] = sum;
                continue;
            }
            const __half hi = __float2half_rn(sum);
            const __half lo = __float2half_rn(sum - __half2float(hi));
            __half *o = reinterpret_cast<__half *>(sums + m * a.xsp + (sb / 8) * 32 + ((sb % 8) / 2) * 8) + (sb & 1);
            o[0] = hi;
            o[2] = lo;
        }
    }
}

template <int QT, int CW, bool M1>
__global__ void __launch_bounds__(32 * (CW + 1), 1) gemv_kernel(const __grid_constant__ Args a) {
    constexpr int NTC = 32 * CW;
    constexpr int QK = Fmt<QT>::QK, BB = Fmt<QT>::BB;
    constexpr int UB = (256 / QK) * BB;  // bytes of one 256-value unit of a row
    constexpr bool KQ = QT == VKF_DEQUANT_Q4_K || QT == VKF_DEQUANT_Q5_K;
    constexpr bool OWN = Step<QT>::OWNED;
    constexpr bool COLS = M1 && KQ;  // sub-block-column decode (StepK1)
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *xs = smem;
    uint8_t *sums = smem + a.off_sums;
    uint8_t *ring = smem + a.off_ring;
    float *red = reinterpret_cast<float *>(smem + a.off_red);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + a.off_bar);
    uint64_t *empty = full + NST_MAX;
    int *slotcnt = reinterpret_cast<int *>(empty + NST_MAX);  // arrivals per reduction slot

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    const int it0 = first_item(cta, a), it1 = first_item(cta + 1, a);
    // Programmatic dependent launch: the next kernel on the stream may start
    // its prologue now; everything this kernel reads or writes that another
    // kernel may touch (X, Y, the scratch) waits for the previous kernel.
    asm volatile("griddepcontrol.launch_dependents;");
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        fence_mbar_init();
    }
    if (threadIdx.x < MAX_SLOTS) slotcnt[threadIdx.x] = 0;
    __syncthreads();

    if (warp == CW) {
        // ---------------- producer ----------------
        // Weights that no kernel writes (a.prefetch) are streamed at once;
        // otherwise the producer too waits for the previous kernel.
        if (!a.prefetch) asm volatile("griddepcontrol.wait;" ::: "memory");
        int tile = it0 / a.S, step = it0 - tile * a.S, s = 0;
        uint32_t ph = 0;
        for (int it = it0, n = 0; it < it1; ++it, ++n) {
            if (n >= a.nst && !mbar_wait(&empty[s], ph ^ 1u, a.err)) break;
            const int u0 = step * a.upi, nu = min(a.upi, a.units - u0);
            // Bytes of this item's units in one row (a partial last unit of a
            // 32-value-block format holds only the blocks that exist), widened
            // to whole 16-byte granules: a 16-byte aligned granule never
            // crosses a page, so the few bytes read either side are mapped.
            const int64_t b0 = (int64_t)u0 * UB;
            const int64_t b1 = min((int64_t)(u0 + nu) * UB, a.row_bytes);
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
            for (int o = 8; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
            if (lane == 0) mbar_arrive_expect_tx(&full[s], total);
            __syncwarp();
            if (sz) bulk_g2s(ring + s * a.stage_bytes + lane * a.rpb, src, sz, &full[s]);
            if (++step == a.S) {
                step = 0;
                ++tile;
            }
            if (++s == a.nst) {
                s = 0;
                ph ^= 1u;
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    asm volatile("griddepcontrol.wait;" ::: "memory");
    load_activations<OWN, KQ, COLS, NTC>(a, xs, sums);
    consumer_bar<CW>();

    const int g = lane >> 2, t = lane & 3;
    // Lanes of columns >= M read a real column (their outputs are dropped),
    // which keeps every fragment load a broadcast or conflict-free.
    const int xcol = g % a.M;
    const uint8_t *xg = xs + xcol * a.xpr;
    const uint8_t *sg = sums + xcol * a.xsp;
    const int rows16m = 16 * a.M;
    // After a bounded wait gives up (error bit already set) the warp keeps
    // walking the same items without waiting or computing, so every consumer
    // warp still reaches the same barriers.
    bool ok = true;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int tile = it0 / a.S, step = it0 - tile * a.S, s = 0;
    uint32_t ph = 0;
    int ubase = 0;  // units of this CTA's earlier items, mod CW
    int slot = 0, done_tile = tile;
    const int first_tile = tile;
    for (int it = it0; it < it1; ++it) {
        if (ok) ok = mbar_wait(&full[s], ph, a.err);
        const int u0 = step * a.upi, nu = min(a.upi, a.units - u0);
        if (ok) {
            const uint8_t *st = ring + s * a.stage_bytes;
            const int64_t row_a = (int64_t)tile * 16 + g;
            const uintptr_t ga = (uintptr_t)a.W + row_a * a.row_bytes + (int64_t)u0 * UB;
            const uintptr_t gb = ga + 8 * a.row_bytes;
            const uint8_t *ra = st + g * a.rpb + (ga & 15), *rb = st + (g + 8) * a.rpb + (gb & 15);
            int u = warp - ubase;
            if (u < 0) u += CW;
            for (; u < nu; u += CW) {
                const int unit = u0 + u;
                if constexpr (COLS) {
                    StepK1<QT == VKF_DEQUANT_Q5_K>::run(ra + u * UB, rb + u * UB, xs + unit * 512, g == t, g == t + 4,
                                                        reinterpret_cast<const float *>(sums + unit * 32), t, acc);
                } else {
                    const int nblk = QK == 32 ? min(8, (a.K - unit * 256) / 32) : 8;
                    Step<QT>::run(ra + u * UB, rb + u * UB, xg + unit * 512, sg + unit * 32, t, nblk, acc);
                }
            }
        }
        ubase += nu;
        while (ubase >= CW) ubase -= CW;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        if (++s == a.nst) {
            s = 0;
            ph ^= 1u;
        }
        const bool tile_end = step == a.S - 1 || it + 1 == it1;
        if (++step == a.S) {
            step = 0;
            ++tile;
        }
        if (!tile_end) continue;

        if constexpr (COLS) StepK1<QT == VKF_DEQUANT_Q5_K>::finish(acc);
        // Park this warp's partial of the finished row block in the block's
        // slot; the last warp to arrive reduces the slot in warp order
        // (deterministic) while the others go on decoding.  A warp runs at
        // most nst items ahead of the slowest, so nst + 2 slots never alias.
        float *p = red + (slot * CW + warp) * rows16m;
        {
            const int c0 = 2 * t, c1 = 2 * t + 1;
            if (c0 < a.M) {
                p[g * a.M + c0] = acc[0];
                p[(g + 8) * a.M + c0] = acc[2];
            }
            if (c1 < a.M) {
                p[g * a.M + c1] = acc[1];
                p[(g + 8) * a.M + c1] = acc[3];
            }
            acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        }
        const int tb = done_tile, sl = slot;
        ++done_tile;
        if (++slot == a.slots) slot = 0;
        __syncwarp();
        int last = 0;
        if (lane == 0) {
            __threadfence_block();
            last = atomicAdd(&slotcnt[sl], 1) == CW - 1;
            if (last) __threadfence_block();
        }
        if (!__shfl_sync(0xffffffffu, last, 0)) continue;

        const float *q = red + sl * CW * rows16m;
        const bool whole = tb * a.S >= it0 && (tb + 1) * a.S <= it1;
        float o[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int rc = lane + 32 * j;
            o[j] = 0.f;
            if (rc < rows16m) {
#pragma unroll 4
                for (int w = 0; w < CW; ++w) o[j] += q[w * rows16m + rc];
            }
        }
        __syncwarp();
        if (lane == 0) slotcnt[sl] = 0;
        if (whole) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int rc = lane + 32 * j, r = rc / a.M, c = rc - r * a.M;
                if (rc < rows16m && tb * 16 + r < a.N) store_y(a, c, tb * 16 + r, o[j]);
            }
            continue;
        }
        // A row block cut between CTAs: publish this CTA's partial; the last
        // contributor to arrive sums all partials in CTA order and stores Y.
        const int which = tb == first_tile ? 0 : 1;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int rc = lane + 32 * j;
            if (rc < rows16m) a.ws[((int64_t)cta * 2 + which) * rows16m + rc] = o[j];
        }
        const int c_first = cta_of_item(tb * a.S, a), c_last = cta_of_item((tb + 1) * a.S - 1, a);
        __syncwarp();
        int fin = 0;
        if (lane == 0) {
            __threadfence();
            fin = atomicAdd(&a.cnt[tb], 1) == c_last - c_first;
            if (fin) __threadfence();
        }
        if (!__shfl_sync(0xffffffffu, fin, 0)) continue;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int rc = lane + 32 * j;
            if (rc >= rows16m) continue;
            float v = 0.f;
            for (int c = c_first; c <= c_last; ++c) {
                const int wc = tb == first_item(c, a) / a.S ? 0 : 1;
                v += __ldcg(a.ws + ((int64_t)c * 2 + wc) * rows16m + rc);
            }
            const int r = rc / a.M, col = rc - r * a.M;
            if (tb * 16 + r < a.N) store_y(a, col, tb * 16 + r, v);
        }
        if (lane == 0) a.cnt[tb] = 0;
    }
}

template <int QT, int CW, bool M1>
struct Launcher {
    static constexpr int QK = Fmt<QT>::QK, BB = Fmt<QT>::BB;
    static constexpr int UB = (256 / QK) * BB;
    static constexpr bool KQ = QT == VKF_DEQUANT_Q4_K || QT == VKF_DEQUANT_Q5_K;
    static constexpr bool OWN = Step<QT>::OWNED;
    static constexpr int NT = 32 * (CW + 1);

    static int launch(Args &a, int sms, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap) {
        auto up = [](int64_t v, int64_t m) { return (v + m - 1) / m * m; };
        a.units = (a.K + 255) / 256;
        // Column pitches: the owned layout's 16-byte fragment loads want
        // columns 64 bytes apart mod 128 banks-wise, the plain layout's
        // 8-byte loads 32 bytes.
        a.xpr = (int)up((int64_t)a.units * 512, 128) + (OWN ? 64 : 32);
        a.xsp = KQ ? (int)up((int64_t)a.units * 32, 16) : 0;
        a.off_sums = a.M * a.xpr;
        const int x_end = (int)up(a.off_sums + (int64_t)a.M * a.xsp, 128);
        if (x_end > X_BUDGET) return VKF_ERR_UNSUPPORTED;
        const int rows16m = 16 * a.M;
        const int slot_bytes = CW * rows16m * 4;
        const int bar_bytes = 2 * NST_MAX * 8 + MAX_SLOTS * 4;
        const int avail = SMEM_MAX - x_end - bar_bytes - 128;
        a.T = (a.N + 15) / 16;

        // Units per item: whole rows when a row fits the budget (a 16-row
        // item is then one contiguous range of the matrix, which DRAM streams
        // at full rate; K-ranges of ~1.5 KB per row measured ~40% slower), a
        // K-split only as far as the row length requires.  A short N (fewer
        // row blocks than SMs) is not split further: the cross-CTA fixups of
        // cut row blocks cost more than the idle SMs (measured).
        const int upi_max = std::max(1, std::min(a.units, ROW_BUDGET / UB));
        a.S = (a.units + upi_max - 1) / upi_max;
        a.upi = (a.units + a.S - 1) / a.S;
        for (;;) {
            const int ng = ((a.upi * UB + 15) / 16 + 1) | 1;  // odd granule count: rows 16 banks apart
            a.rpb = ng * 16;
            a.stage_bytes = 16 * a.rpb;
            a.nst = std::min(NST_MAX, (avail - 2 * slot_bytes) / (a.stage_bytes + slot_bytes));
            if (a.nst >= 2 || a.upi == 1) break;
            a.upi = std::max(1, a.upi / 2);
            a.S = (a.units + a.upi - 1) / a.upi;
            a.upi = (a.units + a.S - 1) / a.S;
        }
        if (a.nst < 2) return VKF_ERR_UNSUPPORTED;
        if ((int64_t)a.T * a.S > (int64_t)1 << 30) return VKF_ERR_UNSUPPORTED;
        a.I = a.T * a.S;
        a.slots = a.nst + 2;
        const int red_bytes = (int)up((int64_t)a.slots * slot_bytes, 128);
        a.off_ring = x_end;
        a.off_red = a.off_ring + a.nst * a.stage_bytes;
        a.off_bar = a.off_red + red_bytes;
        const size_t smem = (size_t)a.off_bar + bar_bytes;
        static bool attr_set[64] = {false};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 64 && !attr_set[dev]) {
            cudaFuncSetAttribute(gemv_kernel<QT, CW, M1>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_MAX);
            attr_set[dev] = true;
        }
        a.G = std::max(1, std::min(sms, a.I));
        if ((size_t)a.G * 2 * rows16m > ws_cap || (size_t)a.T > cnt_cap) return VKF_ERR_INVALID;
        a.ws = ws;
        a.cnt = cnt;
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
        cudaLaunchKernelEx(&cfg, gemv_kernel<QT, CW, M1>, a);
        return check_launch();
    }
};

// 8 consumer warps: with 16, each warp decodes fewer units per item and the
// per-item overhead grows faster than the latency hiding gains (measured).
constexpr int CW_DEFAULT = 8;

template <int QT>
static int launch_q(Args &a, int sms, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap) {
    constexpr bool KQ = QT == VKF_DEQUANT_Q4_K || QT == VKF_DEQUANT_Q5_K;
    if (KQ && a.M == 1) return Launcher<QT, CW_DEFAULT, true>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    return Launcher<QT, CW_DEFAULT, false>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
}

static int dispatch(int wtype, Args &a, int sms, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt,
                    size_t cnt_cap) {
    switch (wtype) {
    case VKF_DEQUANT_Q4_0: return launch_q<VKF_DEQUANT_Q4_0>(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q8_0: return launch_q<VKF_DEQUANT_Q8_0>(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q4_K: return launch_q<VKF_DEQUANT_Q4_K>(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q5_K: return launch_q<VKF_DEQUANT_Q5_K>(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    case VKF_DEQUANT_Q6_K: return launch_q<VKF_DEQUANT_Q6_K>(a, sms, stream, ws, ws_cap, cnt, cnt_cap);
    default: return VKF_ERR_UNSUPPORTED;
    }
}

}  // namespace gemv

// Batch columns per launch so the resident activations fit the budget.
int gemv_cols_per_launch(int K) {
    const size_t units = ((size_t)K + 255) / 256;
    const size_t per = (units * 512 + 127) / 128 * 128 + 64 + units * 32;
    return (int)std::max<size_t>(1, std::min<size_t>(8, (gemv::X_BUDGET - 128) / per));
}
size_t gemv_counters(int N) { return (size_t)(N + 15) / 16; }
size_t gemv_ws_floats(int sms) { return (size_t)sms * 2 * 16 * 8; }

static void fill_args(gemv::Args &a, int wtype, const void *W, const void *X, int64_t ldx_bytes, void *Y, int y_f16,
                      int64_t ldy, int M, int N, int K) {
    a.W = (const uint8_t *)W;
    a.X = (const uint8_t *)X;
    a.Y = Y;
    a.M = M;
    a.N = N;
    a.K = K;
    a.ldx_bytes = ldx_bytes;
    a.ldy = ldy;
    a.row_bytes = (int64_t)K / vkf_qtype_block_values(wtype) * vkf_qtype_block_bytes(wtype);
    a.y_f16 = y_f16;
}

// X: fp16, rows 16-byte aligned (ldx_bytes multiple of 16).  Checked by caller.
int gemv_launch(int wtype, const void *W, const void *X, int64_t ldx_bytes, void *Y, int y_f16, int64_t ldy, int M,
                int N, int K, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap, int prefetch) {
    DeviceState *ds = device_state();
    if (!ds) return VKF_ERR_NO_DEVICE;
    gemv::Args a{};
    fill_args(a, wtype, W, X, ldx_bytes, Y, y_f16, ldy, M, N, K);
    a.err = ds->d_error;
    a.prefetch = prefetch;
    return gemv::dispatch(wtype, a, ds->sm_count, stream, ws, ws_cap, cnt, cnt_cap);
}

// Same launch with the SM count and the kernel error word supplied by the
// caller, so that nothing here allocates device memory (the allocation-free
// entry point in noalloc.cu).
int gemv_launch_raw(int wtype, const void *W, const void *X, int64_t ldx_bytes, void *Y, int y_f16, int64_t ldy,
                    int M, int N, int K, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap,
                    int sms, unsigned *err) {
    gemv::Args a{};
    fill_args(a, wtype, W, X, ldx_bytes, Y, y_f16, ldy, M, N, K);
    a.err = err;
    a.prefetch = 0;
    return gemv::dispatch(wtype, a, sms, stream, ws, ws_cap, cnt, cnt_cap);
}

}  // namespace vkf
