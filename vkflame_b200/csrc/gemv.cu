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
#include <type_traits>
#include <cstdlib>

namespace vkf {
namespace gemv {

#ifdef VKF_GEMV_TIMING
// Debug builds only: per-warp cycle counters [cta][warp][phase], and per
// launch the earliest CTA start / latest CTA end / earliest consumer start
// after the dependency wait (global timer, ns).
__device__ unsigned long long g_timing[512][32][8];
__device__ unsigned long long g_timeline[4096][3];
__device__ unsigned long long g_cta_t[4096][512][5];  // per launch, per CTA: start, dep, prologue, loop, reducer
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
static int g_launch_id = 0;
#define VKF_T0() const long long _t0 = clock64()
#define VKF_TACC(ph, t0) atomicAdd(&g_timing[blockIdx.x][threadIdx.x >> 5][ph], (unsigned long long)(clock64() - (t0)))
#else
#define VKF_T0()
#define VKF_TACC(ph, t0)
#endif

constexpr int NST_MAX = 8;            // ring depth cap
constexpr int ROW_BUDGET = 4400;      // max bytes of one row per item
constexpr int SMEM_MAX = 227 * 1024;
constexpr int SMEM_HALF = 112 * 1024;  // two CTAs per SM
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
    int slots;         // parked-partial slots (row blocks in flight)
    int off_sums, off_ring, off_red, off_bar;
    float *ws;         // partials of cut row blocks: [G][2][16 * M]
    int *cnt;          // per-row-block arrival counters (zero between launches)
    unsigned *err;
    int y_f16;
    int prefetch;      // stream weights before the previous kernel on the stream completes
    int whole_tiles;   // S == 1 and W 16-byte aligned: one copy per row block
    // Fused all-gather (column-sharded multi-GPU, nranks > 0, M = 1, fp16):
    // Y goes into every rank's gathered buffer as 8-byte words {two fp16,
    // epoch} (an aligned 8-byte store is single-copy atomic, so a reader that
    // sees the epoch sees the data: no fence, no completion signal).  Each
    // rank keeps two buffers, selected by the step's parity, so a rank that
    // runs ahead never overwrites words a slower rank has yet to read.
    // x_ll: X is such a gathered buffer; its loader waits (bounded) for the
    // current epoch in every word it reads, and needs no dependency wait.
    // epoch: this call site's run count (the words of its run t carry
    // t + 1; a consumer expects its own count + 1, every op running once per
    // step), incremented by the grid's last CTA.  Only this call site's
    // previous run writes it, so it is read before any dependency wait.
    int nranks, rank, x_ll;
    uint8_t *ypeer[8];     // each rank's buffer 0, at this rank's first word
    int64_t ll_stride;     // bytes from a rank's buffer 0 to its buffer 1
    int64_t x_stride;      // same for X when x_ll
    int *epoch, *done;
#ifdef VKF_GEMV_TIMING
    int launch_id;
#endif
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

// Gathered store of one 16-row block (M = 1): lane l < 16 holds row n0 + l
// (valid: inside N); even lanes write the pair (n, n + 1) as one 8-byte word
// {half2, epoch} to every rank.  All 32 lanes call it.
__device__ __forceinline__ void gather_store(const Args &a, int ep, int n0, float v, bool valid) {
    const float vn = __shfl_down_sync(0xffffffffu, v, 1);
    const int lane = threadIdx.x & 31;
    if (!valid || (lane & 1)) return;
    const __half2 h = __floats2half2_rn(v, vn);
    const uint32_t d = *reinterpret_cast<const uint32_t *>(&h);
    const int64_t off = (int64_t)(ep & 1) * a.ll_stride + (int64_t)((n0 + lane) >> 1) * 8;
    for (int q = 0; q < a.nranks; ++q)
        asm volatile("st.relaxed.sys.global.v2.u32 [%0], {%1, %2};" ::"l"(a.ypeer[q] + off), "r"(d), "r"(ep)
                     : "memory");
}

// 32 fp16 X values (64 bytes) of column m, sub-block sb: plain loads, or
// from a gathered buffer (16 words {half2, epoch}), waiting (bounded) until
// every word carries the current epoch.
__device__ __forceinline__ void load_x64(const Args &a, int ep, int m, int sb, uint4 (&v)[4]) {
    if (!a.x_ll) {
        const uint4 *src = reinterpret_cast<const uint4 *>(a.X + (int64_t)m * a.ldx_bytes + sb * 64);
#pragma unroll
        for (int c = 0; c < 4; ++c) v[c] = __ldg(src + c);
        return;
    }
    const uint8_t *src = a.X + (int64_t)(ep & 1) * a.x_stride + (int64_t)m * a.ldx_bytes + sb * 128;
    uint32_t d[16];
    // All 16 loads in flight at once (one memory latency when the words are
    // there); re-read the set until every epoch matches.
    for (uint32_t n = 0;; ++n) {
        uint32_t e[16];
#pragma unroll
        for (int i = 0; i < 16; i += 2)
            asm volatile("ld.relaxed.sys.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                         : "=r"(d[i]), "=r"(e[i]), "=r"(d[i + 1]), "=r"(e[i + 1])
                         : "l"(src + 8 * i)
                         : "memory");
        bool all = true;
#pragma unroll
        for (int i = 0; i < 16; ++i) all = all && e[i] == (uint32_t)ep;
        if (all) break;
        if (n == (1u << 22)) {
            if (a.err) atomicOr(a.err, VKF_KERR_WAIT_TIMEOUT);
            break;
        }
        __nanosleep(20);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) v[c] = make_uint4(d[4 * c], d[4 * c + 1], d[4 * c + 2], d[4 * c + 3]);
}

// Resident activations: one thread per (column, 32-value sub-block) reads the
// 64 source bytes and stores them in fragment order (groups of four permuted
// (x0, x2, x1, x3); owned layout: swizzled granules) with, for the K-quants,
// their fp32 sum split into hi + lo fp16 in the min-term MMA's B layout
// [super-block][t] = (hi 2t, hi 2t+1, lo 2t, lo 2t+1).  The column forms
// (M = 1) store integer activations instead (SUMS 4, 5).
// Integer column forms (StepK1i, StepQ6i): 16-bit fixed point per 32-value
// run, x = s * (256 xh + xl), s = max|x| / 32639 (so xh, xl fit int8), stored
// in value order (xh at +0, xl at +256 of the unit); the run's scale and sum
// (and, Q6_K, its two 16-value group sums) go to the unit's float area.
template <int SUMS>
__device__ __forceinline__ void quantize_run(const Args &a, const uint4 (&v)[4], int m, int sb, uint8_t *xs,
                                             uint8_t *sums) {
        // Integer column forms (StepK1i, StepQ6i): 16-bit fixed point per
        // 32-value run, x = s * (256 xh + xl), s = max|x| / 32639 (so xh,
        // xl fit int8), stored in value order: xh at +0, xl at +256 of the
        // unit; run scale and sum (and, Q6_K, the two 16-value group sums)
        // in the unit's float area.
        float f[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint32_t w[4] = {v[c].x, v[c].y, v[c].z, v[c].w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float2 p = __half22float2(*reinterpret_cast<const __half2 *>(&w[e]));
                f[8 * c + 2 * e] = p.x;
                f[8 * c + 2 * e + 1] = p.y;
            }
        }
        float amax = 0.f, s0 = 0.f, s1 = 0.f;
#pragma unroll
        for (int k = 0; k < 32; ++k) {
            amax = fmaxf(amax, fabsf(f[k]));
            if (k < 16) s0 += f[k];
            else s1 += f[k];
        }
        const float inv = amax > 0.f ? 32639.0f / amax : 0.f;
        uint32_t hw[8], lw[8];
#pragma unroll
        for (int k4 = 0; k4 < 8; ++k4) {
            uint32_t hb = 0, lb = 0;
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const int q = max(-32639, min(32639, __float2int_rn(f[4 * k4 + e] * inv)));
                const int h = (q + 128) >> 8, l = q - (h << 8);
                hb |= (uint32_t)(h & 0xFF) << (8 * e);
                lb |= (uint32_t)(l & 0xFF) << (8 * e);
            }
            hw[k4] = hb;
            lw[k4] = lb;
        }
        uint8_t *run = xs + m * a.xpr + (sb / 8) * 512 + (sb % 8) * 32;
        reinterpret_cast<uint4 *>(run)[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
        reinterpret_cast<uint4 *>(run)[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
        reinterpret_cast<uint4 *>(run + 256)[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
        reinterpret_cast<uint4 *>(run + 256)[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
        const float sc = amax / 32639.0f;
        const int jj = sb % 8;
        if constexpr (SUMS == 4) {
            float *o = reinterpret_cast<float *>(sums + m * a.xsp + (sb / 8) * 64);
            o[m1_sum_slot(jj)] = sc;
            o[8 + m1_sum_slot(jj)] = s0 + s1;
        } else {
            float *o = reinterpret_cast<float *>(sums + m * a.xsp + (sb / 8) * 96);
            o[jj] = sc;
            o[8 + 2 * jj] = s0;
            o[8 + 2 * jj + 1] = s1;
        }
        
}

// SUMS: 0 none; 1 K-quant hi + lo fp16 (min-term MMA); 4 K-quant and 5 Q6_K
// column forms (integer activations, below).
template <bool OWN, int SUMS, int NTC>
__device__ __forceinline__ void load_activations(const Args &a, int ep, uint8_t *xs, uint8_t *sums) {
    const int nsb = a.K / 32, jobs = a.M * nsb;
    // Every CTA reads the same activations at the same moment: start each CTA
    // at a different run so the requests spread over the row's L2 lines.
    const int rot = (int)(((unsigned)blockIdx.x * 97u) % (unsigned)jobs);
    for (int j0 = threadIdx.x; j0 < jobs; j0 += NTC) {
        int j = j0 + rot;
        if (j >= jobs) j -= jobs;
        const int m = j / nsb, sb = j - m * nsb;
        uint4 v[4];
        load_x64(a, ep, m, sb, v);
        if constexpr (SUMS >= 4) {
            quantize_run<SUMS>(a, v, m, sb, xs, sums);
            continue;
        }
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
        if constexpr (SUMS != 0) {
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
            const __half hi = __float2half_rn(sum);
            const __half lo = __float2half_rn(sum - __half2float(hi));
            __half *o = reinterpret_cast<__half *>(sums + m * a.xsp + (sb / 8) * 32 + ((sb % 8) / 2) * 8) + (sb & 1);
            o[0] = hi;
            o[2] = lo;
        }
    }
}

// Slot arithmetic shared by consumers and the reducer: row block number k of
// this CTA (k = 0, 1, ...) uses slot k % slots, phase (k / slots) & 1.
template <int QT, int CW, bool M1, int CPS>
__global__ void __launch_bounds__(32 * (CW + 2), CPS) gemv_kernel(const __grid_constant__ Args a) {
    constexpr int NTC = 32 * CW;
    constexpr int QK = Fmt<QT>::QK, BB = Fmt<QT>::BB;
    constexpr int UB = (256 / QK) * BB;  // bytes of one 256-value unit of a row
    constexpr bool KQ = QT == VKF_DEQUANT_Q4_K || QT == VKF_DEQUANT_Q5_K;
    constexpr bool OWN = Step<QT>::OWNED;
    constexpr bool Q6 = QT == VKF_DEQUANT_Q6_K;
    constexpr bool COLS = M1 && (KQ || Q6);  // column-form decode (StepK1i, StepQ6i)
    constexpr int SUMS = COLS ? (KQ ? 4 : 5) : (KQ ? 1 : 0);
    constexpr int PW = COLS ? 2 : 4;         // parked floats per lane
    constexpr int PRODUCER = CW, REDUCER = CW + 1;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *xs = smem;
    uint8_t *sums = smem + a.off_sums;
    uint8_t *ring = smem + a.off_ring;
    float *park = reinterpret_cast<float *>(smem + a.off_red);  // [slot][warp][lane][PW]
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + a.off_bar);
    uint64_t *empty = full + NST_MAX;
    uint64_t *parked = empty + NST_MAX;   // per slot: CW consumer arrivals
    uint64_t *freed = parked + MAX_SLOTS; // per slot: reducer done

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x;
    const int it0 = first_item(cta, a), it1 = first_item(cta + 1, a);
    // Programmatic dependent launch: the next kernel on the stream may start
    // its prologue now; everything this kernel reads or writes that another
    // kernel may touch (X, Y, the scratch) waits for the previous kernel.
    asm volatile("griddepcontrol.launch_dependents;");
#ifdef VKF_GEMV_TIMING
    unsigned long long gt0;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(gt0));
    if (threadIdx.x == 0 && a.launch_id < 4096) {
        atomicMin(&g_timeline[a.launch_id][0], gt0);
        g_cta_t[a.launch_id][blockIdx.x][0] = gt0;
    }
#endif
    if (threadIdx.x == 0) {
        for (int s = 0; s < a.nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        for (int s = 0; s < a.slots; ++s) {
            mbar_init(&parked[s], CW);
            mbar_init(&freed[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == PRODUCER) {
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
            if (a.whole_tiles) {
                // Whole rows: the row block is one contiguous, 16-byte aligned
                // range of the matrix and lands as one copy (one TMA operation
                // per row block instead of one per row: the per-row form is
                // held to ~4.8 TB/s by the operation rate at 1.4 KB rows).
                if (lane == 0) {
                    const int rows = min(16, a.N - tile * 16);
                    const uint32_t sz = (uint32_t)(((int64_t)rows * a.row_bytes + 15) & ~(int64_t)15);
                    mbar_arrive_expect_tx(&full[s], sz);
                    bulk_g2s(ring + s * a.stage_bytes, a.W + (int64_t)tile * 16 * a.row_bytes, sz, &full[s]);
                }
            } else {
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
            }
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

    const int rows16m = 16 * a.M;
    if (warp == REDUCER) {
        // ---------------- reducer ----------------
        // Walks the CTA's row blocks in order: waits until all consumer warps
        // have parked their partials, sums them in warp order (deterministic),
        // stores Y, and frees the slot.  A row block cut between CTAs is
        // published to scratch; its last contributor sums all partials in CTA
        // order.  None of this is on the consumers' path.
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const int ep = a.nranks ? *a.epoch + 1 : 0;
        const int first_tile = it0 / a.S, last_tile = (it1 - 1) / a.S;
        bool ok = true;
        for (int tb = first_tile, k = 0; tb <= last_tile && it1 > it0; ++tb, ++k) {
            const int sl = k % a.slots;
            if (ok) ok = mbar_wait(&parked[sl], (uint32_t)(k / a.slots) & 1u, a.err);
            const float *q = park + (size_t)sl * CW * 32 * PW;
            float o[4];
            if constexpr (COLS) {
                // lane = (row r = lane & 15, warp half h = lane >> 4): rows g < 8
                // are .x of lanes g*4 + t, rows g + 8 are .y.
                const int r = lane & 15, h = lane >> 4, g = r & 7, comp = r >> 3;
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < CW / 2; ++w)
#pragma unroll
                    for (int t = 0; t < 4; ++t) v += q[((h * (CW / 2) + w) * 32 + g * 4 + t) * 2 + comp];
                v += __shfl_xor_sync(0xffffffffu, v, 16);
                o[0] = v;
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int rc = lane + 32 * j;
                    o[j] = 0.f;
                    if (rc < rows16m) {
                        const int r = rc / a.M, c = rc - r * a.M;
                        const int g = r & 7, comp = (r >> 3) * 2 + (c & 1), l = g * 4 + (c >> 1);
#pragma unroll 4
                        for (int w = 0; w < CW; ++w) o[j] += q[(w * 32 + l) * 4 + comp];
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&freed[sl]);
            const bool whole = tb * a.S >= it0 && (tb + 1) * a.S <= it1;
            if (whole) {
                if (a.nranks) {  // M = 1: lane l < 16 holds row tb * 16 + l in o[0]
                    gather_store(a, ep, tb * 16, o[0], lane < 16 && tb * 16 + lane < a.N);
                } else if constexpr (COLS) {
                    if (lane < 16 && tb * 16 + lane < a.N) store_y(a, 0, tb * 16 + lane, o[0]);
                } else {
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int rc = lane + 32 * j, r = rc / a.M, c = rc - r * a.M;
                        if (rc < rows16m && tb * 16 + r < a.N) store_y(a, c, tb * 16 + r, o[j]);
                    }
                }
                continue;
            }
            // A row block cut between CTAs: publish this CTA's partial; the last
            // contributor to arrive sums all partials in CTA order and stores Y.
            const int which = tb == first_tile ? 0 : 1;
            float *wsp = a.ws + ((int64_t)cta * 2 + which) * rows16m;
            if constexpr (COLS) {
                if (lane < 16) wsp[lane] = o[0];
            } else {
#pragma unroll
                for (int j = 0; j < 4; ++j)
                    if (lane + 32 * j < rows16m) wsp[lane + 32 * j] = o[j];
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
            if (a.nranks) {
                float v = 0.f;
                if (lane < 16)
                    for (int c = c_first; c <= c_last; ++c) {
                        const int wc = tb == first_item(c, a) / a.S ? 0 : 1;
                        v += __ldcg(a.ws + ((int64_t)c * 2 + wc) * rows16m + lane);
                    }
                gather_store(a, ep, tb * 16, v, lane < 16 && tb * 16 + lane < a.N);
                if (lane == 0) a.cnt[tb] = 0;
                continue;
            }
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
        if (a.nranks) {
            // The grid's last CTA advances this call site's run count (every
            // CTA read it at its start, before arriving here).
            __syncwarp();
            if (lane == 0 && atomicAdd(a.done, 1) == a.G - 1) {
                *a.done = 0;
                atomicAdd(a.epoch, 1);
            }
        }
#ifdef VKF_GEMV_TIMING
        if (lane == 0 && a.launch_id < 4096) {
            unsigned long long ge;
            asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(ge));
            atomicMax(&g_timeline[a.launch_id][1], ge);
            g_cta_t[a.launch_id][blockIdx.x][4] = ge;
        }
#endif
        return;
    }

    // ---------------- consumers ----------------
#ifdef VKF_GEMV_TIMING
    const long long tp0 = clock64();
#endif
    // Pull the activation rows into L2 while the previous kernel finishes.  A
    // prefetch consumes no data (the loads below come after the dependency
    // wait, and L2 is the point of coherence), so it is safe even when the
    // previous kernel writes X; it only hides the DRAM latency of an X that
    // has left L2.
    for (int i = threadIdx.x; i < a.M * (int)((a.K * 2 + 127) / 128); i += NTC) {
        const int m = i / ((a.K * 2 + 127) / 128), l = i - m * ((a.K * 2 + 127) / 128);
        asm volatile("prefetch.global.L2 [%0];" ::"l"(a.X + (int64_t)m * a.ldx_bytes + l * 128));
    }
    // A gathered X is validated word by word (its epochs), so its loader
    // starts without waiting for the previous kernel on the stream.
    if (!(a.nranks && a.x_ll)) asm volatile("griddepcontrol.wait;" ::: "memory");
#ifdef VKF_GEMV_TIMING
    if (lane == 0) VKF_TACC(6, tp0);
    const long long tx0 = clock64();
#endif
#ifdef VKF_GEMV_TIMING
    if (threadIdx.x == 0 && a.launch_id < 4096) {
        unsigned long long gw;
        asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(gw));
        atomicMin(&g_timeline[a.launch_id][2], gw);
        g_cta_t[a.launch_id][blockIdx.x][1] = gw;
    }
#endif
    const int ep = a.nranks ? *a.epoch + 1 : 0;
    load_activations<OWN, SUMS, NTC>(a, ep, xs, sums);
    consumer_bar<CW>();
#ifdef VKF_GEMV_TIMING
    if (threadIdx.x == 0 && a.launch_id < 4096) g_cta_t[a.launch_id][blockIdx.x][2] = gtimer();
#endif
#ifdef VKF_GEMV_TIMING
    if (lane == 0) VKF_TACC(2, tx0);
    const long long tl0 = clock64();
    struct TEnd {
        long long t;
        int lane;
        __device__ ~TEnd() { if (lane == 0) VKF_TACC(3, t); }
    } tend{tl0, lane};
#endif

    const int g = lane >> 2, t = lane & 3;
    // Lanes of columns >= M read a real column (their outputs are dropped),
    // which keeps every fragment load a broadcast or conflict-free.
    const int xcol = g % a.M;
    const uint8_t *xg = xs + xcol * a.xpr;
    const uint8_t *sg = sums + xcol * a.xsp;
    // After a bounded wait gives up (error bit already set) the warp keeps
    // walking the same items without waiting or computing, so every warp
    // still makes the same barrier arrivals.
    bool ok = true;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int tile = it0 / a.S, step = it0 - tile * a.S, s = 0;
    uint32_t ph = 0;
    int ubase = 0;  // units of this CTA's earlier items, mod CW
    int k = 0;      // row blocks finished by this CTA
    int park_slot = 0;
    uint32_t park_phase = 0;  // phase of the slot's current use
    const int64_t row_off_a = (int64_t)g * a.row_bytes, row_off_b = (int64_t)(g + 8) * a.row_bytes;
    for (int it = it0; it < it1; ++it) {
#ifdef VKF_GEMV_TIMING
        const long long tw0 = clock64();
#endif
        if (ok) ok = mbar_wait(&full[s], ph, a.err);
#ifdef VKF_GEMV_TIMING
        if (lane == 0) VKF_TACC(0, tw0);
        const long long td0 = clock64();
#endif
        const int u0 = step * a.upi, nu = min(a.upi, a.units - u0);
        if (ok) {
            const uint8_t *st = ring + s * a.stage_bytes;
            const uint8_t *ra, *rb;
            if (a.whole_tiles) {  // contiguous image of the row block
                ra = st + row_off_a;
                rb = st + row_off_b;
            } else {
                const int64_t row_a = (int64_t)tile * 16 + g;
                const uintptr_t ga = (uintptr_t)a.W + row_a * a.row_bytes + (int64_t)u0 * UB;
                const uintptr_t gb = ga + 8 * a.row_bytes;
                ra = st + g * a.rpb + (ga & 15);
                rb = st + (g + 8) * a.rpb + (gb & 15);
            }
            int u = warp - ubase;
            if (u < 0) u += CW;
            auto unit_step = [&](int uu) {
                const int unit = u0 + uu;
                if constexpr (COLS && KQ) {
                    StepK1i<QT == VKF_DEQUANT_Q5_K>::run(ra + uu * UB, rb + uu * UB, xs + unit * 512, g == t, g == t + 4,
                                                         reinterpret_cast<const float *>(sums + unit * 64), t, acc);
                } else {
                    const int nblk = QK == 32 ? min(8, (a.K - unit * 256) / 32) : 8;
                    Step<QT>::run(ra + uu * UB, rb + uu * UB, xg + unit * 512, sg + unit * 32, t, nblk, acc);
                }
            };
            if constexpr (COLS && Q6) {
                // Q6_K super-blocks are 210 bytes: a unit's words are 4-byte
                // aligned or 2 mod 4 by its parity, uniformly across the warp
                // when rows are a multiple of 4 bytes (K a multiple of 512).
                // Rows a multiple of 4 bytes: every lane's unit has the same alignment
                // (the form must be chosen warp-uniformly around mma.sync); else
                // the shifted form, which serves either alignment.
                const bool rows4 = (a.row_bytes & 3) == 0;
                for (; u < nu; u += CW) {
                    const int unit = u0 + u;
                    const uint8_t *pa = ra + u * UB, *pb = rb + u * UB;
                    const float *sx = reinterpret_cast<const float *>(sums + unit * 96);
                    if (!rows4) StepQ6i::run<2>(pa, pb, xs + unit * 512, g, sx, t, acc);
                        else if ((((uintptr_t)pa | (uintptr_t)pb) & 3) == 0) StepQ6i::run<0>(pa, pb, xs + unit * 512, g, sx, t, acc);
                        else StepQ6i::run<1>(pa, pb, xs + unit * 512, g, sx, t, acc);
                }
            } else {
                for (; u < nu; u += CW) unit_step(u);
            }
        }
#ifdef VKF_GEMV_TIMING
        __syncwarp();
        if (lane == 0) VKF_TACC(1, td0);
#endif
#ifdef VKF_GEMV_TIMING
        const long long ta0 = clock64();
#endif
        ubase += nu;
        while (ubase >= CW) ubase -= CW;
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
#ifdef VKF_GEMV_TIMING
        if (lane == 0) VKF_TACC(5, ta0);
#endif
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

        // Park this warp's partial of the finished row block (one vector store
        // per lane) and signal the reducer; a slot is reused only after the
        // reducer has freed it (slots row blocks earlier).
        const int sl = park_slot;
#ifdef VKF_GEMV_TIMING
        const long long tf0 = clock64();
#endif
        if (k >= a.slots && ok) ok = mbar_wait(&freed[sl], park_phase ^ 1u, a.err);
#ifdef VKF_GEMV_TIMING
        if (lane == 0) VKF_TACC(4, tf0);
#endif
        float *p = park + ((size_t)(sl * CW + warp) * 32 + lane) * PW;
        if constexpr (COLS) {
            *reinterpret_cast<float2 *>(p) = make_float2(acc[0] + acc[1], acc[2] + acc[3]);
        } else {
            *reinterpret_cast<float4 *>(p) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        }
        acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
        __syncwarp();
        if (lane == 0) mbar_arrive(&parked[sl]);
        ++k;
        if (++park_slot == a.slots) {
            park_slot = 0;
            park_phase ^= 1u;
        }
    }
#ifdef VKF_GEMV_TIMING
    if (lane == 0 && a.launch_id < 4096) atomicMax(&g_cta_t[a.launch_id][blockIdx.x][3], gtimer());
#endif
}

// Worst shared-memory bank multiplicity of the decode's weight loads when rows
// sit at `pitch` bytes: 16-byte loads of lanes (g, t) at g * pitch + 32 t in
// 8-lane phases (owned mapping), or 4-byte loads at g * pitch + 4 t across
// the warp (plain mapping).  A contiguous row block (one copy) is used only
// where this stays <= 2.
static int pitch_conflicts(int64_t pitch, bool owned) {
    int worst = 0;
    if (owned) {
        if (pitch % 16) return 32;
        for (int ph = 0; ph < 4; ++ph) {
            int hits[8] = {};
            for (int gg = 2 * ph; gg < 2 * ph + 2; ++gg)
                for (int t = 0; t < 4; ++t) worst = std::max(worst, ++hits[(gg * (pitch / 16) + 2 * t) % 8]);
        }
    } else {
        if (pitch % 4) return 32;
        int hits[32] = {};
        for (int gg = 0; gg < 8; ++gg)
            for (int t = 0; t < 4; ++t) worst = std::max(worst, ++hits[(gg * (pitch / 4) + t) % 32]);
    }
    return worst;
}

template <int QT, int CW, bool M1, int CPS>
struct Launcher {
    static constexpr int QK = Fmt<QT>::QK, BB = Fmt<QT>::BB;
    static constexpr int UB = (256 / QK) * BB;
    static constexpr bool KQ = QT == VKF_DEQUANT_Q4_K || QT == VKF_DEQUANT_Q5_K;
    static constexpr bool OWN = Step<QT>::OWNED;
    static constexpr int NT = 32 * (CW + 2);

    // require_whole: plan only (return VKF_ERR_UNSUPPORTED without launching)
    // unless every item is a whole row block with at least two ring stages.
    // plan_only: every check of a launch, and no launch (VKF_OK if it would launch).
    static int launch(Args &a, int sms, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap,
                      bool require_whole = false, bool plan_only = false) {
        auto up = [](int64_t v, int64_t m) { return (v + m - 1) / m * m; };
        a.units = (a.K + 255) / 256;
        // Column pitches: the owned layout's 16-byte fragment loads want
        // columns 64 bytes apart mod 128 banks-wise, the plain layout's
        // 8-byte loads 32 bytes.
        a.xpr = (int)up((int64_t)a.units * 512, 128) + (OWN ? 64 : 32);
        constexpr bool Q6 = QT == VKF_DEQUANT_Q6_K;
        a.xsp = (M1 && Q6) ? a.units * 96 : (M1 && KQ) ? a.units * 64 : KQ ? (int)up((int64_t)a.units * 32, 16) : 0;
        a.off_sums = a.M * a.xpr;
        const int x_end = (int)up(a.off_sums + (int64_t)a.M * a.xsp, 128);
        if (x_end > X_BUDGET) return VKF_ERR_UNSUPPORTED;
        const int rows16m = 16 * a.M;
        constexpr bool COLS = M1 && (KQ || QT == VKF_DEQUANT_Q6_K);
        const int slot_bytes = CW * 32 * (COLS ? 2 : 4) * 4;
        const int bar_bytes = 2 * NST_MAX * 8 + 2 * MAX_SLOTS * 8;
        const int smem_cap = CPS == 2 ? SMEM_HALF : SMEM_MAX;
        const int avail = smem_cap - x_end - bar_bytes - 128;
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
            a.whole_tiles = a.S == 1 && ((uintptr_t)a.W & 15) == 0 && pitch_conflicts(a.row_bytes, OWN) <= 2;
            if (a.whole_tiles) a.stage_bytes = (int)up(16 * a.row_bytes, 128);
            a.nst = std::min(NST_MAX, (avail - 2 * slot_bytes) / (a.stage_bytes + slot_bytes));
            if (a.nst >= 2 || a.upi == 1) break;
            a.upi = std::max(1, a.upi / 2);
            a.S = (a.units + a.upi - 1) / a.upi;
            a.upi = (a.units + a.S - 1) / a.S;
        }
        if (a.nst < 2) return VKF_ERR_UNSUPPORTED;
        if (require_whole && !a.whole_tiles) return VKF_ERR_UNSUPPORTED;
        if ((int64_t)a.T * a.S > (int64_t)1 << 30) return VKF_ERR_UNSUPPORTED;
        a.I = a.T * a.S;
        a.slots = a.nst + 2;
        const int red_bytes = (int)up((int64_t)a.slots * slot_bytes, 128);
        a.off_ring = x_end;
        a.off_red = a.off_ring + a.nst * a.stage_bytes;
        a.off_bar = a.off_red + red_bytes;
        const size_t smem = (size_t)a.off_bar + bar_bytes;
        const int grid = std::max(1, std::min(CPS * sms, a.I));
        if ((size_t)grid * 2 * rows16m > ws_cap || (size_t)a.T > cnt_cap) return VKF_ERR_INVALID;
        if (plan_only) return VKF_OK;
        static bool attr_set[64] = {false};
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev < 64 && !attr_set[dev]) {
            cudaFuncSetAttribute(gemv_kernel<QT, CW, M1, CPS>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_cap);
            attr_set[dev] = true;
        }
        a.G = grid;
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
#ifdef VKF_GEMV_TIMING
        a.launch_id = g_launch_id++;
#endif
        cudaLaunchKernelEx(&cfg, gemv_kernel<QT, CW, M1, CPS>, a);
        return check_launch();
    }
};

// 8 consumer warps: with 16, each warp decodes fewer units per item and the
// per-item overhead grows faster than the latency hiding gains (measured).
// 8 consumer warps: with 16, each warp decodes fewer units per item and the
// per-item overhead grows faster than the latency hiding gains (measured).
constexpr int CW_DEFAULT = 8;

// M = 1 K-quant and Q6_K launches use the column form.  Two CTAs per SM
// (half the shared memory each) where whole row blocks still fit two ring
// stages: a CTA of the next kernel on the stream can then start, and stream
// its weights, as soon as either CTA of this one finishes (measured ~12 %
// faster on the 14B stack's Q4_K shapes); otherwise one CTA per SM.
template <int QT>
static int launch_q(Args &a, int sms, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap,
                    bool plan_only) {
    constexpr bool COLS_FMT = QT == VKF_DEQUANT_Q4_K || QT == VKF_DEQUANT_Q5_K || QT == VKF_DEQUANT_Q6_K;
    if (COLS_FMT && a.M == 1) {
        Args b = a;
        const int rc =
            Launcher<QT, CW_DEFAULT, true, 2>::launch(b, sms, stream, ws, ws_cap, cnt, cnt_cap, true, plan_only);
        if (rc != VKF_ERR_UNSUPPORTED) return rc;
        return Launcher<QT, CW_DEFAULT, true, 1>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap, false, plan_only);
    }
    return Launcher<QT, CW_DEFAULT, false, 1>::launch(a, sms, stream, ws, ws_cap, cnt, cnt_cap, false, plan_only);
}

static int dispatch(int wtype, Args &a, int sms, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt,
                    size_t cnt_cap, bool plan_only = false) {
    switch (wtype) {
    case VKF_DEQUANT_Q4_0: return launch_q<VKF_DEQUANT_Q4_0>(a, sms, stream, ws, ws_cap, cnt, cnt_cap, plan_only);
    case VKF_DEQUANT_Q8_0: return launch_q<VKF_DEQUANT_Q8_0>(a, sms, stream, ws, ws_cap, cnt, cnt_cap, plan_only);
    case VKF_DEQUANT_Q4_K: return launch_q<VKF_DEQUANT_Q4_K>(a, sms, stream, ws, ws_cap, cnt, cnt_cap, plan_only);
    case VKF_DEQUANT_Q5_K: return launch_q<VKF_DEQUANT_Q5_K>(a, sms, stream, ws, ws_cap, cnt, cnt_cap, plan_only);
    case VKF_DEQUANT_Q6_K: return launch_q<VKF_DEQUANT_Q6_K>(a, sms, stream, ws, ws_cap, cnt, cnt_cap, plan_only);
    default: return VKF_ERR_UNSUPPORTED;
    }
}

}  // namespace gemv

#ifdef VKF_GEMV_TIMING
extern "C" int vkf_gemv_cta_times(void *host, int launch) {
    return (int)cudaMemcpyFromSymbol(host, gemv::g_cta_t, sizeof(unsigned long long) * 512 * 5,
                                     sizeof(unsigned long long) * 512 * 5 * (size_t)launch);
}
extern "C" int vkf_gemv_timeline(void *host, int reset) {
    if (reset) {
        static unsigned long long init[4096][3];
        for (auto &r : init) { r[0] = ~0ull; r[1] = 0; r[2] = ~0ull; }
        gemv::g_launch_id = 0;
        return (int)cudaMemcpyToSymbol(gemv::g_timeline, init, sizeof(init));
    }
    return (int)cudaMemcpyFromSymbol(host, gemv::g_timeline, sizeof(gemv::g_timeline));
}
extern "C" int vkf_gemv_timing(void *host, int reset) {
    if (reset) {
        static unsigned long long z[512 * 32 * 8];
        return (int)cudaMemcpyToSymbol(gemv::g_timing, z, sizeof(z));
    }
    return (int)cudaMemcpyFromSymbol(host, gemv::g_timing, sizeof(gemv::g_timing));
}
#endif

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
                int N, int K, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap, int prefetch,
                const vkf_gather_t *g) {
    DeviceState *ds = device_state();
    if (!ds) return VKF_ERR_NO_DEVICE;
    gemv::Args a{};
    fill_args(a, wtype, W, X, ldx_bytes, Y, y_f16, ldy, M, N, K);
    a.err = ds->d_error;
    a.prefetch = prefetch;
    if (g) {
        a.nranks = g->world;
        a.rank = g->rank;
        for (int q = 0; q < g->world; ++q) a.ypeer[q] = (uint8_t *)g->y_rank[q];
        a.ll_stride = g->stride;
        a.x_ll = g->x_gathered;
        a.x_stride = g->x_stride;
        a.epoch = g->epoch;
        a.done = g->done;
    }
    return gemv::dispatch(wtype, a, ds->sm_count, stream, ws, ws_cap, cnt, cnt_cap);
}

// Same launch with the SM count and the kernel error word supplied by the
// caller, so that nothing here allocates device memory (the allocation-free
// entry point in noalloc.cu).  plan_only: run every check, launch nothing.
int gemv_launch_raw(int wtype, const void *W, const void *X, int64_t ldx_bytes, void *Y, int y_f16, int64_t ldy,
                    int M, int N, int K, cudaStream_t stream, float *ws, size_t ws_cap, int *cnt, size_t cnt_cap,
                    int sms, unsigned *err, int plan_only) {
    gemv::Args a{};
    fill_args(a, wtype, W, X, ldx_bytes, Y, y_f16, ldy, M, N, K);
    a.err = err;
    a.prefetch = 0;
    return gemv::dispatch(wtype, a, sms, stream, ws, ws_cap, cnt, cnt_cap, plan_only != 0);
}

}  // namespace vkf
