// chain.cu — the decode linears of one token as ONE persistent kernel (M = 1).
//
// A decoder's linears run as a chain: each reads an earlier linear's output.
// Launched one kernel per linear, every link pays a kernel boundary (the
// next kernel's CTAs become resident only as the previous kernel's leave,
// and its weight stream starts late), and with column sharding over several
// GPUs every link also waits for the slowest rank.  Here one cooperative
// launch (one CTA per SM, all resident) walks the whole list:
//
//   producer warp  streams the packed weight items of every linear this CTA
//                  owns, in order, into a byte ring in shared memory (bulk
//                  copies, mbarrier transaction counts).  Weights depend on
//                  nothing, so it runs ahead across linear boundaries while
//                  the consumers wait for their activations: the weight
//                  stream never stops for the chain.
//   8 consumer     per linear: load the activation row (from the gathered
//   warps          buffer of the linear that produced it, waiting word by
//                  word for this run's epoch; or a plain fp16 row), quantise
//                  it into shared memory, then decode the ring's items with
//                  the M = 1 integer column forms of gemv_q.cuh (StepK1i,
//                  StepQ6i) and park each finished row block's partials.
//   reducer warp   sums parked partials in warp order, stores the outputs:
//                  as {fp16 pair, epoch} words into every rank's gathered
//                  buffer (NVLink peer stores; world size 1: the local one),
//                  or as a plain fp16 row.  Row blocks cut between CTAs are
//                  finished by their last contributor (per-linear scratch
//                  and counters, so no slot is ever reused within a run).
//
// The gathered-buffer word protocol is the one of vkflame_quant_linear_gather
// (include/vkflame_rt.h): an aligned 8-byte store is single-copy atomic, so
// a reader that sees its epoch in a word sees the values; two buffers by the
// run's parity; the run count (epoch) is advanced by the grid's last CTA.
// Every wait is bounded in time (error bit and the place it gave up, then the
// kernel walks on without waiting).
//
// Replaces, for a whole decode step, the per-call chain of the reference's
// quantised mul_mat (shim/hip_runtime_shim.cpp:1102-1172): one launch per
// token instead of three dispatches and two temporary buffers per linear.

#include "gemv_q.cuh"

#include <algorithm>
#include <cstdlib>
#include <vector>

namespace vkf {
namespace chain {

using gemv::StepK1i;
using gemv::StepQ6i;
using gemv::m1_sum_slot;

constexpr int CW = 8;                  // consumer warps
constexpr int NT = 32 * (CW + 2);      // + producer + reducer
constexpr int NSLOT = 8;               // ring items in flight
constexpr int PSLOTS = 6;              // parked row blocks in flight
constexpr int SMEM = 227 * 1024;
constexpr int ROW_BUDGET = 4400;       // max bytes of one row per item (default)
constexpr int PARK_BYTES = CW * 32 * 2 * 4;

struct Lin {
    const uint8_t *W;
    int qt, K, N;
    int units, ub;         // 256-value units per row, bytes per unit
    int64_t row_bytes;
    int S, upi, T, I;      // items per row block, units per item, row blocks, items
    int whole;             // one copy per row block (S == 1, 16-byte aligned rows)
    int rpb;               // split items: smem pitch of one row
    int item_bytes;        // smem bytes of one item (128-byte multiple)
    const uint8_t *X;      // plain fp16 row, or this rank's gathered buffer 0 of the source linear
    int x_ll;              // X is gathered words
    int64_t x_stride;      // gathered X: bytes from buffer 0 to buffer 1
    uint8_t *ypeer[VKF_MAX_RANKS];  // gathered output: every rank's buffer 0 at this rank's first word
    int64_t y_stride;
    __half *y_plain;       // plain fp16 output instead (nullptr: gathered)
    float *ws;             // [G][2][16] partials of cut row blocks
    int *cnt;              // [T] arrival counters (zero between runs)
};

struct Geo {
    const uint8_t *W;
    int64_t row_bytes;
    int qt, units, ub, S, upi, I, N, whole, rpb, item_bytes;
};
__device__ __forceinline__ Geo geo(const Lin &L) {
    return Geo{L.W, L.row_bytes, L.qt, L.units, L.ub, L.S, L.upi, L.I, L.N, L.whole, L.rpb, L.item_bytes};
}

struct Params {
    const Lin *lin;
    int n;
    int nranks;
    int G;
    int ring_bytes;
    int off_sums, off_park, off_ring, off_bar;
    int *epoch, *done;
    unsigned *err;
    unsigned long long *trace;  // optional [n][2]: latest X-ready, latest row-block store over CTAs (globaltimer ns)
    int *fail;                  // [4]: first wait that gave up: role (1 producer, 2 reducer, 3 consumer
                                // ring, 4 consumer park slot, 5 activations), linear, item, CTA
};

__device__ __forceinline__ int first_item(int c, int I, int G) { return (int)((int64_t)c * I / G); }
__device__ __forceinline__ int cta_of_item(int i, int I, int G) { return (int)(((int64_t)(i + 1) * G - 1) / I); }
__device__ __forceinline__ void consumer_bar() { asm volatile("bar.sync 1, %0;" ::"n"(CW * 32) : "memory"); }
__device__ __forceinline__ unsigned long long gtimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Every wait gives up after WAIT_NS of globaltimer time (or at once, after a
// short grace, when another wait on this device already gave up), sets the
// kernel error bit and records the first failure's place; the kernel then
// walks on without waiting, so it always ends.
constexpr unsigned long long WAIT_NS = 2000000000ull;

__device__ __forceinline__ bool gave_up(unsigned *err) {
    return (*(volatile unsigned *)err & VKF_KERR_WAIT_TIMEOUT) != 0;
}

__device__ __noinline__ void record_fail(const Params &p, int role, int li, int it) {
    atomicOr(p.err, VKF_KERR_WAIT_TIMEOUT);
    if (atomicCAS(&p.fail[0], 0, role) == 0) {
        p.fail[1] = li;
        p.fail[2] = it;
        p.fail[3] = blockIdx.x;
    }
}

__device__ __forceinline__ bool wait_bar(uint64_t *bar, uint32_t parity, const Params &p, int role, int li, int it) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = gtimer();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63) == 0) {
            const unsigned long long dt = gtimer() - t0;
            if (dt > WAIT_NS || (dt > 1000000ull && gave_up(p.err))) {
                record_fail(p, role, li, it);
                return false;
            }
        }
    }
}

// Byte ring placement: deterministic in the item sequence, so the producer
// and every consumer warp compute the same offsets independently.
__device__ __forceinline__ int ring_place(int &head, int bytes, int ring) {
    const int off = head + bytes > ring ? 0 : head;
    head = off + bytes;
    return off;
}

// 32 fp16 activations (run sb) of a plain row or of a gathered buffer (16
// words {half2, epoch}; re-read until every word carries ep, bounded).
__device__ __forceinline__ void load_run(const Lin &L, int ep, int sb, uint4 (&v)[4], const Params &p, int li) {
    if (!L.x_ll) {
        const uint4 *src = reinterpret_cast<const uint4 *>(L.X + sb * 64);
#pragma unroll
        for (int c = 0; c < 4; ++c) v[c] = __ldg(src + c);
        return;
    }
    const uint8_t *src = L.X + (int64_t)(ep & 1) * L.x_stride + sb * 128;
    uint32_t d[16];
    unsigned long long t0 = 0;
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
        if (n == 0) t0 = gtimer();
        else if ((n & 15) == 0) {
            const unsigned long long dt = gtimer() - t0;
            if (dt > WAIT_NS || (dt > 1000000ull && gave_up(p.err))) {
                record_fail(p, 5, li, sb);
                break;
            }
        }
        __nanosleep(32);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) v[c] = make_uint4(d[4 * c], d[4 * c + 1], d[4 * c + 2], d[4 * c + 3]);
}

// One 32-value run as 16-bit fixed point x = s (256 xh + xl), s = max|x| /
// 32639 (xh, xl int8; value order, xh at +0, xl at +256 of the unit), with
// the run's scale and sums in the unit's float area: K-quants [s | X] in the
// m1_sum_slot order, Q6_K [s (8) | X16 (16)].  The layout StepK1i / StepQ6i read.
__device__ __forceinline__ void quantize_run(const uint4 (&v)[4], int sb, bool q6, uint8_t *xs, uint8_t *sums) {
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
    uint8_t *run = xs + (sb / 8) * 512 + (sb % 8) * 32;
    reinterpret_cast<uint4 *>(run)[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    reinterpret_cast<uint4 *>(run)[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
    reinterpret_cast<uint4 *>(run + 256)[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    reinterpret_cast<uint4 *>(run + 256)[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
    const float sc = amax / 32639.0f;
    const int jj = sb % 8;
    if (!q6) {
        float *o = reinterpret_cast<float *>(sums + (sb / 8) * 64);
        o[m1_sum_slot(jj)] = sc;
        o[8 + m1_sum_slot(jj)] = s0 + s1;
    } else {
        float *o = reinterpret_cast<float *>(sums + (sb / 8) * 96);
        o[jj] = sc;
        o[8 + 2 * jj] = s0;
        o[8 + 2 * jj + 1] = s1;
    }
}

// Output of one 16-row block (lane l < 16 holds row n0 + l): gathered words
// {fp16 Y[n], fp16 Y[n + 1], epoch} to every rank (even lanes), or plain fp16.
__device__ __forceinline__ void store_block(const Lin &L, int nranks, int ep, int n0, float v, bool valid) {
    const float vn = __shfl_down_sync(0xffffffffu, v, 1);
    const int lane = threadIdx.x & 31;
    if (!valid) return;
    if (L.y_plain) {
        L.y_plain[n0 + lane] = __float2half_rn(v);
        return;
    }
    if (lane & 1) return;
    const __half2 h = __floats2half2_rn(v, vn);
    const uint32_t d = *reinterpret_cast<const uint32_t *>(&h);
    const int64_t off = (int64_t)(ep & 1) * L.y_stride + (int64_t)((n0 + lane) >> 1) * 8;
    for (int q = 0; q < nranks; ++q)
        asm volatile("st.relaxed.sys.global.v2.u32 [%0], {%1, %2};" ::"l"(L.ypeer[q] + off), "r"(d), "r"(ep)
                     : "memory");
}

__global__ void __launch_bounds__(NT, 1) chain_kernel(const __grid_constant__ Params p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *xs = smem;
    uint8_t *sums = smem + p.off_sums;
    float *park = reinterpret_cast<float *>(smem + p.off_park);  // [slot][warp][lane][2]
    uint8_t *ring = smem + p.off_ring;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + p.off_bar);
    uint64_t *empty = full + NSLOT;
    uint64_t *parked = empty + NSLOT;
    uint64_t *freed = parked + PSLOTS;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x, G = p.G;
    // Every thread reads this run's count before any CTA can finish.
    const int ep = *p.epoch + 1;
    if (threadIdx.x == 0) {
        for (int s = 0; s < NSLOT; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], CW);
        }
        for (int s = 0; s < PSLOTS; ++s) {
            mbar_init(&parked[s], CW);
            mbar_init(&freed[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == CW) {
        // ---------------- producer ----------------
        // Lane 0 places items; for split items lanes 0..15 copy one row each.
        int head = 0, n = 0, oldest = 0;
        int q_off[NSLOT], q_len[NSLOT];
        bool ok = true;
        for (int li = 0; li < p.n && ok; ++li) {
            const Lin &L = p.lin[li];
            // The hot fields in registers (every asm "memory" clobber would
            // otherwise force a reload from global memory).
            const Geo H = geo(L);
            const int i0 = first_item(cta, H.I, G), i1 = first_item(cta + 1, H.I, G);
            for (int it = i0; it < i1; ++it, ++n) {
                const int bytes = H.item_bytes;
                const int off = ring_place(head, bytes, p.ring_bytes);
                // Wait until the oldest items in flight no longer overlap
                // [off, off + bytes) and a slot is free.
                for (;;) {
                    bool clash = n - oldest >= NSLOT;
                    for (int j = oldest; j < n && !clash; ++j) {
                        const int s = j % NSLOT;
                        clash = off < q_off[s] + q_len[s] && q_off[s] < off + bytes;
                    }
                    if (!clash) break;
                    if (!wait_bar(&empty[oldest % NSLOT], (uint32_t)(oldest / NSLOT) & 1u, p, 1, li, it)) {
                        ok = false;
                        break;
                    }
                    ++oldest;
                }
                if (!ok) break;
                const int s = n % NSLOT;
                q_off[s] = off;
                q_len[s] = bytes;
                const int tile = it / H.S, step = it - tile * H.S;
                uint8_t *dst = ring + off;
                if (H.whole) {
                    if (lane == 0) {
                        const int rows = min(16, H.N - tile * 16);
                        const uint32_t sz = (uint32_t)(((int64_t)rows * H.row_bytes + 15) & ~(int64_t)15);
                        mbar_arrive_expect_tx(&full[s], sz);
                        bulk_g2s(dst, H.W + (int64_t)tile * 16 * H.row_bytes, sz, &full[s]);
                    }
                } else {
                    const int u0 = step * H.upi, nu = min(H.upi, H.units - u0);
                    const int64_t b0 = (int64_t)u0 * H.ub, b1 = (int64_t)(u0 + nu) * H.ub;
                    const int row = tile * 16 + lane;
                    uint32_t sz = 0;
                    const uint8_t *src = nullptr;
                    if (lane < 16 && row < H.N) {
                        const uint8_t *q = H.W + (int64_t)row * H.row_bytes + b0;
                        const uint32_t mis = (uint32_t)((uintptr_t)q & 15);
                        src = q - mis;
                        sz = (uint32_t)((mis + (b1 - b0) + 15) & ~15);
                    }
                    uint32_t total = sz;
#pragma unroll
                    for (int o = 8; o; o >>= 1) total += __shfl_xor_sync(0xffffffffu, total, o);
                    if (lane == 0) mbar_arrive_expect_tx(&full[s], total);
                    __syncwarp();
                    if (sz) bulk_g2s(dst + lane * H.rpb, src, sz, &full[s]);
                }
                __syncwarp();
            }
        }
        return;
    }

    if (warp == CW + 1) {
        // ---------------- reducer ----------------
        int k = 0;  // row blocks of this CTA so far (all linears)
        bool ok = true;
        for (int li = 0; li < p.n; ++li) {
            const Lin &L = p.lin[li];
            // The hot fields in registers (every asm "memory" clobber would
            // otherwise force a reload from global memory).
            const Geo H = geo(L);
            const int i0 = first_item(cta, H.I, G), i1 = first_item(cta + 1, H.I, G);
            if (i1 <= i0) continue;
            const int first_tile = i0 / H.S, last_tile = (i1 - 1) / H.S;
            for (int tb = first_tile; tb <= last_tile; ++tb, ++k) {
                const int sl = k % PSLOTS;
                if (ok) ok = wait_bar(&parked[sl], (uint32_t)(k / PSLOTS) & 1u, p, 2, li, tb);
                const float *q = park + (size_t)sl * CW * 32 * 2;
                // lane = (row r = lane & 15, warp half h = lane >> 4): rows g < 8
                // are .x of lanes g*4 + t, rows g + 8 are .y.
                const int r = lane & 15, h = lane >> 4, g = r & 7, comp = r >> 3;
                float v = 0.f;
#pragma unroll
                for (int w = 0; w < CW / 2; ++w)
#pragma unroll
                    for (int t = 0; t < 4; ++t) v += q[((h * (CW / 2) + w) * 32 + g * 4 + t) * 2 + comp];
                v += __shfl_xor_sync(0xffffffffu, v, 16);
                __syncwarp();
                if (lane == 0) mbar_arrive(&freed[sl]);
                const bool valid = lane < 16 && tb * 16 + lane < H.N;
                const bool whole = tb * H.S >= i0 && (tb + 1) * H.S <= i1;
                if (whole) {
                    store_block(L, p.nranks, ep, tb * 16, v, valid);
                } else {
                    // Cut between CTAs: publish; the last contributor finishes.
                    const int which = tb == first_tile ? 0 : 1;
                    float *wsp = L.ws + ((int64_t)cta * 2 + which) * 16;
                    if (lane < 16) wsp[lane] = v;
                    // The tile's contributors are the owners of its S items (with
                    // fewer items than CTAs, CTAs between them may own none).
                    int owners = 0;
                    for (int i = tb * H.S, prev = -1; i < (tb + 1) * H.S; ++i) {
                        const int c = cta_of_item(i, H.I, G);
                        owners += c != prev;
                        prev = c;
                    }
                    __syncwarp();
                    int fin = 0;
                    if (lane == 0) {
                        __threadfence();
                        fin = atomicAdd(&L.cnt[tb], 1) == owners - 1;
                        if (fin) __threadfence();
                    }
                    if (__shfl_sync(0xffffffffu, fin, 0)) {
                        float t = 0.f;
                        if (lane < 16)
                            for (int i = tb * H.S, prev = -1; i < (tb + 1) * H.S; ++i) {
                                const int c = cta_of_item(i, H.I, G);
                                if (c == prev) continue;
                                prev = c;
                                const int wc = tb == first_item(c, H.I, G) / H.S ? 0 : 1;
                                t += __ldcg(L.ws + ((int64_t)c * 2 + wc) * 16 + lane);
                            }
                        store_block(L, p.nranks, ep, tb * 16, t, valid);
                        if (lane == 0) L.cnt[tb] = 0;
                    }
                }
                if (p.trace && lane == 0) atomicMax(&p.trace[2 * li + 1], gtimer());
            }
        }
        __syncwarp();
        if (lane == 0 && atomicAdd(p.done, 1) == G - 1) {
            *p.done = 0;
            __threadfence();
            atomicAdd(p.epoch, 1);
        }
        return;
    }

    // ---------------- consumers ----------------
    const int g = lane >> 2, t = lane & 3;
    bool ok = true;
    int head = 0, n = 0;   // ring replay (same placement as the producer)
    int ubase = 0;         // units of earlier items, mod CW (round-robin start)
    int k = 0, park_slot = 0;
    uint32_t park_phase = 0;
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    const uint8_t *x_have = nullptr;  // plain activation row resident in xs (nullptr: none)
    bool x_have_q6 = false;
    int x_r0 = 0, x_r1 = 0;
    for (int li = 0; li < p.n; ++li) {
        const Lin &L = p.lin[li];
        // The hot fields in registers (every asm "memory" clobber would
        // otherwise force a reload from global memory).
        const Geo H = geo(L);
        const int i0 = first_item(cta, H.I, G), i1 = first_item(cta + 1, H.I, G);
        if (i1 <= i0) continue;
        const bool q6 = H.qt == VKF_DEQUANT_Q6_K, q5 = H.qt == VKF_DEQUANT_Q5_K;
        const int sum_b = q6 ? 96 : 64;
        // Activations of this linear: the runs of the units this CTA's items
        // cover.  The barrier before keeps the previous linear's readers.
        // Skipped when the previous linear of this CTA quantised the same
        // plain row, with the same sums layout, over at least these runs.
        const int ua = (i0 % H.S) * H.upi, ue = H.S == 1 ? H.units : std::min(H.units, ((i1 - 1) % H.S + 1) * H.upi);
        const bool all_units = (i1 - i0) >= H.S || i0 / H.S != (i1 - 1) / H.S;
        const int r0 = all_units ? 0 : ua * 8, r1 = all_units ? H.units * 8 : ue * 8;
        const bool same_x = !L.x_ll && L.X == x_have && q6 == x_have_q6 && r0 >= x_r0 && r1 <= x_r1;
        if (!same_x) {
            consumer_bar();
            for (int sb = r0 + threadIdx.x; sb < r1; sb += CW * 32) {
                uint4 v[4];
                load_run(L, ep, sb, v, p, li);
                quantize_run(v, sb, q6, xs, sums);
            }
            consumer_bar();
            x_have = L.x_ll ? nullptr : L.X;
            x_have_q6 = q6;
            x_r0 = r0;
            x_r1 = r1;
        }
        if (p.trace && threadIdx.x == 0) atomicMax(&p.trace[2 * li], gtimer());
        const int64_t row_off_a = (int64_t)g * H.row_bytes, row_off_b = (int64_t)(g + 8) * H.row_bytes;
        for (int it = i0; it < i1; ++it, ++n) {
            const int s = n % NSLOT;
            const int off = ring_place(head, H.item_bytes, p.ring_bytes);
            if (ok) ok = wait_bar(&full[s], (uint32_t)(n / NSLOT) & 1u, p, 3, li, it);
            const int tile = it / H.S, step = it - tile * H.S;
            const int u0 = step * H.upi, nu = min(H.upi, H.units - u0);
            if (ok) {
                const uint8_t *st = ring + off;
                const uint8_t *ra, *rb;
                if (H.whole) {
                    ra = st + row_off_a;
                    rb = st + row_off_b;
                } else {
                    const uintptr_t ga = (uintptr_t)H.W + ((int64_t)tile * 16 + g) * H.row_bytes + (int64_t)u0 * H.ub;
                    const uintptr_t gb = ga + 8 * H.row_bytes;
                    ra = st + g * H.rpb + (ga & 15);
                    rb = st + (g + 8) * H.rpb + (gb & 15);
                }
                int u = warp - ubase;
                if (u < 0) u += CW;
                if (q6) {
                    // Rows a multiple of 4 bytes: every lane's unit has the same alignment
                // (the form must be chosen warp-uniformly around mma.sync); else
                // the shifted form, which serves either alignment.
                const bool rows4 = (H.row_bytes & 3) == 0;
                for (; u < nu; u += CW) {
                        const int unit = u0 + u;
                        const uint8_t *pa = ra + u * 210, *pb = rb + u * 210;
                        const float *sx = reinterpret_cast<const float *>(sums + unit * 96);
                        if (!rows4) StepQ6i::run<2>(pa, pb, xs + unit * 512, g, sx, t, acc);
                        else if ((((uintptr_t)pa | (uintptr_t)pb) & 3) == 0) StepQ6i::run<0>(pa, pb, xs + unit * 512, g, sx, t, acc);
                        else StepQ6i::run<1>(pa, pb, xs + unit * 512, g, sx, t, acc);
                    }
                } else if (q5) {
                    for (; u < nu; u += CW) {
                        const int unit = u0 + u;
                        StepK1i<true>::run(ra + u * 176, rb + u * 176, xs + unit * 512, g == t, g == t + 4,
                                           reinterpret_cast<const float *>(sums + unit * sum_b), t, acc);
                    }
                } else {
                    for (; u < nu; u += CW) {
                        const int unit = u0 + u;
                        StepK1i<false>::run(ra + u * 144, rb + u * 144, xs + unit * 512, g == t, g == t + 4,
                                            reinterpret_cast<const float *>(sums + unit * sum_b), t, acc);
                    }
                }
            }
            ubase += nu;
            while (ubase >= CW) ubase -= CW;
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
            const bool tile_end = step == H.S - 1 || it + 1 == i1;
            if (!tile_end) continue;
            const int sl = park_slot;
            if (k >= PSLOTS && ok) ok = wait_bar(&freed[sl], park_phase ^ 1u, p, 4, li, it);
            float *pp = park + ((size_t)(sl * CW + warp) * 32 + lane) * 2;
            *reinterpret_cast<float2 *>(pp) = make_float2(acc[0] + acc[1], acc[2] + acc[3]);
            acc[0] = acc[1] = acc[2] = acc[3] = 0.f;
            __syncwarp();
            if (lane == 0) mbar_arrive(&parked[sl]);
            ++k;
            if (++park_slot == PSLOTS) {
                park_slot = 0;
                park_phase ^= 1u;
            }
        }
    }
}

// Worst shared-memory bank multiplicity of the decode's weight loads with rows
// `pitch` bytes apart (same rule as the per-linear GEMV: contiguous row
// blocks only where this stays <= 2).
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

}  // namespace chain
}  // namespace vkf

using namespace vkf;

struct vkf_chain {
    int device = -1;
    int world = 1, rank = 0;
    chain::Params p{};
    size_t smem = 0;
    void *dev_mem = nullptr;   // descriptors | scratch | counters | epoch, done
    unsigned long long *trace = nullptr;
    int n = 0;
};

static size_t up(size_t v, size_t m) { return (v + m - 1) / m * m; }

extern "C" int vkflame_chain_create(const vkf_chain_linear_t *lin, int n, int world, int rank, unsigned flags,
                                    vkf_chain_t **out) {
    using namespace vkf::chain;
    if (!out || !lin || n <= 0 || world < 1 || world > VKF_MAX_RANKS || rank < 0 || rank >= world)
        return set_status(VKF_ERR_INVALID);
    *out = nullptr;
    DeviceState *ds = device_state();
    if (!ds) return set_status(VKF_ERR_NO_DEVICE);
    const int G = ds->sm_count;
    // Bytes of one row per ring item (whole rows up to this, else K-ranges);
    // VKFLAME_CHAIN_ROW_BUDGET overrides it for measurements.
    static const int row_budget = [] {
        const char *e = getenv("VKFLAME_CHAIN_ROW_BUDGET");
        const int v = e ? atoi(e) : 0;
        return v >= 256 ? v : ROW_BUDGET;
    }();
    std::vector<Lin> L(n);
    int units_max = 1;
    for (int i = 0; i < n; ++i) {
        const vkf_chain_linear_t &c = lin[i];
        Lin &d = L[i];
        if (c.wtype != VKF_DEQUANT_Q4_K && c.wtype != VKF_DEQUANT_Q5_K && c.wtype != VKF_DEQUANT_Q6_K)
            return set_status(VKF_ERR_UNSUPPORTED);
        if (c.K <= 0 || c.K % 256 || c.N <= 0 || c.N % 2 || !c.W) return set_status(VKF_ERR_INVALID);
        d.W = (const uint8_t *)c.W;
        d.qt = c.wtype;
        d.K = c.K;
        d.N = c.N;
        d.units = c.K / 256;
        d.ub = c.wtype == VKF_DEQUANT_Q4_K ? 144 : c.wtype == VKF_DEQUANT_Q5_K ? 176 : 210;
        d.row_bytes = (int64_t)d.units * d.ub;
        const uintptr_t wa = (uintptr_t)c.W;
        if (c.wtype == VKF_DEQUANT_Q6_K ? (wa & 1) : (wa & 3)) return set_status(VKF_ERR_BADPTR);
        const bool owned = c.wtype != VKF_DEQUANT_Q6_K;
        d.T = (c.N + 15) / 16;
        if (16 * d.row_bytes <= 16 * row_budget && (wa & 15) == 0 && (16 * d.row_bytes) % 16 == 0 &&
            pitch_conflicts(d.row_bytes, owned) <= 2) {
            d.whole = 1;
            d.S = 1;
            d.upi = d.units;
            d.rpb = 0;
            d.item_bytes = (int)up((size_t)16 * d.row_bytes, 128);
        } else {
            d.whole = 0;
            const int upi_max = std::max(1, row_budget / d.ub);
            d.S = (d.units + upi_max - 1) / upi_max;
            d.upi = (d.units + d.S - 1) / d.S;
            const int ng = ((d.upi * d.ub + 15) / 16 + 1) | 1;  // odd granule count per row
            d.rpb = ng * 16;
            d.item_bytes = (int)up((size_t)16 * d.rpb, 128);
        }
        d.I = d.T * d.S;
        units_max = std::max(units_max, d.units);
        // activations
        if (c.x_src >= 0) {
            if (c.x_src >= i || world < 1) return set_status(VKF_ERR_INVALID);
            const vkf_chain_linear_t &src = lin[c.x_src];
            if (!src.y_rank[rank] || src.y_plain || src.N * world < c.K) return set_status(VKF_ERR_INVALID);
            d.x_ll = 1;
            d.X = nullptr;  // resolved below: this rank's buffer 0 (word 0)
            d.x_stride = src.y_stride;
        } else {
            if (!c.x_plain || ((uintptr_t)c.x_plain & 15)) return set_status(VKF_ERR_BADPTR);
            d.x_ll = 0;
            d.X = (const uint8_t *)c.x_plain;
        }
        // outputs
        d.y_plain = (__half *)c.y_plain;
        if (!c.y_plain) {
            for (int q = 0; q < world; ++q) {
                if (!c.y_rank[q] || ((uintptr_t)c.y_rank[q] & 7)) return set_status(VKF_ERR_BADPTR);
                d.ypeer[q] = (uint8_t *)c.y_rank[q];
            }
            if (c.y_stride % 16) return set_status(VKF_ERR_INVALID);
            d.y_stride = c.y_stride;
        } else if (((uintptr_t)c.y_plain & 1) || world != 1) {
            return set_status(VKF_ERR_INVALID);
        }
    }
    // Shared memory: resident activations + sums, park slots, ring, barriers.
    const int xs_bytes = (int)up((size_t)units_max * 512, 128);
    const int sums_bytes = (int)up((size_t)units_max * 96, 128);
    const int park_bytes = PSLOTS * PARK_BYTES;
    const int bar_bytes = (2 * NSLOT + 2 * PSLOTS) * 8;
    const int fixed = xs_bytes + sums_bytes + park_bytes + (int)up(bar_bytes, 128);
    const int ring = SMEM - fixed;
    int item_max = 0;
    for (auto &d : L) item_max = std::max(item_max, d.item_bytes);
    if (ring < 2 * item_max) return set_status(VKF_ERR_UNSUPPORTED);
    // Device memory: descriptors, per-linear scratch and counters, epoch/done.
    size_t off_ws = up(sizeof(Lin) * n, 256), total = off_ws;
    std::vector<size_t> ws_off(n), cnt_off(n);
    for (int i = 0; i < n; ++i) {
        ws_off[i] = total;
        total += up((size_t)G * 2 * 16 * sizeof(float), 256);
    }
    for (int i = 0; i < n; ++i) {
        cnt_off[i] = total;
        total += up((size_t)L[i].T * sizeof(int), 256);
    }
    const size_t off_ctl = total;
    total += 256;
    const size_t off_trace = total;
    const bool tracing = (flags & VKF_CHAIN_TRACE) != 0;
    if (tracing) total += up((size_t)n * 2 * sizeof(unsigned long long), 256);
    void *mem = nullptr;
    if (cudaMalloc(&mem, total) != cudaSuccess) {
        cudaGetLastError();
        return set_status(VKF_ERR_NOMEM);
    }
    uint8_t *base = (uint8_t *)mem;
    for (int i = 0; i < n; ++i) {
        L[i].ws = (float *)(base + ws_off[i]);
        L[i].cnt = (int *)(base + cnt_off[i]);
        if (L[i].x_ll) {
            // This rank's own buffer 0 of the source linear: its y_rank[rank]
            // points at this rank's first word; step back to word 0.
            const vkf_chain_linear_t &src = lin[lin[i].x_src];
            L[i].X = (const uint8_t *)src.y_rank[rank] - (int64_t)rank * (src.N / 2) * 8;
        }
    }
    // Both run on the legacy default stream, which does not order itself
    // before a non-blocking stream's chain launch: finish them here.
    if (cudaMemset(mem, 0, total) != cudaSuccess ||
        cudaMemcpy(mem, L.data(), sizeof(Lin) * n, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(mem);
        return set_status(VKF_ERR_CUDA);
    }
    auto *c = new vkf_chain;
    c->device = ds->device;
    c->world = world;
    c->rank = rank;
    c->n = n;
    c->dev_mem = mem;
    c->smem = SMEM;
    Params &p = c->p;
    p.lin = (const Lin *)mem;
    p.n = n;
    p.nranks = world;
    p.G = G;
    p.ring_bytes = ring;
    p.off_sums = xs_bytes;
    p.off_park = xs_bytes + sums_bytes;
    p.off_ring = p.off_park + park_bytes;
    p.off_bar = p.off_ring + ring;
    p.epoch = (int *)(base + off_ctl);
    p.done = (int *)(base + off_ctl + 4);
    p.fail = (int *)(base + off_ctl + 16);
    p.err = ds->d_error;
    p.trace = tracing ? (unsigned long long *)(base + off_trace) : nullptr;
    c->trace = p.trace;
    if (cudaFuncSetAttribute(chain_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess) {
        cudaGetLastError();
        cudaFree(mem);
        delete c;
        return set_status(VKF_ERR_CUDA);
    }
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, chain_kernel, NT, SMEM) != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        cudaFree(mem);
        delete c;
        return set_status(VKF_ERR_UNSUPPORTED);
    }
    *out = c;
    return set_status(VKF_OK);
}

extern "C" int vkflame_chain_run(vkf_chain_t *c, void *stream) {
    if (!c) return set_status(VKF_ERR_INVALID);
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev != c->device) return set_status(VKF_ERR_INVALID);
    if (c->trace) {
        if (cudaMemsetAsync(c->trace, 0, (size_t)c->n * 16, (cudaStream_t)stream) != cudaSuccess)
            return set_status(VKF_ERR_CUDA);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(c->p.G);
    cfg.blockDim = dim3(chain::NT);
    cfg.dynamicSmemBytes = c->smem;
    cfg.stream = (cudaStream_t)stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: CTAs wait on one another's outputs
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, chain::chain_kernel, c->p);
    return set_status(check_launch());
}

extern "C" int vkflame_chain_trace(const vkf_chain_t *c, unsigned long long *host) {
    if (!c || !host || !c->trace) return set_status(VKF_ERR_INVALID);
    return set_status(cudaMemcpy(host, c->trace, (size_t)c->n * 16, cudaMemcpyDeviceToHost) == cudaSuccess
                          ? VKF_OK
                          : VKF_ERR_CUDA);
}

extern "C" int vkflame_chain_epoch(const vkf_chain_t *c, int *host) {
    if (!c || !host) return set_status(VKF_ERR_INVALID);
    return set_status(cudaMemcpy(host, c->p.epoch, sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess ? VKF_OK
                                                                                                       : VKF_ERR_CUDA);
}

extern "C" int vkflame_chain_status(const vkf_chain_t *c, int *fail) {
    if (!c || !fail) return set_status(VKF_ERR_INVALID);
    return set_status(cudaMemcpy(fail, c->p.fail, 4 * sizeof(int), cudaMemcpyDeviceToHost) == cudaSuccess
                          ? VKF_OK
                          : VKF_ERR_CUDA);
}

extern "C" int vkflame_chain_destroy(vkf_chain_t *c) {
    if (!c) return set_status(VKF_OK);
    int cur = 0;
    cudaGetDevice(&cur);
    cudaSetDevice(c->device);
    cudaDeviceSynchronize();
    cudaFree(c->dev_mem);
    cudaSetDevice(cur);
    delete c;
    return set_status(VKF_OK);
}
