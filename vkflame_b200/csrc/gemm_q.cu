// gemm_q.cu — prefill GEMM (M > 8) of ggml-quantised weights with the
// dequant fused into shared memory, on tcgen05 tensor cores.
//
//   Y[m, n] = sum_k X[m, k] * dequant(W)[n, k]      X fp16 [M x K], W ggml rows
//
// Replaces the reference's quantised mul_mat chain (shim/hip_runtime_shim.cpp:
// 1129-1166: dequant W to an fp32 buffer, dequant X, then a K-serial GEMM)
// and this library's own earlier widen-then-GEMM form: W is read from HBM
// once, as packed blocks, and never exists in memory as fp16.
//
// Roles are swapped against the plain GEMM: the weight tile is the MMA's A
// operand (128 weight rows = the 128 TMEM lanes) and the activations the B
// operand (NB x BX rows of X = TMEM columns, up to 512), so a weight tile is
// dequantised once per up to 512 activation rows and the accumulator's lanes
// are output columns.
//
// Work split (stream-K): the flattened (tile, 256-value K stage) space is cut
// into one equal contiguous range per CTA, so every SM does the same number
// of MMAs whatever the tile count.  A CTA's range is [tail of a tile][whole
// tiles][head of a tile]: whole tiles store Y; a tile's later parts (tails,
// or a middle when a range lies inside one tile) publish fp32 partials to
// scratch at the START of their CTAs' runs; the tile's head is processed at
// the END of its CTA's run, so that CTA finds the partials ready (a bounded
// wait guards it), adds them in CTA order (deterministic) and stores Y.
//
// Warps:
//   0        TMA producer of the X tiles (fp16, 128-byte swizzle, K-major),
//            one 64-value K-block per stage;
//   1        allocates the TMEM accumulator (double-buffered when 2 x NB x BX
//            columns fit); one thread issues tcgen05.mma kind::f16;
//   2..5     epilogue: tcgen05.ld, partial publish / fixup, Y stores;
//   6        TMA producer of the packed weight bytes: ONE 2-D tensor copy
//            per 128 rows x 256 values (a map over the ggml buffer with
//            8-byte elements; no per-row operations);
//   7..7+CV  converters: decode the packed bytes of a K-block into fp16 and
//            store them in the 128-byte-swizzled K-major layout tcgen05
//            reads (the layout a SWIZZLE_128B tensor copy would write), then
//            fence the generic-proxy stores for the async proxy and arrive.
// Each fp16 weight is the value the reference's dequant shader computes,
// rounded once to fp16 (the same rounding as the widen path it replaces).
// The MMA stage's barrier completes when the X copy has landed AND all
// converter warps have arrived.

#include "tc_common.cuh"
#include "rt_internal.h"

#include <cuda.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <climits>
#include <type_traits>

namespace vkf {
namespace qgemm {

constexpr int BW = 128;   // weight rows per tile (MMA M, TMEM lanes)
constexpr int KV = 64;    // K values per MMA stage (128 bytes of fp16 per row)
constexpr int RV = 256;   // K values per packed-weight stage (the work unit)
#ifndef VKF_QGEMM_CV
#define VKF_QGEMM_CV 8
#endif
constexpr int CV = VKF_QGEMM_CV;  // converter warps
constexpr int RPL = BW / (8 * CV);  // rows per converter lane (8 row groups of 4 lanes per warp)
constexpr int W_RAW = 6, W_CONV = 7;
constexpr int NT = 32 * (W_CONV + CV);
constexpr int A_BYTES = BW * 128;
constexpr int SMEM_CAP = 232448;
constexpr int EPI_BUF = 16384;  // one Y staging buffer: 32 rows (one TMEM chunk) of 128 fp32 columns

// Packed bytes of one row's 256 values.
template <int QT>
struct Packed;
template <> struct Packed<VKF_DEQUANT_Q4_0> { static constexpr int RB = 8 * 18; };
template <> struct Packed<VKF_DEQUANT_Q8_0> { static constexpr int RB = 8 * 34; };
template <> struct Packed<VKF_DEQUANT_Q4_K> { static constexpr int RB = 144; };
template <> struct Packed<VKF_DEQUANT_Q5_K> { static constexpr int RB = 176; };
// Q6_K: 210 packed bytes per row and 256 values, so row pitches are not
// 16-byte multiples and no tensor map describes the rows.  Each row's 210
// bytes are fetched as 16-byte cp.async granules from the boundary below
// them (at most 224 bytes) into a 240-byte slot (15 granules: odd, so eight
// consecutive rows' 16-byte loads hit eight distinct bank groups); the
// converter reads the row at the slot + its start's offset mod 16.
template <> struct Packed<VKF_DEQUANT_Q6_K> { static constexpr int RB = 240; };
template <int QT> constexpr bool row_copies() { return QT == VKF_DEQUANT_Q6_K; }
constexpr int Q6_ROW = 210;

#ifdef VKF_QGEMM_TIMING
// Cycle accumulators per CTA: [0] converter raw wait, [1] converter empty
// wait, [2] converter work, [3] MMA full wait, [4] MMA thread done (since
// start), [5] X producer empty wait, [6] epilogue busy, [7] total.
__device__ unsigned long long g_qt[512][8];
#define QT_T0 const long long _t0 = clock64()
#define QT_ACC(i) if (lane == 0) atomicAdd(&g_qt[blockIdx.x][i], (unsigned long long)(clock64() - _t0))
#else
#define QT_T0
#define QT_ACC(i)
#endif

struct Params {
    int M, N, K;
    void *Y;
    int64_t ldy;
    int y_f16;
    int y_tma;        // Y written by 2-D tensor stores (16-byte aligned rows)
    int prefetch;     // W written by no kernel: stream it before the dependency wait
    int units;        // tiles x (K / 256)
    float *ws;        // per CTA: [NB*BX/4][128][4] fp32 partials (4-column groups)
    int *flags;       // [grid] partial published (reset by the consumer)
    unsigned *err;
    const uint8_t *W; // the ggml rows (row-copy formats)
    int64_t row_bytes;
};

// Segment walk shared by every role: CTA c owns units [u0, u1); a segment is
// the part of one tile inside that range.
struct Seg {
    int tile, kr0, kr1;
};
__device__ __forceinline__ int unit_begin(int c, int units) { return (int)((int64_t)c * units / gridDim.x); }
__device__ __forceinline__ int cta_of_unit(int u, int units) {
    return (int)(((int64_t)(u + 1) * gridDim.x - 1) / units);
}

__device__ __forceinline__ uint32_t lds16(const uint8_t *p) { return *reinterpret_cast<const uint16_t *>(p); }
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t *>(&h); }
__device__ __forceinline__ __half2 u2h(uint32_t u) { return *reinterpret_cast<__half2 *>(&u); }

// get_scale_min_k4 (dequant_q4_k.glsl:16-24) for sub-blocks j and j+1
// (j even) from the 12 packed scale bytes.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t *s, int &sc, int &mn) {
    if (j < 4) {
        sc = s[j] & 63;
        mn = s[j + 4] & 63;
    } else {
        sc = (s[j + 4] & 0xF) | ((s[j - 4] >> 6) << 4);
        mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// One converter lane's share of a 64-value K-block of row `rp` (the row's
// 256-value packed stage): 16 values as two 16-byte chunks (chunk indices
// within the K-block in ca, cb).  cp = lane & 3 selects which 16.
template <int QT>
__device__ __forceinline__ void convert16(const uint8_t *rp, int kk, int cp, uint4 &oa, uint4 &ob, int &ca,
                                          int &cb) {
    uint32_t o[8];
    if constexpr (QT == VKF_DEQUANT_Q8_0) {  // dequant_q8_0.glsl: d * q; chunks 2cp, 2cp+1
        const uint8_t *bp = rp + 34 * (2 * kk + (cp >> 1));
        const __half2 d2 = __half2half2(*reinterpret_cast<const __half *>(bp));
        // 16 code bytes at a 2-byte aligned address: five aligned words, shifted.
        const uint8_t *cpt = bp + 2 + 16 * (cp & 1);
        const uint32_t *wp = reinterpret_cast<const uint32_t *>((uintptr_t)cpt & ~(uintptr_t)3);
        const uint32_t sh = ((uintptr_t)cpt & 3) * 8;
        uint32_t w[5];
#pragma unroll
        for (int i = 0; i < 5; ++i) w[i] = wp[i];
        const __half2 off = __float2half2_rn(1152.0f);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            // fp16 1024 + (q + 128), exact; minus 1152 = q, exact; one rounding in the product.
            const uint32_t x = __funnelshift_r(w[i], w[i + 1], sh) ^ 0x80808080u;
            o[2 * i] = h2u(__hmul2(__hsub2(u2h(__byte_perm(x, 0x64646464u, 0x4140)), off), d2));
            o[2 * i + 1] = h2u(__hmul2(__hsub2(u2h(__byte_perm(x, 0x64646464u, 0x4342)), off), d2));
        }
        ca = 2 * cp;
        cb = 2 * cp + 1;
    } else if constexpr (QT == VKF_DEQUANT_Q4_0) {  // dequant_q4_0.glsl: d * (q - 8)
        // chunk ca = low nibbles of 8 code bytes, cb = ca + 2 their high nibbles
        const uint8_t *bp = rp + 18 * (2 * kk + (cp >> 1));
        const __half2 d2 = __half2half2(*reinterpret_cast<const __half *>(bp));
        const uint8_t *cpt = bp + 2 + 8 * (cp & 1);
        const uint32_t w0 = lds16(cpt) | (lds16(cpt + 2) << 16), w1 = lds16(cpt + 4) | (lds16(cpt + 6) << 16);
        const uint32_t ws[4] = {w0, w1, w0 >> 4, w1 >> 4};
        const __half2 off = __float2half2_rn(1032.0f);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t p0 = __byte_perm(ws[i], 0, 0x4140), p1 = __byte_perm(ws[i], 0, 0x4342);
            o[2 * i] = h2u(__hmul2(__hsub2(u2h((p0 & 0x000F000Fu) | 0x64006400u), off), d2));
            o[2 * i + 1] = h2u(__hmul2(__hsub2(u2h((p1 & 0x000F000Fu) | 0x64006400u), off), d2));
        }
        ca = (cp & 1) + 4 * (cp >> 1);
        cb = ca + 2;
    } else {  // Q4_K / Q5_K, dequant_q4_k.glsl:35-57, dequant_q5_k.glsl:37-74: d*sc*q - dmin*m
        // chunk cp = low nibbles (sub-block 2kk), cp + 4 = high nibbles (2kk + 1)
        constexpr bool Q5 = QT == VKF_DEQUANT_Q5_K;
        const int j = 2 * kk;
        const __half2 d2 = __half2half2(*reinterpret_cast<const __half *>(rp));
        const float dmin = __half2float(*reinterpret_cast<const __half *>(rp + 2));
        int sc0, mn0, sc1, mn1;
        scale_min_k4(j, rp + 4, sc0, mn0);
        scale_min_k4(j + 1, rp + 4, sc1, mn1);
        // Half2 form (as convert32): q * sc exact, then one fma with d and
        // -fp16(dmin * m).
        const __half2 sc2[2] = {__float2half2_rn((float)sc0), __float2half2_rn((float)sc1)};
        const __half2 sco[2] = {__float2half2_rn(-1024.0f * (float)sc0), __float2half2_rn(-1024.0f * (float)sc1)};
        const __half2 mm2[2] = {__float2half2_rn(-dmin * (float)mn0), __float2half2_rn(-dmin * (float)mn1)};
        const uint2 q = *reinterpret_cast<const uint2 *>(rp + (Q5 ? 48 : 16) + 32 * kk + 8 * cp);
        uint2 h = make_uint2(0u, 0u);
        if constexpr (Q5) h = *reinterpret_cast<const uint2 *>(rp + 16 + 8 * cp);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
            const uint32_t qw[2] = {(q.x >> (4 * half)) & 0x0F0F0F0Fu, (q.y >> (4 * half)) & 0x0F0F0F0Fu};
            uint32_t hw[2] = {0u, 0u};
            if constexpr (Q5) {
                hw[0] = ((h.x >> (j + half)) & 0x01010101u) << 4;
                hw[1] = ((h.y >> (j + half)) & 0x01010101u) << 4;
            }
#pragma unroll
            for (int i = 0; i < 2; ++i) {
                const uint32_t c = qw[i] | hw[i];
                const uint32_t p0 = __byte_perm(c, 0x64646464u, 0x5140), p1 = __byte_perm(c, 0x64646464u, 0x7362);
                o[4 * half + 2 * i] = h2u(__hfma2(__hfma2(u2h(p0), sc2[half], sco[half]), d2, mm2[half]));
                o[4 * half + 2 * i + 1] = h2u(__hfma2(__hfma2(u2h(p1), sc2[half], sco[half]), d2, mm2[half]));
            }
        }
        ca = cp;
        cb = cp + 4;
    }
    oa = make_uint4(o[0], o[1], o[2], o[3]);
    ob = make_uint4(o[4], o[5], o[6], o[7]);
}

// 32 values (32-value block / sub-block B, 0..7, of the 256-value stage) of
// one row, as 16 fp16 pairs in K order, for the TMEM-resident A operand.
// rp is the row's stage (16-byte aligned: row pitches are 16-byte
// multiples); loads are 16-byte and, with one row per lane and odd pitches in
// 16-byte units, bank-conflict free.  Same arithmetic as convert16.
template <int QT, int B>
__device__ __forceinline__ void convert32(const uint8_t *rp, uint32_t (&o)[16]) {
    if constexpr (QT == VKF_DEQUANT_Q8_0) {
        constexpr int A0 = (34 * B) & ~15, OFF = 34 * B - A0, NV = (OFF + 34 + 15) / 16;
        uint32_t w[4 * NV + 1] = {};  // +1: the funnel shift's upper word past the window (shift 0 there)
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const uint4 t = *reinterpret_cast<const uint4 *>(rp + A0 + 16 * i);
            w[4 * i] = t.x; w[4 * i + 1] = t.y; w[4 * i + 2] = t.z; w[4 * i + 3] = t.w;
        }
        const uint32_t dw = w[OFF / 4] >> (8 * (OFF % 4));
        const __half2 d2 = __half2half2(__ushort_as_half((unsigned short)(dw & 0xFFFF)));
        const __half2 off = __float2half2_rn(1152.0f);
        constexpr int C0 = OFF + 2;  // first code byte in the window
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const uint32_t x = __funnelshift_r(w[C0 / 4 + j], w[C0 / 4 + j + 1], 8 * (C0 % 4)) ^ 0x80808080u;
            o[2 * j] = h2u(__hmul2(__hsub2(u2h(__byte_perm(x, 0x64646464u, 0x4140)), off), d2));
            o[2 * j + 1] = h2u(__hmul2(__hsub2(u2h(__byte_perm(x, 0x64646464u, 0x4342)), off), d2));
        }
    } else if constexpr (QT == VKF_DEQUANT_Q4_0) {
        constexpr int A0 = (18 * B) & ~15, OFF = 18 * B - A0, NV = (OFF + 18 + 15) / 16;
        uint32_t w[4 * NV + 1] = {};
#pragma unroll
        for (int i = 0; i < NV; ++i) {
            const uint4 t = *reinterpret_cast<const uint4 *>(rp + A0 + 16 * i);
            w[4 * i] = t.x; w[4 * i + 1] = t.y; w[4 * i + 2] = t.z; w[4 * i + 3] = t.w;
        }
        const uint32_t dw = w[OFF / 4] >> (8 * (OFF % 4));
        const __half2 d2 = __half2half2(__ushort_as_half((unsigned short)(dw & 0xFFFF)));
        const __half2 off = __float2half2_rn(1032.0f);
        constexpr int C0 = OFF + 2;
#pragma unroll
        for (int j = 0; j < 4; ++j) {  // code bytes 4j..4j+3: values 4j.. (low), 16+4j.. (high)
            const uint32_t x = __funnelshift_r(w[C0 / 4 + j], w[C0 / 4 + j + 1], 8 * (C0 % 4));
            const uint32_t p0 = __byte_perm(x, 0, 0x4140), p1 = __byte_perm(x, 0, 0x4342);
            o[2 * j] = h2u(__hmul2(__hsub2(u2h((p0 & 0x000F000Fu) | 0x64006400u), off), d2));
            o[2 * j + 1] = h2u(__hmul2(__hsub2(u2h((p1 & 0x000F000Fu) | 0x64006400u), off), d2));
            o[8 + 2 * j] = h2u(__hmul2(__hsub2(u2h(((p0 >> 4) & 0x000F000Fu) | 0x64006400u), off), d2));
            o[8 + 2 * j + 1] = h2u(__hmul2(__hsub2(u2h(((p1 >> 4) & 0x000F000Fu) | 0x64006400u), off), d2));
        }
    } else {  // Q4_K / Q5_K: sub-block B = low (B even) or high (B odd) nibbles of qs[32 (B/2) ..]
        constexpr bool Q5 = QT == VKF_DEQUANT_Q5_K;
        const uint4 hd = *reinterpret_cast<const uint4 *>(rp);
        const uint32_t sw[3] = {hd.y, hd.z, hd.w};  // the 12 scale bytes
        auto sb = [&](int i) { return (int)((sw[i >> 2] >> (8 * (i & 3))) & 0xFF); };
        int sc, mn;
        if constexpr (B < 4) {
            sc = sb(B) & 63;
            mn = sb(B + 4) & 63;
        } else {
            sc = (sb(B + 4) & 0xF) | ((sb(B - 4) >> 6) << 4);
            mn = (sb(B + 4) >> 4) | ((sb(B) >> 6) << 4);
        }
        // Half2 form: (1024 + q) * sc - 1024 * sc = q * sc exactly (an
        // integer < 2048; 1024 * sc <= 64512 is exact too), then one fma
        // with d and -fp16(dmin * m): the weight rounded once, plus the fp16
        // rounding of the min term (<= 2^-12 * 0.63 absolute at this
        // format's largest dmin * m).
        const __half2 d2 = __half2half2(__ushort_as_half((unsigned short)(hd.x & 0xFFFF)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(hd.x >> 16)));
        const __half2 sc2 = __float2half2_rn((float)sc), sco = __float2half2_rn(-1024.0f * (float)sc);
        const __half2 mm2 = __float2half2_rn(-dmin * (float)mn);
        constexpr int QO = (Q5 ? 48 : 16) + 32 * (B / 2);
        const uint4 q0 = *reinterpret_cast<const uint4 *>(rp + QO), q1 = *reinterpret_cast<const uint4 *>(rp + QO + 16);
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        uint32_t hw[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
        if constexpr (Q5) {
            const uint4 h0 = *reinterpret_cast<const uint4 *>(rp + 16), h1 = *reinterpret_cast<const uint4 *>(rp + 32);
            const uint32_t hv[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
            for (int i = 0; i < 8; ++i) hw[i] = ((hv[i] >> B) & 0x01010101u) << 4;
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t c = ((qw[i] >> (4 * (B & 1))) & 0x0F0F0F0Fu) | hw[i];
            const uint32_t p0 = __byte_perm(c, 0x64646464u, 0x5140), p1 = __byte_perm(c, 0x64646464u, 0x7342);
            o[2 * i] = h2u(__hfma2(__hfma2(u2h(p0), sc2, sco), d2, mm2));
            o[2 * i + 1] = h2u(__hfma2(__hfma2(u2h(p1), sc2, sco), d2, mm2));
        }
    }
}

// 32 bytes at (even) byte offset p of a shared-memory row slot (16-byte
// aligned): three aligned 16-byte loads, then the words selected and shifted
// by p's offset within its granule (2-byte granularity).
__device__ __forceinline__ void lds32_at(const uint8_t *slot, int p, uint32_t (&out)[8]) {
    const uint8_t *b = slot + (p & ~15);
    const uint4 a0 = *reinterpret_cast<const uint4 *>(b), a1 = *reinterpret_cast<const uint4 *>(b + 16),
                a2 = *reinterpret_cast<const uint4 *>(b + 32);
    const uint32_t w[12] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w, a2.x, a2.y, a2.z, a2.w};
    // The word offset differs from lane to lane (rows start at different
    // offsets): two levels of predicated selects, no branches (a four-way
    // choice compiled to divergent branches and stalled the converters).
    const bool s2 = (p & 8) != 0, s1 = (p & 4) != 0;
    const uint32_t sh = (uint32_t)(p & 3) * 8;
    uint32_t t[10], v[9];
#pragma unroll
    for (int j = 0; j < 10; ++j) t[j] = s2 ? w[j + 2] : w[j];
#pragma unroll
    for (int j = 0; j < 9; ++j) v[j] = s1 ? t[j + 1] : t[j];
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = __funnelshift_r(v[j], v[j + 1], sh);
}

// Q6_K (dequant_q6_k.glsl:28-58), the 32 values of sub-block B (ip = B / 4,
// s = B % 4): code q = nibble of ql[64 ip + 32 (s & 1) + l] (low for s < 2)
// | bits 2s, 2s + 1 of qh[32 ip + l] << 4; value = d * sc * (q - 32) with
// sc = scales[8 ip + 2 s + l / 16].  In half2: (1024 + q) - 1056 = q - 32
// exactly, times sc (exact unless |sc (q - 32)| > 2048 and odd: one
// rounding of at most 2^-12 relative), times d (one rounding).  The fp32 form
// (exact product, one rounding) took three times the instructions and held
// the prefill to a third of the Q4_K rate.  row: the row's slot; off: the
// row's first byte within it.
template <int B>
__device__ __forceinline__ void convert32_q6(const uint8_t *row, int off, uint32_t (&o)[16]) {
    constexpr int IP = B / 4, S = B % 4;
    uint32_t ql[8], qh[8];
    lds32_at(row, off + 64 * IP + 32 * (S & 1), ql);
    lds32_at(row, off + 128 + 32 * IP, qh);
    const uint32_t scw = *reinterpret_cast<const uint16_t *>(row + off + 192 + 8 * IP + 2 * S);
    const __half2 d2 = __half2half2(__ushort_as_half(*reinterpret_cast<const uint16_t *>(row + off + 208)));
    const __half2 sc0 = __float2half2_rn((float)(int8_t)(scw & 0xFF)), sc1 = __float2half2_rn((float)(int8_t)(scw >> 8));
    const __half2 off2 = __float2half2_rn(1056.0f);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const uint32_t nib = (S >= 2 ? ql[j] >> 4 : ql[j]) & 0x0F0F0F0Fu;
        const uint32_t c = nib | (((qh[j] >> (2 * S)) & 0x03030303u) << 4);
        const __half2 sc = j < 4 ? sc0 : sc1;
        const __half2 q01 = __hsub2(u2h(__byte_perm(c, 0x64646464u, 0x5140)), off2);
        const __half2 q23 = __hsub2(u2h(__byte_perm(c, 0x64646464u, 0x7362)), off2);
        o[2 * j] = h2u(__hmul2(__hmul2(q01, sc), d2));
        o[2 * j + 1] = h2u(__hmul2(__hmul2(q23, sc), d2));
    }
}

// Row (within a group of 8) served by lane group g = lane >> 2, ordered so
// that each 8-lane store phase writes 8 distinct 16-byte bank groups of the
// swizzled tile: chunk sets {2cp} (Q8_0) pair rows r, r^1; {cp} (K-quants)
// rows r, r^4; {(cp&1) + 4(cp>>1)} (Q4_0) rows r, r^2.
template <int QT>
__device__ __forceinline__ int row_of_group(int g) {
    const int lo = g & 1, hi = g >> 1;  // lo: the row pair inside a phase
    if constexpr (QT == VKF_DEQUANT_Q8_0) return 2 * hi + lo;
    else if constexpr (QT == VKF_DEQUANT_Q4_0) return (hi & 1) + 4 * (hi >> 1) + 2 * lo;
    else return hi + 4 * lo;
}

// A later part's published flag; gives up after WAIT_LIMIT_NS like mbar_wait.
__device__ __forceinline__ bool wait_flag(const int *f, unsigned *err) {
    uint64_t t0 = 0;
    for (uint32_t i = 0;; ++i) {
        int v;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
        if (v) return true;
        if ((i & 255) == 0) {
            const uint64_t t = globaltimer_ns();
            if (i == 0) t0 = t;
            else if (t - t0 >= WAIT_LIMIT_NS) break;
        }
        __nanosleep(64);
    }
    if (err) atomicOr(err, VKF_KERR_WAIT_TIMEOUT);
    return false;
}

__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }
// AND of v over the four epilogue warps (keeps their barrier sequences equal).
__device__ __forceinline__ bool epi_all(bool v) {
    uint32_t r;
    asm volatile(
        "{\n .reg .pred p, q;\n setp.ne.u32 q, %1, 0;\n bar.red.and.pred p, 1, 128, q;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(r)
        : "r"((uint32_t)v)
        : "memory");
    return r != 0;
}

template <int QT, int BX, int NB, int NS, int RS, bool ATM>
__global__ void __launch_bounds__(NT, 1)
    qgemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW,
                 const __grid_constant__ CUtensorMap tmY, const __grid_constant__ Params p) {
    constexpr int RB = Packed<QT>::RB;
    constexpr int NC = NB * BX;  // accumulator columns per tile
    // ATM: the converted weight tile lives in TMEM (NS stages x 32 columns
    // after the accumulators) instead of shared memory.
    constexpr int BOFF = ATM ? 0 : A_BYTES;  // X tile offset within a stage
    constexpr int B_BYTES = NC * 128, STAGE = BOFF + B_BYTES;
    constexpr int RAW_BYTES = (BW * RB + 127) / 128 * 128;
    constexpr int A_COLS = ATM ? NS * 32 : 0;
    constexpr int NBUF = 2 * NC + A_COLS <= 512 ? 2 : 1;
    static_assert(NC + A_COLS <= 512, "TMEM columns");
    constexpr int TNEED = NBUF * NC + A_COLS;
    constexpr uint32_t IDESC = tc::instr_desc(tc::KIND_F16, BW, BX);
    constexpr uint32_t TCOLS = TNEED <= 32 ? 32 : TNEED <= 64 ? 64 : TNEED <= 128 ? 128 : TNEED <= 256 ? 256 : 512;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    uint8_t *raw = smem + NS * STAGE;
    uint8_t *ystage = raw + RS * RAW_BYTES;  // 2 x EPI_BUF
    uint64_t *ab_full = reinterpret_cast<uint64_t *>(ystage + 2 * EPI_BUF);
    uint64_t *ab_empty = ab_full + NS;
    uint64_t *raw_full = ab_empty + NS;
    uint64_t *raw_empty = raw_full + RS;
    uint64_t *acc_full = raw_empty + RS;
    uint64_t *acc_empty = acc_full + 2;
    uint32_t *tslot = reinterpret_cast<uint32_t *>(acc_empty + 2);
    int *sflag = reinterpret_cast<int *>(tslot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int x_tiles = (p.M + NC - 1) / NC;
    const int KR = p.K / RV;
    const int u_begin = unit_begin(blockIdx.x, p.units), u_end = unit_begin(blockIdx.x + 1, p.units);
    auto seg_at = [&](int u) {
        Seg sg;
        sg.tile = u / KR;
        sg.kr0 = u - sg.tile * KR;
        sg.kr1 = min(KR, sg.kr0 + (u_end - u));
        return sg;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&ab_full[s], CV + 1);
            mbar_init(&ab_empty[s], 1);
        }
        for (int s = 0; s < RS; ++s) {
            mbar_init(&raw_full[s], row_copies<QT>() ? 32 : 1);  // row copies: one arrival per producer lane
            mbar_init(&raw_empty[s], CV);
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
#ifdef VKF_QGEMM_TIMING
    const long long t_start = clock64();
#endif

    // Programmatic dependent launch: dependents may start their set-up now.
    // Everything another kernel may write (X, Y, the scratch partials and
    // flags, and W unless it is static) is touched only after the wait.
    asm volatile("griddepcontrol.launch_dependents;");
    if (warp == 0) {
        // ---- X tiles: NB boxes of BX rows per K-block ----
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (lane == 0) {
            int g = 0;
            bool ok = true;
            for (int u = u_begin; u < u_end && ok;) {
                const Seg sg = seg_at(u);
                u += sg.kr1 - sg.kr0;
                const int m0 = (sg.tile % x_tiles) * NC;
                for (int kb = sg.kr0 * (RV / KV); kb < sg.kr1 * (RV / KV); ++kb, ++g) {
                    const int s = g % NS;
                    {
                        QT_T0;
                        if (g >= NS && !(ok = mbar_wait(&ab_empty[s], ((g / NS) & 1) ^ 1, p.err))) break;
                        QT_ACC(5);
                    }
                    mbar_arrive_expect_tx(&ab_full[s], B_BYTES);
#pragma unroll
                    for (int h = 0; h < NB; ++h)
                        tc::tma_load_2d(smem + s * STAGE + BOFF + h * BX * 128, &tmX, kb * KV, m0 + h * BX,
                                        &ab_full[s]);
                }
            }
        }
    } else if (warp == W_RAW) {
        // ---- packed weight bytes: one tensor copy per 128 rows x 256 values ----
        if (!p.prefetch) asm volatile("griddepcontrol.wait;" ::: "memory");
        if constexpr (row_copies<QT>()) {
            // 16-byte cp.async granules (4 rows per lane, at most 14 granules
            // from the boundary below each row's start): one bulk copy per row
            // measured 1.5x slower (the TMA unit's operation rate at 224-byte
            // copies).  Each lane
            // arrives on the stage barrier (count 32) when its copies land.
            int g = 0;
            bool ok = true;
            for (int u = u_begin; u < u_end && ok;) {
                const Seg sg = seg_at(u);
                u += sg.kr1 - sg.kr0;
                const int n0 = (sg.tile / x_tiles) * BW;
                for (int kr = sg.kr0; kr < sg.kr1; ++kr, ++g) {
                    const int s = g % RS;
                    if (g >= RS && !(ok = mbar_wait(&raw_empty[s], ((g / RS) & 1) ^ 1, p.err))) break;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const int r = lane + 32 * i;
                        if (n0 + r >= p.N) continue;
                        const uint8_t *q = p.W + (int64_t)(n0 + r) * p.row_bytes + (int64_t)kr * Q6_ROW;
                        const uint32_t mis = (uint32_t)((uintptr_t)q & 15);
                        const uint8_t *src = q - mis;
                        const uint32_t dst = smem_addr(raw + s * RAW_BYTES + r * RB);
                        const int ng = (int)((mis + Q6_ROW + 15) >> 4);
                        for (int j = 0; j < ng; ++j)
                            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst + 16 * j), "l"(src + 16 * j)
                                         : "memory");
                    }
                    asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_addr(&raw_full[s]))
                                 : "memory");
                }
            }
        } else if (lane == 0) {
            int g = 0;
            bool ok = true;
            for (int u = u_begin; u < u_end && ok;) {
                const Seg sg = seg_at(u);
                u += sg.kr1 - sg.kr0;
                const int n0 = (sg.tile / x_tiles) * BW;
                for (int kr = sg.kr0; kr < sg.kr1; ++kr, ++g) {
                    const int s = g % RS;
                    if (g >= RS && !(ok = mbar_wait(&raw_empty[s], ((g / RS) & 1) ^ 1, p.err))) break;
                    mbar_arrive_expect_tx(&raw_full[s], BW * RB);
                    tc::tma_load_2d(raw + s * RAW_BYTES, &tmW, kr * (RB / 8), n0, &raw_full[s]);
                }
            }
        }
    } else if (warp >= W_CONV && ATM) {
        // ---- converters, TMEM form: warp owns TMEM lane quarter warp % 4
        // (rows 32 q .. 32 q + 31, one row per lane) and half h of each
        // K-block's 64 values; one tcgen05.st of 16 columns per K-block ----
        const int qq = warp & 3, h = (warp - W_CONV) >> 2;
        const int row = 32 * qq + lane;
        const uint32_t ta0 = tmem0 + ((uint32_t)(32 * qq) << 16) + NBUF * NC + 16 * h;
        int g = 0, gr = 0;
        bool ok = true;
        for (int u = u_begin; u < u_end && ok; ++u, ++gr) {
            const int rs = gr % RS;
            {
                QT_T0;
                if (!(ok = mbar_wait(&raw_full[rs], (gr / RS) & 1, p.err))) break;
                QT_ACC(0);
            }
            const uint8_t *rp = raw + rs * RAW_BYTES + row * RB;
            int roff = 0;  // row-copy formats: the row's first byte within its slot
            if constexpr (row_copies<QT>()) {
                const int tile = u / KR, kr = u - tile * KR;
                const int64_t n = (int64_t)(tile / x_tiles) * BW + row;
                roff = (int)((uintptr_t)(p.W + n * p.row_bytes + (int64_t)kr * Q6_ROW) & 15);
            }
            auto kblock = [&](auto kk_c) {
                constexpr int KK = decltype(kk_c)::value;
                const int s = g % NS;
                if (ok) {
                    QT_T0;
                    if (g >= NS) ok = mbar_wait(&ab_empty[s], ((g / NS) & 1) ^ 1, p.err);
                    QT_ACC(1);
                }
                if (ok) {
                    QT_T0;
                    tc::fence_after_sync();  // the MMAs that read this TMEM stage are complete
                    uint32_t o[16];
                    if constexpr (row_copies<QT>()) {
                        if (h == 0) convert32_q6<2 * KK>(rp, roff, o);
                        else convert32_q6<2 * KK + 1>(rp, roff, o);
                    } else {
                        if (h == 0) convert32<QT, 2 * KK>(rp, o);
                        else convert32<QT, 2 * KK + 1>(rp, o);
                    }
                    tc::tmem_st16(ta0 + 32 * s, o);
                    tc::tmem_wait_st();
                    tc::fence_before_sync();
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&ab_full[s]);
                    QT_ACC(2);
                }
                ++g;
            };
            kblock(std::integral_constant<int, 0>{});
            kblock(std::integral_constant<int, 1>{});
            kblock(std::integral_constant<int, 2>{});
            kblock(std::integral_constant<int, 3>{});
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[rs]);
        }
    } else if (warp >= W_CONV && !row_copies<QT>()) {
        // ---- converters: warp cw owns rows 16 cw .. 16 cw + 15 ----
        const int cw = warp - W_CONV;
        const int cp = lane & 3;
        int rows[RPL];
#pragma unroll
        for (int i = 0; i < RPL; ++i) rows[i] = (BW / CV) * cw + 8 * i + row_of_group<QT>(lane >> 2);
        int g = 0, gr = 0;
        bool ok = true;
        for (int u = u_begin; u < u_end && ok; ++u, ++gr) {
            const int rs = gr % RS;
            {
                QT_T0;
                if (!(ok = mbar_wait(&raw_full[rs], (gr / RS) & 1, p.err))) break;
                QT_ACC(0);
            }
            const uint8_t *rt = raw + rs * RAW_BYTES;
#pragma unroll 1
            for (int kk = 0; kk < RV / KV; ++kk, ++g) {
                const int s = g % NS;
                {
                    QT_T0;
                    if (g >= NS && !(ok = mbar_wait(&ab_empty[s], ((g / NS) & 1) ^ 1, p.err))) break;
                    QT_ACC(1);
                }
                QT_T0;
                uint8_t *at = smem + s * STAGE;
#pragma unroll
                for (int i = 0; i < RPL; ++i) {
                    const int r = rows[i];
                    uint4 va, vb;
                    int ca, cb;
                    convert16<QT>(rt + r * RB, kk, cp, va, vb, ca, cb);
                    uint8_t *rowp = at + (r >> 3) * 1024 + (r & 7) * 128;
                    *reinterpret_cast<uint4 *>(rowp + ((ca ^ (r & 7)) << 4)) = va;
                    *reinterpret_cast<uint4 *>(rowp + ((cb ^ (r & 7)) << 4)) = vb;
                }
                // generic-proxy stores -> visible to the tensor core's async proxy
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
                if (lane == 0) mbar_arrive(&ab_full[s]);
                QT_ACC(2);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&raw_empty[rs]);
        }
    } else if (warp == 1) {
        // ---- MMA issuer ----
        if (lane == 0) {
            int g = 0, it = 0;
            bool ok = true;
            for (int u = u_begin; u < u_end && ok; ++it) {
                const Seg sg = seg_at(u);
                u += sg.kr1 - sg.kr0;
                const int b = NBUF == 2 ? (it & 1) : 0;
                const int use = NBUF == 2 ? (it >> 1) : it;  // earlier uses of buffer b
                if (use >= 1 && !(ok = mbar_wait(&acc_empty[b], (use - 1) & 1, p.err))) break;
                tc::fence_after_sync();
                const uint32_t tmem = tmem0 + b * NC;
                const int kb0 = sg.kr0 * (RV / KV), kb1 = sg.kr1 * (RV / KV);
                for (int kb = kb0; kb < kb1; ++kb, ++g) {
                    const int s = g % NS;
                    {
                        QT_T0;
                        if (!(ok = mbar_wait(&ab_full[s], (g / NS) & 1, p.err))) break;
                        QT_ACC(3);
                    }
                    tc::fence_after_sync();
                    const uint32_t sa = smem_addr(smem + s * STAGE), sb = sa + BOFF;
#pragma unroll
                    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
                        for (int h = 0; h < NB; ++h) {
                            const uint64_t bd = tc::smem_desc_sw128(sb + h * BX * 128 + kk * 32);
                            const uint32_t acc = (kb > kb0 || kk) ? 1u : 0u;
                            if constexpr (ATM)
                                tc::mma_f16_ta(tmem + h * BX, tmem0 + NBUF * NC + 32 * s + 8 * kk, bd, IDESC, acc);
                            else
                                tc::mma<tc::KIND_F16>(tmem + h * BX, tc::smem_desc_sw128(sa + kk * 32), bd, IDESC, acc);
                        }
                    tc::commit(&ab_empty[s]);
                }
                tc::commit(&acc_full[b]);
            }
#ifdef VKF_QGEMM_TIMING
            atomicAdd(&g_qt[blockIdx.x][4], (unsigned long long)(clock64() - t_start));
#endif
        }
    } else {
        // ---- epilogue (warps 2..5): TMEM lane = weight row = output column ----
        const int q = warp & 3;
        asm volatile("griddepcontrol.wait;" ::: "memory");
        const int tid = threadIdx.x - 64;  // 0..127 over the four epilogue warps
        int it = 0;
        uint32_t ybuf = 0;  // Y staging buffers used so far
        for (int u = u_begin; u < u_end; ++it) {
            const Seg sg = seg_at(u);
            u += sg.kr1 - sg.kr0;
            const int b = NBUF == 2 ? (it & 1) : 0;
            const int use = NBUF == 2 ? (it >> 1) : it;
            const int m0 = (sg.tile % x_tiles) * NC, nl = 32 * q + lane, n = (sg.tile / x_tiles) * BW + nl;
            bool ok = epi_all(mbar_wait(&acc_full[b], use & 1, p.err));
#ifdef VKF_QGEMM_TIMING
            const long long te0 = clock64();
#endif
            tc::fence_after_sync();
            const uint32_t tmem = tmem0 + b * NC + ((uint32_t)(32 * q) << 16);
            const bool whole = sg.kr0 == 0 && sg.kr1 == KR;
            if (sg.kr0 > 0) {
                // a later part of the tile: publish the partial for the head's
                // CTA as float4 groups [chunk][4-column group][lane][4], so a
                // warp's store of one group is 512 contiguous bytes
                float4 *wsp = reinterpret_cast<float4 *>(p.ws + (size_t)blockIdx.x * NC * BW) + nl;
#pragma unroll 1
                for (int cc = 0; cc < NC / 32; ++cc) {
                    uint32_t r[32];
                    tc::tmem_ld32(tmem + 32 * cc, r);
#pragma unroll
                    for (int j4 = 0; j4 < 8; ++j4)
                        __stcg(wsp + (size_t)(cc * 8 + j4) * BW,
                               make_float4(__uint_as_float(r[4 * j4]), __uint_as_float(r[4 * j4 + 1]),
                                           __uint_as_float(r[4 * j4 + 2]), __uint_as_float(r[4 * j4 + 3])));
                }
                tc::fence_before_sync();
                epi_bar();
                if (tid == 0) {
                    __threadfence();
                    asm volatile("st.release.gpu.global.b32 [%0], %1;" ::"l"(p.flags + blockIdx.x), "r"(1) : "memory");
                }
            } else {
                // whole tile, or the head: add the later parts (CTAs c+1 .. c_last) first
                int c_last = blockIdx.x;
                if (!whole) {
                    c_last = cta_of_unit(sg.tile * KR + KR - 1, p.units);
                    if (tid == 0) {
                        bool fine = ok;
                        for (int c = blockIdx.x + 1; c <= c_last && fine; ++c) fine = wait_flag(p.flags + c, p.err);
                        *sflag = fine;
                    }
                    epi_bar();
                    ok = ok && *sflag;
                }
#pragma unroll 1
                for (int cc = 0; cc < NC / 32; ++cc) {
                    // partial loads first (independent of TMEM): their L2
                    // latency overlaps the accumulator read
                    float v[32];
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = 0.f;
                    if (ok)
                        for (int c = blockIdx.x + 1; c <= c_last; ++c) {
                            const float4 *wsp = reinterpret_cast<const float4 *>(p.ws + (size_t)c * NC * BW) +
                                                (size_t)(cc * 8) * BW + nl;
                            float4 t[8];
#pragma unroll
                            for (int j4 = 0; j4 < 8; ++j4) t[j4] = __ldcg(wsp + (size_t)j4 * BW);
#pragma unroll
                            for (int j4 = 0; j4 < 8; ++j4) {
                                v[4 * j4] += t[j4].x;
                                v[4 * j4 + 1] += t[j4].y;
                                v[4 * j4 + 2] += t[j4].z;
                                v[4 * j4 + 3] += t[j4].w;
                            }
                        }
                    uint32_t r[32];
                    tc::tmem_ld32(tmem + 32 * cc, r);
                    const int mc = m0 + 32 * cc;
                    // own part first, then the later parts in CTA order
#pragma unroll
                    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) + v[j];
                    if (p.y_tma) {
                        // Stage the chunk's 32 rows x 128 columns in shared memory and
                        // write them with one tensor store (out-of-range rows
                        // and columns are clipped by the store).  Every
                        // epilogue thread takes part in every barrier.
                        if (mc >= p.M) continue;  // uniform across the epilogue warps
                        auto stage_store = [&](auto sr_c) {
                            constexpr int SR = decltype(sr_c)::value;
#pragma unroll
                            for (int sub = 0; sub < 32; sub += SR, ++ybuf) {
                                uint8_t *buf = ystage + (ybuf & 1) * EPI_BUF;
                                if (tid == 0) tc::bulk_wait_read<1>();
                                epi_bar();
#pragma unroll
                                for (int i = 0; i < SR; ++i) {
                                    if (p.y_f16)
                                        reinterpret_cast<__half *>(buf)[i * BW + nl] = __float2half_rn(v[sub + i]);
                                    else
                                        reinterpret_cast<float *>(buf)[i * BW + nl] = v[sub + i];
                                }
                                tc::fence_proxy_async();
                                epi_bar();
                                if (tid == 0 && ok) {
                                    tc::tma_store_2d(&tmY, buf, n - nl, mc + sub);
                                    tc::bulk_commit();
                                }
                            }
                        };
                        stage_store(std::integral_constant<int, 32>{});
                        continue;
                    }
                    if (!ok || n >= p.N || mc >= p.M) continue;
                    const int nm = min(32, p.M - mc);
                    if (p.y_f16) {
                        __half *yp = reinterpret_cast<__half *>(p.Y) + (int64_t)mc * p.ldy + n;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < nm) yp[(int64_t)j * p.ldy] = __float2half_rn(v[j]);
                    } else {
                        float *yp = reinterpret_cast<float *>(p.Y) + (int64_t)mc * p.ldy + n;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (j < nm) yp[(int64_t)j * p.ldy] = v[j];
                    }
                }
                // flags consumed: leave them zeroed for the next launch
                if (!whole && tid == 0)
                    for (int c = blockIdx.x + 1; c <= c_last; ++c) p.flags[c] = 0;
                tc::fence_before_sync();
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&acc_empty[b]);
#ifdef VKF_QGEMM_TIMING
            if (q == 2 && lane == 0) atomicAdd(&g_qt[blockIdx.x][6], (unsigned long long)(clock64() - te0));
#endif
            if (!ok) break;
        }
        if (tid == 0) tc::bulk_wait_all();  // Y tensor stores performed before exit
    }
    tc::fence_before_sync();
    __syncthreads();
#ifdef VKF_QGEMM_TIMING
    if (threadIdx.x == 0) atomicAdd(&g_qt[blockIdx.x][7], (unsigned long long)(clock64() - t_start));
#endif
    if (warp == 1) {
        tc::fence_after_sync();
        tc::tmem_free(tmem0, TCOLS);
    }
}

#ifndef VKF_QGEMM_ATM
#define VKF_QGEMM_ATM 1
#endif
constexpr bool ATM_DEFAULT = VKF_QGEMM_ATM != 0;

template <int QT, int BX, int NB, bool ATM = ATM_DEFAULT>
struct Cfg {
    static constexpr int RB = Packed<QT>::RB;
    static constexpr int RAW_BYTES = (BW * RB + 127) / 128 * 128;
    static constexpr int STAGE = (ATM ? 0 : A_BYTES) + NB * BX * 128;
    static constexpr int FIXED = 1024 + 256 + 2 * EPI_BUF;
#ifndef VKF_QGEMM_NSMAX
#define VKF_QGEMM_NSMAX 4
#endif
#ifndef VKF_QGEMM_RSMIN
#define VKF_QGEMM_RSMIN 2
#endif
    // Deepest A/B ring (<= 4) that still leaves RSMIN packed stages (a
    // packed stage feeds four K-blocks; three instead of two measured no
    // different), then as many packed stages (<= 6) as fit.
    // Row-copy formats (Q6_K) keep three packed stages: their per-row
    // granule fetches have a longer latency per stage than one tensor copy.
    static constexpr int RSMIN = row_copies<QT>() ? 3 : VKF_QGEMM_RSMIN;
    static constexpr int NSF = (SMEM_CAP - FIXED - RSMIN * RAW_BYTES) / STAGE;
    static constexpr int NS = NSF >= VKF_QGEMM_NSMAX ? VKF_QGEMM_NSMAX : NSF;
    static constexpr int RS0 = (SMEM_CAP - FIXED - NS * STAGE) / RAW_BYTES;
    static constexpr int RS = RS0 > 6 ? 6 : RS0;
    static constexpr size_t SMEM = (size_t)NS * STAGE + (size_t)RS * RAW_BYTES + FIXED;
    // TMEM: accumulator columns plus, with ATM, 32 columns per stage
    static constexpr bool FITS = NS >= 2 && RS >= 2 && (!ATM || (NB * BX + NS * 32 <= 512 && CV == 8));
};

// Columns per tile (NB x BX) for M activation rows; mirrors launch_q.  The
// converted weight tile lives in TMEM (tiles of up to 256 activation rows;
// more rows take several tiles, each decoding the weights again, which the
// half2 conversion makes cheap: Q4_K 5120 x 13824, M = 512, 70 us against 83
// us for the shared-memory form with one 512-column tile).  The 512-column
// shared-memory form is kept for builds with VKF_QGEMM_ATM=0 where its ring
// fits.
template <int QT>
static int tile_cols(int M) {
    if constexpr (Cfg<QT, 256, 2, false>::FITS) {
        if (M > 256) return 512;
    }
    return M > 128 ? 256 : M > 64 ? 128 : M > 32 ? 64 : 32;
}

static int grid_for(int units) {
    DeviceState *ds = device_state();
    return std::max(1, std::min(units, ds ? ds->sm_count : 148));
}

template <int QT, int BX, int NB, bool ATM>
static int launch(const void *W, const void *X, int64_t ldx, void *Y, int y_f16, int64_t ldy, int M, int N, int K,
                  float *ws, int prefetch, cudaStream_t stream) {
    using C = Cfg<QT, BX, NB, ATM>;
    static_assert(C::FITS, "ring does not fit shared memory");
    constexpr int NC = BX * NB;
    const int64_t row_bytes = (int64_t)K / RV * (row_copies<QT>() ? Q6_ROW : C::RB);
    CUtensorMap tx, tw;
    memset(&tw, 0, sizeof(tw));
    if (!make_kmajor_map(&tx, X, 2, M, K, ldx, BX) ||
        (!row_copies<QT>() && !make_byte_matrix_map(&tw, W, N, row_bytes, C::RB, BW)))
        return VKF_ERR_UNSUPPORTED;
    auto kern = qgemm_kernel<QT, BX, NB, C::NS, C::RS, ATM>;
    static bool attr[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 64 && !attr[dev]) {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM) != cudaSuccess)
            return VKF_ERR_CUDA;
        attr[dev] = true;
    }
    DeviceState *ds = device_state();
    if (!ds) return VKF_ERR_NO_DEVICE;
    const int tiles = ((M + NC - 1) / NC) * ((N + BW - 1) / BW);
    const int units = tiles * (K / RV);
    const int grid = grid_for(units);
    int *flags = stream_counters(stream, (size_t)grid);
    if (!flags) return VKF_ERR_NOMEM;
    // Y rows 16-byte aligned: tensor stores of 32 rows (one TMEM chunk) x 128 columns
    CUtensorMap ty;
    memset(&ty, 0, sizeof(ty));
    const int esize = y_f16 ? 2 : 4;
    const int y_tma = make_rowmajor_map(&ty, Y, esize, M, N, ldy, BW, 32) ? 1 : 0;
    Params p{M, N, K, Y, ldy, y_f16, y_tma, prefetch, units, ws, flags, ds->d_error, (const uint8_t *)W, row_bytes};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(NT);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = stream;
    cudaLaunchAttribute la[1];
    la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    la[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = la;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, kern, tx, tw, ty, p);
    return check_launch();
}

// Activation columns per tile: all of M up to 512 (one weight-tile decode per
// 512 activation rows), in one or two MMAs of up to 256 columns; 256 for
// Q8_0, whose 34 KB packed stages leave no room for a 512-column ring.
template <int QT>
static int launch_q(const void *W, const void *X, int64_t ldx, void *Y, int y_f16, int64_t ldy, int M, int N, int K,
                    float *ws, int prefetch, cudaStream_t stream) {
    switch (tile_cols<QT>(M)) {
    case 512:
        if constexpr (Cfg<QT, 256, 2, false>::FITS)
            return launch<QT, 256, 2, false>(W, X, ldx, Y, y_f16, ldy, M, N, K, ws, prefetch, stream);
        return VKF_ERR_UNSUPPORTED;
    case 256: return launch<QT, 256, 1, ATM_DEFAULT>(W, X, ldx, Y, y_f16, ldy, M, N, K, ws, prefetch, stream);
    case 128: return launch<QT, 128, 1, ATM_DEFAULT>(W, X, ldx, Y, y_f16, ldy, M, N, K, ws, prefetch, stream);
    case 64: return launch<QT, 64, 1, ATM_DEFAULT>(W, X, ldx, Y, y_f16, ldy, M, N, K, ws, prefetch, stream);
    default: return launch<QT, 32, 1, ATM_DEFAULT>(W, X, ldx, Y, y_f16, ldy, M, N, K, ws, prefetch, stream);
    }
}

template <int QT>
static size_t ws_bytes_q(int M, int N, int K) {
    const int nc = tile_cols<QT>(M);
    const int64_t units = (int64_t)((M + nc - 1) / nc) * ((N + BW - 1) / BW) * (K / RV);
    return (size_t)grid_for((int)std::min<int64_t>(units, INT32_MAX)) * nc * BW * sizeof(float);
}

}  // namespace qgemm

// Fused-dequant prefill GEMM; VKF_ERR_UNSUPPORTED when the format or the
// buffer geometry is not one it serves (the caller then widens W first):
// Q4_0, Q8_0, Q4_K, Q5_K, Q6_K with K a multiple of 256, W 16-byte aligned; X fp16
// rows 16-byte aligned.
bool qgemm_supported(int wtype, const void *W, int K) {
    return (wtype == VKF_DEQUANT_Q4_0 || wtype == VKF_DEQUANT_Q8_0 || wtype == VKF_DEQUANT_Q4_K ||
            wtype == VKF_DEQUANT_Q5_K || wtype == VKF_DEQUANT_Q6_K) &&
           K % qgemm::RV == 0 && ((uintptr_t)W & 15) == 0;
}

// Scratch the launch needs for the partials of split tiles (bytes).
size_t qgemm_ws_bytes(int wtype, int M, int N, int K) {
    switch (wtype) {
    case VKF_DEQUANT_Q4_0: return qgemm::ws_bytes_q<VKF_DEQUANT_Q4_0>(M, N, K);
    case VKF_DEQUANT_Q8_0: return qgemm::ws_bytes_q<VKF_DEQUANT_Q8_0>(M, N, K);
    case VKF_DEQUANT_Q4_K: return qgemm::ws_bytes_q<VKF_DEQUANT_Q4_K>(M, N, K);
    case VKF_DEQUANT_Q5_K: return qgemm::ws_bytes_q<VKF_DEQUANT_Q5_K>(M, N, K);
    case VKF_DEQUANT_Q6_K: return qgemm::ws_bytes_q<VKF_DEQUANT_Q6_K>(M, N, K);
    default: return 0;
    }
}

// ws: at least qgemm_ws_bytes(...) of device scratch, 16-byte aligned.
// prefetch: W is written by no kernel (static model weights), so its bytes
// may stream while the previous kernel on the stream finishes.
int qgemm_launch(int wtype, const void *W, const void *X, int64_t ldx, void *Y, int y_f16, int64_t ldy, int M, int N,
                 int K, float *ws, int prefetch, cudaStream_t stream) {
    if (!qgemm_supported(wtype, W, K) || ((uintptr_t)X & 15) || (ldx * 2) % 16) return VKF_ERR_UNSUPPORTED;
    if ((int64_t)((M + 511) / 512) * ((N + 127) / 128) * (K / qgemm::RV) > INT32_MAX / 2) return VKF_ERR_UNSUPPORTED;
    switch (wtype) {
    case VKF_DEQUANT_Q4_0: return qgemm::launch_q<VKF_DEQUANT_Q4_0>(W, X, ldx, Y, y_f16, ldy, M, N, K, ws, prefetch, stream);
    case VKF_DEQUANT_Q8_0: return qgemm::launch_q<VKF_DEQUANT_Q8_0>(W, X, ldx, Y, y_f16, ldy, M, N, K, ws, prefetch, stream);
    case VKF_DEQUANT_Q4_K: return qgemm::launch_q<VKF_DEQUANT_Q4_K>(W, X, ldx, Y, y_f16, ldy, M, N, K, ws, prefetch, stream);
    case VKF_DEQUANT_Q5_K: return qgemm::launch_q<VKF_DEQUANT_Q5_K>(W, X, ldx, Y, y_f16, ldy, M, N, K, ws, prefetch, stream);
    case VKF_DEQUANT_Q6_K: return qgemm::launch_q<VKF_DEQUANT_Q6_K>(W, X, ldx, Y, y_f16, ldy, M, N, K, ws, prefetch, stream);
    default: return VKF_ERR_UNSUPPORTED;
    }
}

}  // namespace vkf

#ifdef VKF_QGEMM_TIMING
extern "C" int vkf_qgemm_timing(void *host, int reset) {
    if (reset) {
        static unsigned long long z[512][8];
        return (int)cudaMemcpyToSymbol(vkf::qgemm::g_qt, z, sizeof(z));
    }
    return (int)cudaMemcpyFromSymbol(host, vkf::qgemm::g_qt, sizeof(vkf::qgemm::g_qt));
}
#endif
