// gemv_q.cuh — per-format decode of one 256-value unit of a 16-row group into
// m16n8k16 tensor-core fragments, for the decode GEMV (M <= 8).
//
// A = 16 weight rows (thread (g, t) = (lane >> 2, lane & 3) holds rows g and
// g + 8), B = the M <= 8 activation columns, fp32 accumulators.  Every MMA's
// 16 k-slots may hold any 16 values of the unit as long as the activation
// fragment holds the matching values; two assignments are used:
//
//   plain   (Q4_0, Q8_0, Q6_K): the 16 slots cover 16 consecutive values;
//           thread t owns values 4t..4t+3, one 32-bit word of weight bytes.
//           Slots (2t, 2t+1) hold values (4t, 4t+2) and (2t+8, 2t+9) hold
//           (4t+1, 4t+3): the half2 pairs one LOP3 extracts from bytes (0,2)
//           and (1,3) of the word.  Activations are stored (x0, x2, x1, x3)
//           per group of four, so a fragment is one 64-bit load.
//   owned   (Q4_K, Q5_K): thread t owns the 32 quant bytes 32t..32t+31 of
//           the super-block, i.e. sub-blocks 2t (low nibbles) and 2t+1 (high
//           nibbles) of dequant_q4_k.glsl:41-57, read as two 16-byte loads;
//           it needs only its own two 6-bit scales and mins.  The activation
//           groups of four are stored with a 16-byte-granule XOR swizzle so
//           that the four threads' 16-byte fragment loads hit distinct banks.
//
// Exactness.  The A operand is always an integer that fp16 represents
// exactly: q-8 (Q4_0), q (Q8_0), sc*q (Q4_K, <= 945; Q5_K, <= 1953), q-32
// (Q6_K), m (K-quant mins).  They are produced from "1024 + code" fp16 bit
// patterns with one fp16 FMA whose exact result is that integer, so its
// single rounding is exact.  Products with fp16 activations are exact in the
// fp32 accumulator; the per-block fp32 scales (d, d*sc, dmin) are applied to
// the fp32 partial sums.  The only roundings are fp32 accumulation (and the
// hi + lo fp16 split of the K-quant sub-block sums, exact to ~2^-22).
#pragma once

#include "device_common.cuh"

namespace vkf {
namespace gemv {

// QK values per block, BB bytes per block.  A work unit is 256 values of a
// row: one super-block, or eight 32-value blocks.
template <int QT> struct Fmt;
template <> struct Fmt<VKF_DEQUANT_Q4_0> { static constexpr int QK = 32, BB = 18; };
template <> struct Fmt<VKF_DEQUANT_Q8_0> { static constexpr int QK = 32, BB = 34; };
template <> struct Fmt<VKF_DEQUANT_Q4_K> { static constexpr int QK = 256, BB = 144; };
template <> struct Fmt<VKF_DEQUANT_Q5_K> { static constexpr int QK = 256, BB = 176; };
template <> struct Fmt<VKF_DEQUANT_Q6_K> { static constexpr int QK = 256, BB = 210; };

// fp16 constants (bit patterns)
constexpr uint32_t H2_MAGIC = 0x64006400u;  // (1024, 1024)
constexpr uint32_t H2_1024 = 0x64006400u;
constexpr uint32_t H2_1032 = 0x64086408u;   // 1024 + 8
constexpr uint32_t H2_1056 = 0x64206420u;   // 1024 + 32
constexpr uint32_t H2_1152 = 0x64806480u;   // 1024 + 128
constexpr uint32_t H2_SIXTEENTH = 0x2C002C00u;  // 1/16
constexpr uint32_t H2_M72 = 0xD480D480u;    // -72
constexpr uint32_t H2_M96 = 0xD600D600u;    // -96
constexpr uint32_t H2_M1024 = 0xE400E400u;  // -1024
constexpr uint32_t H2_M64 = 0xD400D400u;    // -64

__device__ __forceinline__ uint32_t lop3_and_xor(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(r) : "r"(a), "r"(b), "r"(c));  // (a & b) ^ c
    return r;
}

// B fragment of the 16 k-values starting at k0 of one activation column.
// The column is stored permuted within each group of four values as
// (x0, x2, x1, x3), so thread t's fragment (b0 = (x[4t], x[4t+2]),
// b1 = (x[4t+1], x[4t+3])) is one 64-bit load.
__device__ __forceinline__ void xfrag(const uint8_t *xcol, int k0, int t, uint32_t &b0, uint32_t &b1) {
    uint2 v = *reinterpret_cast<const uint2 *>(xcol + (k0 + 4 * t) * 2);
    b0 = v.x;
    b1 = v.y;
}

__device__ __forceinline__ uint32_t ld32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }

__device__ __forceinline__ float hbits(const uint8_t *p) { return half_bits_to_float(ld_u16(p)); }

__device__ __forceinline__ void zero4(float (&p)[4]) { p[0] = p[1] = p[2] = p[3] = 0.f; }

// Accumulates one work unit for rows (g, g+8) of a 16-row group.
//   ra, rb: smem start of the unit's blocks for rows g and g+8 (a 256-value
//           unit: one super-block, or eight 32-value blocks)
//   xc:     permuted activations of column g at the unit's first value
//   xs:     (Q4_K, Q5_K) sub-block sums of column g for this super-block
//   nblk:   32-value blocks present (tail unit of Q4_0 / Q8_0)
template <int QT> struct Step;

template <> struct Step<VKF_DEQUANT_Q4_0> {
    static constexpr bool OWNED = false;
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xc,
                                               const uint8_t *, int t, int nblk, float (&acc)[4]) {
#pragma unroll 8
        for (int c = 0; c < 8; ++c) {
            if (c >= nblk) break;
            const uint8_t *ba = ra + c * 18, *bb = rb + c * 18;
            float da = hbits(ba), db = hbits(bb);
            uint32_t wa = ld_u32_a2(ba + 2 + 4 * t), wb = ld_u32_a2(bb + 2 + 4 * t);
            uint32_t wa8 = wa >> 8, wb8 = wb >> 8;
            uint32_t alo[4], ahi[4];
            alo[0] = hsub2_u(lop3_and_or(wa, 0x000F000Fu, H2_MAGIC), H2_1032);
            alo[1] = hsub2_u(lop3_and_or(wb, 0x000F000Fu, H2_MAGIC), H2_1032);
            alo[2] = hsub2_u(lop3_and_or(wa8, 0x000F000Fu, H2_MAGIC), H2_1032);
            alo[3] = hsub2_u(lop3_and_or(wb8, 0x000F000Fu, H2_MAGIC), H2_1032);
            ahi[0] = hfma2_u(lop3_and_or(wa, 0x00F000F0u, H2_MAGIC), H2_SIXTEENTH, H2_M72);
            ahi[1] = hfma2_u(lop3_and_or(wb, 0x00F000F0u, H2_MAGIC), H2_SIXTEENTH, H2_M72);
            ahi[2] = hfma2_u(lop3_and_or(wa8, 0x00F000F0u, H2_MAGIC), H2_SIXTEENTH, H2_M72);
            ahi[3] = hfma2_u(lop3_and_or(wb8, 0x00F000F0u, H2_MAGIC), H2_SIXTEENTH, H2_M72);
            uint32_t b0, b1, b2, b3;
            xfrag(xc, c * 32, t, b0, b1);
            xfrag(xc, c * 32 + 16, t, b2, b3);
            float p[4];
            zero4(p);
            mma_16816(p, alo, b0, b1);
            mma_16816(p, ahi, b2, b3);
            acc[0] = fmaf(da, p[0], acc[0]);
            acc[1] = fmaf(da, p[1], acc[1]);
            acc[2] = fmaf(db, p[2], acc[2]);
            acc[3] = fmaf(db, p[3], acc[3]);
        }
    }
};

template <> struct Step<VKF_DEQUANT_Q8_0> {
    static constexpr bool OWNED = false;
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xc,
                                               const uint8_t *, int t, int nblk, float (&acc)[4]) {
#pragma unroll 8
        for (int c = 0; c < 8; ++c) {
            if (c >= nblk) break;
            const uint8_t *ba = ra + c * 34, *bb = rb + c * 34;
            float da = hbits(ba), db = hbits(bb);
            float p[4];
            zero4(p);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t wa = ld_u32_a2(ba + 2 + 16 * h + 4 * t), wb = ld_u32_a2(bb + 2 + 16 * h + 4 * t);
                uint32_t a[4];
                a[0] = hsub2_u(lop3_and_xor(wa, 0x00FF00FFu, 0x64806480u), H2_1152);
                a[1] = hsub2_u(lop3_and_xor(wb, 0x00FF00FFu, 0x64806480u), H2_1152);
                a[2] = hsub2_u(lop3_and_xor(wa >> 8, 0x00FF00FFu, 0x64806480u), H2_1152);
                a[3] = hsub2_u(lop3_and_xor(wb >> 8, 0x00FF00FFu, 0x64806480u), H2_1152);
                uint32_t b0, b1;
                xfrag(xc, c * 32 + 16 * h, t, b0, b1);
                mma_16816(p, a, b0, b1);
            }
            acc[0] = fmaf(da, p[0], acc[0]);
            acc[1] = fmaf(da, p[1], acc[1]);
            acc[2] = fmaf(db, p[2], acc[2]);
            acc[3] = fmaf(db, p[3], acc[3]);
        }
    }
};

__device__ __forceinline__ uint4 lds128(const uint8_t *p) { return *reinterpret_cast<const uint4 *>(p); }

// Byte offset, within one column's 512-byte super-block block of the owned
// activation layout, of the fragment group holding value v (0..255): groups
// of four values (x0, x2, x1, x3), two groups per 16-byte granule, granule
// j = v / 8 stored at j ^ ((j / 8) & 3).
__host__ __device__ __forceinline__ int owned_group_offset(int v) {
    const int q = v >> 2, j = q >> 1;
    return ((j ^ ((j >> 3) & 3)) << 4) + ((q & 1) << 3);
}

// Per-thread constants of one K-quant row for the thread's sub-blocks 2t and
// 2t+1 (get_scale_min_k4, dequant_q4_k.glsl:16-24), from the 16-byte header
// [d, dmin, scales[12]]:
//   sl, cl:  (sc_2t, sc_2t) and -1024 * sc_2t   (low nibbles: (1024+q)*sc - 1024*sc)
//   sh, ch:  sc_2t+1 / 16 and -64 * sc_2t+1     (high nibbles: (1024+16q)*sc/16 - 64*sc)
//   am:      (m_2t, m_2t+1)                     (min-term MMA operand)
struct KRow {
    uint32_t sl, cl, sh, ch, am;
    float d, dm;
    __device__ __forceinline__ KRow(const uint4 h, int t) {
        const uint32_t scA = h.y & 0x3F3F3F3Fu, mA = h.z & 0x3F3F3F3Fu;
        const uint32_t scB = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
        const uint32_t mB = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
        const uint32_t scw = t < 2 ? scA : scB, mw = t < 2 ? mA : mB;
        const uint32_t b = (uint32_t)(t & 1) * 2;  // byte of sub-block 2t in its word
        const uint32_t sel = b * 0x0101u + 0x4040u;  // [byte b, 0x64, byte b, 0x64]
        const uint32_t lo = hsub2_u(prmt(scw, 0x64646464u, sel), H2_1024);
        const uint32_t hi = hsub2_u(prmt(scw, 0x64646464u, sel + 0x0101u), H2_1024);
        sl = lo;
        cl = hmul2_u(lo, H2_M1024);
        sh = hmul2_u(hi, H2_SIXTEENTH);
        ch = hmul2_u(hi, H2_M64);
        am = hsub2_u(prmt(mw, 0x64646464u, b + 0x4040u + (b + 1) * 0x100u), H2_1024);
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));
        d = f.x;
        dm = f.y;
    }
};

// Q4_K and Q5_K (dequant_q4_k.glsl / dequant_q5_k.glsl): value = (d*sc)*q - dmin*m,
// owned mapping.  MMA pair i (i = 0..7) takes quant word i of the thread's
// chunk: its low nibbles (bytes 0,2 | 1,3) form the sub-block-2t MMA, its high
// nibbles the sub-block-2t+1 MMA; A = sc*q (exact).  Q5_K ORs the fifth bit
// qh[l] bit 2t / 2t+1 (dequant_q5_k.glsl:52-69) into the codes first.  The min
// term sum_j m_j * X_j (X_j the activation sum over sub-block j) is one MMA:
// thread t's k-slots hold m_2t, m_2t+1 against X_2t, X_2t+1 split into fp16
// hi (slots 2t, 2t+1) + lo (slots 2t+8, 2t+9), precomputed once per CTA.
template <bool Q5> struct StepK {
    static constexpr bool OWNED = true;
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xc,
                                               const uint8_t *xs, int t, int, float (&acc)[4]) {
        constexpr int QS = Q5 ? 48 : 16;
        const KRow ka(lds128(ra), t), kb(lds128(rb), t);
        uint32_t wa[8], wb[8];
        {
            const uint4 a0 = lds128(ra + QS + 32 * t), a1 = lds128(ra + QS + 16 + 32 * t);
            const uint4 b0 = lds128(rb + QS + 32 * t), b1 = lds128(rb + QS + 16 + 32 * t);
            wa[0] = a0.x; wa[1] = a0.y; wa[2] = a0.z; wa[3] = a0.w; wa[4] = a1.x; wa[5] = a1.y; wa[6] = a1.z; wa[7] = a1.w;
            wb[0] = b0.x; wb[1] = b0.y; wb[2] = b0.z; wb[3] = b0.w; wb[4] = b1.x; wb[5] = b1.y; wb[6] = b1.z; wb[7] = b1.w;
        }
        uint32_t ha[8], hb[8];
        if constexpr (Q5) {
            const uint4 a0 = lds128(ra + 16), a1 = lds128(ra + 32), b0 = lds128(rb + 16), b1 = lds128(rb + 32);
            ha[0] = a0.x; ha[1] = a0.y; ha[2] = a0.z; ha[3] = a0.w; ha[4] = a1.x; ha[5] = a1.y; ha[6] = a1.z; ha[7] = a1.w;
            hb[0] = b0.x; hb[1] = b0.y; hb[2] = b0.z; hb[3] = b0.w; hb[4] = b1.x; hb[5] = b1.y; hb[6] = b1.z; hb[7] = b1.w;
        }
        float p0[4] = {0.f, 0.f, 0.f, 0.f}, p1[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            const uint4 xl = lds128(xc + owned_group_offset(64 * t + 4 * i));
            const uint4 xh = lds128(xc + owned_group_offset(64 * t + 32 + 4 * i));
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const uint32_t a = wa[i + e], b = wb[i + e], a8 = a >> 8, b8 = b >> 8;
                uint32_t la0 = lop3_and_or(a, 0x000F000Fu, H2_MAGIC), la1 = lop3_and_or(a8, 0x000F000Fu, H2_MAGIC);
                uint32_t lb0 = lop3_and_or(b, 0x000F000Fu, H2_MAGIC), lb1 = lop3_and_or(b8, 0x000F000Fu, H2_MAGIC);
                uint32_t hA0 = lop3_and_or(a, 0x00F000F0u, H2_MAGIC), hA1 = lop3_and_or(a8, 0x00F000F0u, H2_MAGIC);
                uint32_t hB0 = lop3_and_or(b, 0x00F000F0u, H2_MAGIC), hB1 = lop3_and_or(b8, 0x00F000F0u, H2_MAGIC);
                if constexpr (Q5) {
                    // qh byte l bit 2t -> code bit 4 (low), bit 2t+1 -> code bit 8 of the 16q form (high)
                    const uint32_t qa = ha[i + e], qb = hb[i + e];
                    const int s = 2 * t;
                    la0 = lop3_and_or(s <= 4 ? qa << (4 - s) : qa >> (s - 4), 0x00100010u, la0);
                    lb0 = lop3_and_or(s <= 4 ? qb << (4 - s) : qb >> (s - 4), 0x00100010u, lb0);
                    la1 = lop3_and_or(qa >> (4 + s), 0x00100010u, la1);
                    lb1 = lop3_and_or(qb >> (4 + s), 0x00100010u, lb1);
                    hA0 = lop3_and_or(qa << (7 - s), 0x01000100u, hA0);
                    hB0 = lop3_and_or(qb << (7 - s), 0x01000100u, hB0);
                    hA1 = lop3_and_or(qa >> (s + 1), 0x01000100u, hA1);
                    hB1 = lop3_and_or(qb >> (s + 1), 0x01000100u, hB1);
                }
                const uint32_t AL[4] = {hfma2_u(la0, ka.sl, ka.cl), hfma2_u(lb0, kb.sl, kb.cl), hfma2_u(la1, ka.sl, ka.cl),
                                        hfma2_u(lb1, kb.sl, kb.cl)};
                const uint32_t AH[4] = {hfma2_u(hA0, ka.sh, ka.ch), hfma2_u(hB0, kb.sh, kb.ch), hfma2_u(hA1, ka.sh, ka.ch),
                                        hfma2_u(hB1, kb.sh, kb.ch)};
                if (e == 0) {
                    mma_16816(p0, AL, xl.x, xl.y);
                    mma_16816(p0, AH, xh.x, xh.y);
                } else {
                    mma_16816(p1, AL, xl.z, xl.w);
                    mma_16816(p1, AH, xh.z, xh.w);
                }
            }
        }
        const uint2 sv = *reinterpret_cast<const uint2 *>(xs + 8 * t);
        float pm[4] = {0.f, 0.f, 0.f, 0.f};
        const uint32_t am[4] = {ka.am, kb.am, ka.am, kb.am};
        mma_16816(pm, am, sv.x, sv.y);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float d = i < 2 ? ka.d : kb.d, dm = i < 2 ? ka.dm : kb.dm;
            acc[i] = fmaf(-dm, pm[i], fmaf(d, p0[i] + p1[i], acc[i]));
        }
    }
};

// M = 1 column forms.  With one activation column, seven of the MMA's eight
// B columns would be idle; instead they carry scale groups: a lane supplies
// its activation fragment only in the column assigned to its own values and
// zero registers elsewhere (a predicated-off load costs no shared-memory
// bandwidth), so each column of the accumulator sums one scale group, and the
// scales, mins and offsets are applied once per group in fp32 instead of to
// every weight.  The codes enter the MMA as raw integers.
// Position (t, e) of sub-block j in the per-super-block sums [t][e] (floats).
__host__ __device__ __forceinline__ int m1_sum_slot(int j) {
    const int e = (j >> 1) & 1, b = j - 2 * e;  // b in {0, 1, 4, 5}
    const int t = 2 * (b & 1) + (b >> 2);
    return 2 * t + e;
}

template <> struct Step<VKF_DEQUANT_Q4_K> : StepK<false> {};
template <> struct Step<VKF_DEQUANT_Q5_K> : StepK<true> {};

// Q6_K (dequant_q6_k.glsl:28-58): value = d * sc16 * (q6 - 32), one int8 scale
// per 16 values; A operand = q6 - 32 (exact), each MMA's partial scaled by
// d*sc in fp32.  PART = ip selects the 128-value half.
template <int IP> struct StepQ6 {
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xc, int t,
                                               float (&acc)[4]) {
        const float da = hbits(ra + 208), db = hbits(rb + 208);
        const int8_t *sa = reinterpret_cast<const int8_t *>(ra + 192);
        const int8_t *sb = reinterpret_cast<const int8_t *>(rb + 192);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            const uint32_t qha = ld_u32_a2(ra + 128 + 32 * IP + 16 * h + 4 * t);
            const uint32_t qhb = ld_u32_a2(rb + 128 + 32 * IP + 16 * h + 4 * t);
#pragma unroll
            for (int half = 0; half < 2; ++half) {  // ql bytes at +0 / +32 (s & 1)
                const uint32_t qla = ld_u32_a2(ra + 64 * IP + 32 * half + 16 * h + 4 * t);
                const uint32_t qlb = ld_u32_a2(rb + 64 * IP + 32 * half + 16 * h + 4 * t);
                const uint32_t qla8 = qla >> 8, qlb8 = qlb >> 8;
#pragma unroll
                for (int hiN = 0; hiN < 2; ++hiN) {
                    const int s = half + 2 * hiN;
                    uint32_t a[4];
                    if (hiN == 0) {
                        a[0] = hsub2_u(lop3_and_or(qha << (4 - 2 * s), 0x00300030u, lop3_and_or(qla, 0x000F000Fu, H2_MAGIC)), H2_1056);
                        a[1] = hsub2_u(lop3_and_or(qhb << (4 - 2 * s), 0x00300030u, lop3_and_or(qlb, 0x000F000Fu, H2_MAGIC)), H2_1056);
                        a[2] = hsub2_u(lop3_and_or(qha >> (4 + 2 * s), 0x00300030u, lop3_and_or(qla8, 0x000F000Fu, H2_MAGIC)), H2_1056);
                        a[3] = hsub2_u(lop3_and_or(qhb >> (4 + 2 * s), 0x00300030u, lop3_and_or(qlb8, 0x000F000Fu, H2_MAGIC)), H2_1056);
                    } else {
                        a[0] = hfma2_u(lop3_and_or(qha << (8 - 2 * s), 0x03000300u, lop3_and_or(qla, 0x00F000F0u, H2_MAGIC)), H2_SIXTEENTH, H2_M96);
                        a[1] = hfma2_u(lop3_and_or(qhb << (8 - 2 * s), 0x03000300u, lop3_and_or(qlb, 0x00F000F0u, H2_MAGIC)), H2_SIXTEENTH, H2_M96);
                        a[2] = hfma2_u(lop3_and_or(qha >> (2 * s), 0x03000300u, lop3_and_or(qla8, 0x00F000F0u, H2_MAGIC)), H2_SIXTEENTH, H2_M96);
                        a[3] = hfma2_u(lop3_and_or(qhb >> (2 * s), 0x03000300u, lop3_and_or(qlb8, 0x00F000F0u, H2_MAGIC)), H2_SIXTEENTH, H2_M96);
                    }
                    uint32_t b0, b1;
                    xfrag(xc, 128 * IP + 32 * s + 16 * h, t, b0, b1);
                    float p[4];
                    zero4(p);
                    mma_16816(p, a, b0, b1);
                    const int is = 8 * IP + 2 * s + h;
                    const float fa = da * (float)sa[is], fb = db * (float)sb[is];
                    acc[0] = fmaf(fa, p[0], acc[0]);
                    acc[1] = fmaf(fa, p[1], acc[1]);
                    acc[2] = fmaf(fb, p[2], acc[2]);
                    acc[3] = fmaf(fb, p[3], acc[3]);
                }
            }
        }
    }
};

// Q4_K and Q5_K, M = 1 column form (owned mapping: thread t holds the quant
// bytes 32t .. 32t + 31, sub-blocks 2t (low nibbles) and 2t + 1 (high)).
// The activations are 16-bit fixed point per 32-value sub-block,
// x = s_j * (256 * xh + xl) with xh, xl int8, and the codes enter
// `mma.sync.m16n8k32.s8` as raw int8 (one LOP3 makes four codes:
// q & 0x0F0F0F0F, (q >> 4) & 0x0F0F0F0F).  Lane (g', t) feeds its
// activations only into column t (low nibbles, sub-block 2t) or 4 + t (high
// nibbles, 2t + 1); thread (g, t) then owns columns 2t, 2t + 1 = sub-blocks
// j1 = 4 (t & 1) + t / 2 and j1 + 2.  Per sub-block and row the int32 sums
// are exact (|D| < 2^24 for Q4_K); the thread applies
//     acc += d*sc_j*s_j * (256 Dh + Dl) - dmin*m_j * X_j.
// Activation layout per super-block: xh[256] | xl[256] (int8, value order),
// then per sub-block s_j (fp32) in [t][2] order, X_j (fp32) in [t][2] order.
__device__ __forceinline__ void mma_16832_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

template <bool Q5> struct StepK1i {
    static constexpr bool OWNED = true;
    __device__ __forceinline__ static float byte_f(uint32_t w, uint32_t b) {
        return __uint_as_float(prmt(w, 0x4B000000u, b | 0x7540u)) - 8388608.0f;
    }
    // xu: the unit's 512 activation bytes; sx: the unit's [s (8 floats) | X (8 floats)].
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xu, bool lo_on,
                                               bool hi_on, const float *sx, int t, float (&acc)[4]) {
        constexpr int QS = Q5 ? 48 : 16;
        const uint4 hA = lds128(ra), hB = lds128(rb);
        uint32_t wa[8], wb[8];
        {
            const uint4 a0 = lds128(ra + QS + 32 * t), a1 = lds128(ra + QS + 16 + 32 * t);
            const uint4 b0 = lds128(rb + QS + 32 * t), b1 = lds128(rb + QS + 16 + 32 * t);
            wa[0] = a0.x; wa[1] = a0.y; wa[2] = a0.z; wa[3] = a0.w; wa[4] = a1.x; wa[5] = a1.y; wa[6] = a1.z; wa[7] = a1.w;
            wb[0] = b0.x; wb[1] = b0.y; wb[2] = b0.z; wb[3] = b0.w; wb[4] = b1.x; wb[5] = b1.y; wb[6] = b1.z; wb[7] = b1.w;
        }
        uint32_t ha[8], hb[8];
        if constexpr (Q5) {
            const uint4 a0 = lds128(ra + 16), a1 = lds128(ra + 32), b0 = lds128(rb + 16), b1 = lds128(rb + 32);
            ha[0] = a0.x; ha[1] = a0.y; ha[2] = a0.z; ha[3] = a0.w; ha[4] = a1.x; ha[5] = a1.y; ha[6] = a1.z; ha[7] = a1.w;
            hb[0] = b0.x; hb[1] = b0.y; hb[2] = b0.z; hb[3] = b0.w; hb[4] = b1.x; hb[5] = b1.y; hb[6] = b1.z; hb[7] = b1.w;
        }
        int Dh[4] = {0, 0, 0, 0}, Dl[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
            // B: 8 consecutive int8 of the thread's values (64t + 4i .. +7, low; +32, high)
            uint2 lh = make_uint2(0, 0), ll = make_uint2(0, 0), hh = make_uint2(0, 0), hl = make_uint2(0, 0);
            if (lo_on) {
                lh = *reinterpret_cast<const uint2 *>(xu + 64 * t + 4 * i);
                ll = *reinterpret_cast<const uint2 *>(xu + 256 + 64 * t + 4 * i);
            }
            if (hi_on) {
                hh = *reinterpret_cast<const uint2 *>(xu + 64 * t + 32 + 4 * i);
                hl = *reinterpret_cast<const uint2 *>(xu + 256 + 64 * t + 32 + 4 * i);
            }
            uint32_t AL[4] = {wa[i] & 0x0F0F0F0Fu, wb[i] & 0x0F0F0F0Fu, wa[i + 1] & 0x0F0F0F0Fu, wb[i + 1] & 0x0F0F0F0Fu};
            uint32_t AH[4] = {(wa[i] >> 4) & 0x0F0F0F0Fu, (wb[i] >> 4) & 0x0F0F0F0Fu, (wa[i + 1] >> 4) & 0x0F0F0F0Fu,
                              (wb[i + 1] >> 4) & 0x0F0F0F0Fu};
            if constexpr (Q5) {
                // fifth bit: qh[l] bit 2t (low) / 2t + 1 (high) -> code bit 4 of each byte
                const int s = 2 * t;
                AL[0] |= ((ha[i] >> s) & 0x01010101u) << 4;
                AL[1] |= ((hb[i] >> s) & 0x01010101u) << 4;
                AL[2] |= ((ha[i + 1] >> s) & 0x01010101u) << 4;
                AL[3] |= ((hb[i + 1] >> s) & 0x01010101u) << 4;
                AH[0] |= ((ha[i] >> (s + 1)) & 0x01010101u) << 4;
                AH[1] |= ((hb[i] >> (s + 1)) & 0x01010101u) << 4;
                AH[2] |= ((ha[i + 1] >> (s + 1)) & 0x01010101u) << 4;
                AH[3] |= ((hb[i + 1] >> (s + 1)) & 0x01010101u) << 4;
            }
            mma_16832_s8(Dh, AL, lh.x, lh.y);
            mma_16832_s8(Dl, AL, ll.x, ll.y);
            mma_16832_s8(Dh, AH, hh.x, hh.y);
            mma_16832_s8(Dl, AH, hl.x, hl.y);
        }
        const uint32_t b1 = (uint32_t)(t >> 1), b2 = b1 + 2;
        const float2 sj = *reinterpret_cast<const float2 *>(sx + 2 * t);
        const float2 xj = *reinterpret_cast<const float2 *>(sx + 8 + 2 * t);
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const uint4 h = r ? hB : hA;
            uint32_t scw, mw;
            if (t & 1) {
                scw = (h.w & 0x0F0F0F0Fu) | ((h.y >> 2) & 0x30303030u);
                mw = ((h.w >> 4) & 0x0F0F0F0Fu) | ((h.z >> 2) & 0x30303030u);
            } else {
                scw = h.y & 0x3F3F3F3Fu;
                mw = h.z & 0x3F3F3F3Fu;
            }
            const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));
            const float qa = (float)(256 * Dh[2 * r] + Dl[2 * r]), qb = (float)(256 * Dh[2 * r + 1] + Dl[2 * r + 1]);
            float &o0 = acc[2 * r], &o1 = acc[2 * r + 1];
            o0 = fmaf(dd.x * byte_f(scw, b1) * sj.x, qa, fmaf(-dd.y * byte_f(mw, b1), xj.x, o0));
            o1 = fmaf(dd.x * byte_f(scw, b2) * sj.y, qb, fmaf(-dd.y * byte_f(mw, b2), xj.y, o1));
        }
    }
};

// Q6_K, M = 1 column form.  MMA (ip, s) (m16n8k32.s8) covers the 32
// values l = 0..31 of run (ip, s); thread t holds l = 8t .. 8t + 7 (words e = 0,
// 1), all in scale group h = t >> 1, so lanes of column c = 2s + (t >> 1)
// feed activations and, after the four MMAs of half ip, column 2s + h holds
// group 8 ip + 2s + h.  A = the 6-bit code q (0..63) byte-wise: nibble of
// ql[64 ip + 32 (s & 1) + l] (low for s < 2, high for s >= 2) | qh bits 2s, 2s+1
// moved to bits 4, 5 (dequant_q6_k.glsl:34-58).  Activations as for StepK1i
// (x = s_j * (256 xh + xl) per 32-value run j = 4 ip + s); thread (g, t) owns
// groups (ip, t, h) and adds  d * sc * (s_j * (256 Dh + Dl) - 32 * X16).
// Odd super-blocks start 2 mod 4: their words are two aligned words and a
// byte permute (AL4 = 1); rows of 2 mod 4 bytes mix both within a warp and
// take the lane-by-lane form (AL4 = 2): mma.sync must be executed by the
// whole warp, so the form is chosen warp-uniformly.
struct StepQ6i {
    // AL: 0 the address is 4-byte aligned; 1 it is 2 mod 4 (two aligned
    // words and a byte permute); 2 either, lane by lane (a funnel shift by
    // the address: rows of 2 mod 4 bytes, where lanes of one warp differ).
    template <int AL> __device__ __forceinline__ static uint32_t w32(const uint8_t *p) {
        if constexpr (AL == 0) return *reinterpret_cast<const uint32_t *>(p);
        if constexpr (AL == 1) {
            const uint32_t lo = *reinterpret_cast<const uint32_t *>(p - 2), hi = *reinterpret_cast<const uint32_t *>(p + 2);
            return prmt(lo, hi, 0x5432);
        }
        const uintptr_t a = (uintptr_t)p;
        const uint32_t *q = reinterpret_cast<const uint32_t *>(a & ~(uintptr_t)3);
        return __funnelshift_r(q[0], q[1], (uint32_t)(a & 3) * 8);
    }
    template <int S> __device__ __forceinline__ static uint32_t code(uint32_t q0, uint32_t q1, uint32_t qh) {
        const uint32_t ql = (S & 1) ? q1 : q0;
        const uint32_t nib = S < 2 ? (ql & 0x0F0F0F0Fu) : ((ql >> 4) & 0x0F0F0F0Fu);
        const uint32_t hs = S == 0 ? qh << 4 : S == 1 ? qh << 2 : S == 2 ? qh : qh >> 2;
        return lop3_and_or(hs, 0x30303030u, nib);
    }
    // xu: the unit's xh[256] | xl[256]; sx: s[8] (runs) | X16[16] (groups).
    template <int AL4>
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xu, int g,
                                               const float *sx, int t, float (&acc)[4]) {
        const float da = half_bits_to_float(ld_u16(ra + 208)), db = half_bits_to_float(ld_u16(rb + 208));
#pragma unroll
        for (int ip = 0; ip < 2; ++ip) {
            uint32_t a0[2], a1[2], ah[2], b0[2], b1[2], bh[2];
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int o = 64 * ip + 8 * t + 4 * e, oh = 128 + 32 * ip + 8 * t + 4 * e;
                a0[e] = w32<AL4>(ra + o);
                a1[e] = w32<AL4>(ra + o + 32);
                ah[e] = w32<AL4>(ra + oh);
                b0[e] = w32<AL4>(rb + o);
                b1[e] = w32<AL4>(rb + o + 32);
                bh[e] = w32<AL4>(rb + oh);
            }
            int Dh[4] = {0, 0, 0, 0}, Dl[4] = {0, 0, 0, 0};
#define VKF_Q6I_MMA(S)                                                                                   \
    {                                                                                                    \
        const uint32_t A[4] = {code<S>(a0[0], a1[0], ah[0]), code<S>(b0[0], b1[0], bh[0]),               \
                               code<S>(a0[1], a1[1], ah[1]), code<S>(b0[1], b1[1], bh[1])};               \
        uint2 xh = make_uint2(0, 0), xl = make_uint2(0, 0);                                              \
        if (g == 2 * S + (t >> 1)) {                                                                     \
            xh = *reinterpret_cast<const uint2 *>(xu + 128 * ip + 32 * S + 8 * t);                       \
            xl = *reinterpret_cast<const uint2 *>(xu + 256 + 128 * ip + 32 * S + 8 * t);                 \
        }                                                                                                \
        mma_16832_s8(Dh, A, xh.x, xh.y);                                                                 \
        mma_16832_s8(Dl, A, xl.x, xl.y);                                                                 \
    }
            VKF_Q6I_MMA(0)
            VKF_Q6I_MMA(1)
            VKF_Q6I_MMA(2)
            VKF_Q6I_MMA(3)
#undef VKF_Q6I_MMA
            // Columns 2t, 2t+1 = groups 8 ip + 2t + h of run 4 ip + t.
            const uint32_t sa = ld_u16(ra + 192 + 8 * ip + 2 * t), sb = ld_u16(rb + 192 + 8 * ip + 2 * t);
            const float sj = sx[4 * ip + t];
            const float2 x16 = *reinterpret_cast<const float2 *>(sx + 8 + 8 * ip + 2 * t);
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                const uint32_t sw = r ? sb : sa;
                const float d = r ? db : da;
#pragma unroll
                for (int hh = 0; hh < 2; ++hh) {
                    const float dsc = d * (float)(int8_t)(sw >> (8 * hh));
                    const float q = (float)(256 * Dh[2 * r + hh] + Dl[2 * r + hh]);
                    float &o = acc[2 * r + hh];
                    o = fmaf(dsc * sj, q, fmaf(-32.0f * dsc, hh ? x16.y : x16.x, o));
                }
            }
        }
    }
};

template <> struct Step<VKF_DEQUANT_Q6_K> {
    static constexpr bool OWNED = false;
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xc,
                                               const uint8_t *, int t, int, float (&acc)[4]) {
        StepQ6<0>::run(ra, rb, xc, t, acc);
        StepQ6<1>::run(ra, rb, xc, t, acc);
    }
};

}  // namespace gemv
}  // namespace vkf
