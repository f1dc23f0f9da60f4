// gemv_q.cuh — per-format decode of one work unit of a 16-row group into
// m16n8k16 tensor-core fragments, for the decode GEMV (M <= 8).
//
// Fragment mapping.  The 16 k-slots of each MMA cover 16 consecutive values
// of one 32-value (sub-)block; thread t (= lane & 3) owns the 4 values
// 4t..4t+3, so its weight bytes are one 32-bit word.  Within the MMA, slot
// (2t, 2t+1) holds values (4t, 4t+2) and slot (2t+8, 2t+9) holds (4t+1, 4t+3):
// exactly the half2 pairs a single LOP3 extracts from bytes (0,2) and (1,3)
// of the word.  The activations (B fragment) are stored with the same
// permutation, so the dot product is unchanged.
//
// Exactness.  The A operand is always an integer that fp16 represents
// exactly: q-8 (Q4_0), q (Q8_0), sc*q (Q4_K, <= 945; Q5_K, <= 1953), q-32
// (Q6_K), m (K-quant mins).  They are produced from "1024 + code" fp16 bit
// patterns with one fp16 operation whose exact result is that integer, so the
// single rounding is exact.  Products with fp16 activations are exact in the
// fp32 accumulator; the per-block fp32 scales (d, d*sc, dmin) are applied to
// the fp32 partial sums.  The only roundings are fp32 accumulation (and the
// hi + lo fp16 split of the K-quant sub-block sums, exact to ~2^-22).
#pragma once

#include "device_common.cuh"

namespace vkf {
namespace gemv {

// QK values per block, BB bytes per block, PARTS work units per 256 values
// (1: a warp decodes whole super-blocks / 8-block groups).
template <int QT> struct Fmt;
template <> struct Fmt<VKF_DEQUANT_Q4_0> { static constexpr int QK = 32, BB = 18, PARTS = 1; };
template <> struct Fmt<VKF_DEQUANT_Q8_0> { static constexpr int QK = 32, BB = 34, PARTS = 1; };
template <> struct Fmt<VKF_DEQUANT_Q4_K> { static constexpr int QK = 256, BB = 144, PARTS = 1; };
template <> struct Fmt<VKF_DEQUANT_Q5_K> { static constexpr int QK = 256, BB = 176, PARTS = 1; };
template <> struct Fmt<VKF_DEQUANT_Q6_K> { static constexpr int QK = 256, BB = 210, PARTS = 1; };

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
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xc,
                                               const uint8_t *, int t, int, int nblk, float (&acc)[4]) {
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
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xc,
                                               const uint8_t *, int t, int, int nblk, float (&acc)[4]) {
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

// [code, 0x64, code, 0x64] from byte `idx` of w: half2 (1024+code, 1024+code).
__device__ __forceinline__ uint32_t dup_byte_magic(uint32_t w, int idx) {
    return prmt(w, 0x64646464u, (uint32_t)(idx * 0x101 + 0x4040));
}

// Unpacked 6-bit scales/mins of a K-quant super-block, four per word:
// sc[0..3], sc[4..7], m[0..3], m[4..7] (get_scale_min_k4, dequant_q4_k.glsl:16-24).
struct KScales {
    uint32_t scA, scB, mA, mB;
    __device__ __forceinline__ explicit KScales(const uint8_t *s) {
        uint32_t s0 = ld32(s), s1 = ld32(s + 4), s2 = ld32(s + 8);
        scA = s0 & 0x3F3F3F3Fu;
        mA = s1 & 0x3F3F3F3Fu;
        scB = (s2 & 0x0F0F0F0Fu) | ((s0 >> 2) & 0x30303030u);
        mB = ((s2 >> 4) & 0x0F0F0F0Fu) | ((s1 >> 2) & 0x30303030u);
    }
    __device__ __forceinline__ uint32_t sc(int j) const { return hsub2_u(dup_byte_magic(j < 4 ? scA : scB, j & 3), H2_1024); }
    __device__ __forceinline__ uint32_t mn(int j) const { return hsub2_u(dup_byte_magic(j < 4 ? mA : mB, j & 3), H2_1024); }
};

// Q4_K and Q5_K (dequant_q4_k.glsl / dequant_q5_k.glsl): value = (d*sc)*q - dmin*m.
// A operand = sc*q (exact).  The min term sum_j m_j * X_j, X_j the sum of
// the activations over sub-block j, is one extra MMA per super-block whose
// k-slots are the 8 sub-blocks: A = m_j, B = X_j split into fp16 hi (slots
// 0..7) + lo (slots 8..15), precomputed once per CTA.  Each call decodes a
// range of 64-value chunks [IL0, IL0 + NIL); IL0 == 0 also does the min MMA.
template <bool Q5, int IL0, int NIL> struct StepK {
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xc,
                                               const uint8_t *xs, int t, float (&acc)[4]) {
        constexpr int QS = Q5 ? 48 : 16;
        const float da = hbits(ra), db = hbits(rb);
        KScales ka(ra + 4), kb(rb + 4);
        float p1[2][4];
        zero4(p1[0]);
        zero4(p1[1]);
#pragma unroll
        for (int i = 0; i < NIL; ++i) {
            const int il = IL0 + i;
            const int j0 = 2 * il, j1 = 2 * il + 1;
            uint32_t sla = ka.sc(j0), slb = kb.sc(j0);
            uint32_t cla = hmul2_u(sla, H2_M1024), clb = hmul2_u(slb, H2_M1024);
            uint32_t sha = ka.sc(j1), shb = kb.sc(j1);
            uint32_t cha = hmul2_u(sha, H2_M64), chb = hmul2_u(shb, H2_M64);
            sha = hmul2_u(sha, H2_SIXTEENTH);
            shb = hmul2_u(shb, H2_SIXTEENTH);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                uint32_t wa = ld32(ra + QS + 32 * il + 16 * h + 4 * t);
                uint32_t wb = ld32(rb + QS + 32 * il + 16 * h + 4 * t);
                uint32_t wa8 = wa >> 8, wb8 = wb >> 8;
                uint32_t la0 = lop3_and_or(wa, 0x000F000Fu, H2_MAGIC), la1 = lop3_and_or(wa8, 0x000F000Fu, H2_MAGIC);
                uint32_t lb0 = lop3_and_or(wb, 0x000F000Fu, H2_MAGIC), lb1 = lop3_and_or(wb8, 0x000F000Fu, H2_MAGIC);
                uint32_t ha0 = lop3_and_or(wa, 0x00F000F0u, H2_MAGIC), ha1 = lop3_and_or(wa8, 0x00F000F0u, H2_MAGIC);
                uint32_t hb0 = lop3_and_or(wb, 0x00F000F0u, H2_MAGIC), hb1 = lop3_and_or(wb8, 0x00F000F0u, H2_MAGIC);
                if constexpr (Q5) {
                    // 5th bit: qh[l] bit j0 (low nibbles) / j1 (high nibbles), dequant_q5_k.glsl:57-69
                    const uint32_t qa = ld32(ra + 16 + 16 * h + 4 * t), qb = ld32(rb + 16 + 16 * h + 4 * t);
                    auto lo02 = [&](uint32_t q) { return j0 <= 4 ? (q << (4 - j0)) : (q >> (j0 - 4)); };
                    la0 = lop3_and_or(lo02(qa), 0x00100010u, la0);
                    lb0 = lop3_and_or(lo02(qb), 0x00100010u, lb0);
                    la1 = lop3_and_or(qa >> (4 + j0), 0x00100010u, la1);
                    lb1 = lop3_and_or(qb >> (4 + j0), 0x00100010u, lb1);
                    ha0 = lop3_and_or(qa << (8 - j1), 0x01000100u, ha0);
                    hb0 = lop3_and_or(qb << (8 - j1), 0x01000100u, hb0);
                    ha1 = lop3_and_or(qa >> j1, 0x01000100u, ha1);
                    hb1 = lop3_and_or(qb >> j1, 0x01000100u, hb1);
                }
                const uint32_t alo[4] = {hfma2_u(la0, sla, cla), hfma2_u(lb0, slb, clb), hfma2_u(la1, sla, cla),
                                         hfma2_u(lb1, slb, clb)};
                const uint32_t ahi[4] = {hfma2_u(ha0, sha, cha), hfma2_u(hb0, shb, chb), hfma2_u(ha1, sha, cha),
                                         hfma2_u(hb1, shb, chb)};
                uint32_t b0, b1, b2, b3;
                xfrag(xc, 64 * il + 16 * h, t, b0, b1);
                xfrag(xc, 64 * il + 32 + 16 * h, t, b2, b3);
                mma_16816(p1[h], alo, b0, b1);
                mma_16816(p1[h], ahi, b2, b3);
            }
        }
        float p2[4];
        zero4(p2);
        if constexpr (IL0 == 0) {
            // thread t holds sub-blocks 2t, 2t+1: A = (m, m) for rows g, g+8; B = sums (hi | lo)
            const uint32_t sel = (t & 1) ? 0x4342u : 0x4140u;
            uint32_t am[4];
            am[0] = am[2] = hsub2_u(prmt(t < 2 ? ka.mA : ka.mB, 0x64646464u, sel), H2_1024);
            am[1] = am[3] = hsub2_u(prmt(t < 2 ? kb.mA : kb.mB, 0x64646464u, sel), H2_1024);
            const uint2 v = *reinterpret_cast<const uint2 *>(xs + 8 * t);
            mma_16816(p2, am, v.x, v.y);
        }
        const float dma = IL0 == 0 ? hbits(ra + 2) : 0.f, dmb = IL0 == 0 ? hbits(rb + 2) : 0.f;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const float d = i < 2 ? da : db, dm = i < 2 ? dma : dmb;
            acc[i] = fmaf(-dm, p2[i], fmaf(d, p1[0][i] + p1[1][i], acc[i]));
        }
    }
};

template <> struct Step<VKF_DEQUANT_Q4_K> {
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xc,
                                               const uint8_t *xs, int t, int part, int, float (&acc)[4]) {
        StepK<false, 0, 4>::run(ra, rb, xc, xs, t, acc);
    }
};
template <> struct Step<VKF_DEQUANT_Q5_K> {
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xc,
                                               const uint8_t *xs, int t, int part, int, float (&acc)[4]) {
        StepK<true, 0, 4>::run(ra, rb, xc, xs, t, acc);
    }
};

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

template <> struct Step<VKF_DEQUANT_Q6_K> {
    __device__ __forceinline__ static void run(const uint8_t *ra, const uint8_t *rb, const uint8_t *xc,
                                               const uint8_t *, int t, int part, int, float (&acc)[4]) {
        StepQ6<0>::run(ra, rb, xc, t, acc);
        StepQ6<1>::run(ra, rb, xc, t, acc);
    }
};

}  // namespace gemv
}  // namespace vkf
