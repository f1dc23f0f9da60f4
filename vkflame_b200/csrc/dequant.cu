// dequant.cu — ggml block formats -> fp32, bit-exact with the reference's
// kernels/dequant_*.glsl.
//
// Work unit: 256 output values (one Q4_K/Q5_K/Q6_K super-block, or eight
// 32-value blocks of Q4_0/Q4_1/Q5_0/Q8_0/Q8_1).  One warp per unit, each lane
// producing 8 consecutive values with two 16-byte stores, so the fp32 output
// (4 B/value, the dominant traffic) is written fully coalesced.  Every value
// uses the shader's own formula with explicitly rounded fp32 operations
// (__fmul_rn/__fadd_rn: no contraction), and every product is exact (fp16
// scale x small integer), so the results equal the shaders' bit for bit.

#include "device_common.cuh"

namespace vkf {
namespace {

__device__ __forceinline__ float h2f(const uint8_t *p) {
    return half_bits_to_float((uint16_t)(p[0] | (p[1] << 8)));
}

// Values [v0, v0+8) of 32-value block `b` (v0 in {0, 8, 16, 24}).
template <int QT>
__device__ __forceinline__ void dq_block32(const uint8_t *b, int v0, float (&o)[8]) {
    if constexpr (QT == VKF_DEQUANT_Q4_0) {  // dequant_q4_0.glsl:25-36
        float d = h2f(b), dm = __fmul_rn(-8.0f, d);
        const uint8_t *qs = b + 2;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int v = v0 + i;
            unsigned q = v < 16 ? (qs[v] & 0xFu) : (qs[v - 16] >> 4);
            o[i] = __fadd_rn(__fmul_rn(d, (float)q), dm);
        }
    } else if constexpr (QT == VKF_DEQUANT_Q4_1) {  // dequant_q4_1.glsl:25-36
        float d = h2f(b), m = h2f(b + 2);
        const uint8_t *qs = b + 4;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int v = v0 + i;
            unsigned q = v < 16 ? (qs[v] & 0xFu) : (qs[v - 16] >> 4);
            o[i] = __fadd_rn(__fmul_rn(d, (float)q), m);
        }
    } else if constexpr (QT == VKF_DEQUANT_Q5_0) {  // dequant_q5_0.glsl:27-46
        float d = h2f(b), dm = __fmul_rn(-16.0f, d);
        uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
        const uint8_t *qs = b + 6;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int v = v0 + i;
            unsigned x;
            if (v < 16) x = (qs[v] & 0xFu) | (((qh >> v) << 4) & 0x10u);
            else x = (qs[v - 16] >> 4) | ((qh >> (v - 16 + 12)) & 0x10u);
            o[i] = __fadd_rn(__fmul_rn((float)x, d), dm);
        }
    } else if constexpr (QT == VKF_DEQUANT_Q8_0 || QT == VKF_DEQUANT_Q8_1) {  // dequant_q8_{0,1}.glsl
        float d = h2f(b);
        const int8_t *qs = reinterpret_cast<const int8_t *>(b + (QT == VKF_DEQUANT_Q8_0 ? 2 : 4));
#pragma unroll
        for (int i = 0; i < 8; ++i) o[i] = __fmul_rn(d, (float)qs[v0 + i]);
    }
}

// get_scale_min_k4 (dequant_q4_k.glsl:16-24).
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t *s, float &sc, float &mn) {
    if (j < 4) {
        sc = (float)(s[j] & 63u);
        mn = (float)(s[j + 4] & 63u);
    } else {
        sc = (float)((s[j + 4] & 0xFu) | ((s[j - 4] >> 6) << 4));
        mn = (float)((s[j + 4] >> 4) | ((s[j] >> 6) << 4));
    }
}

// Values [v0, v0+8) of a 256-value super-block (v0 multiple of 8).
template <int QT>
__device__ __forceinline__ void dq_super(const uint8_t *b, int v0, float (&o)[8]) {
    if constexpr (QT == VKF_DEQUANT_Q4_K || QT == VKF_DEQUANT_Q5_K) {  // dequant_q4_k.glsl:35-57, q5_k:37-74
        float dall = h2f(b), dmin = h2f(b + 2);
        int il = v0 >> 6, w = v0 & 63;
        bool hi = w >= 32;
        int l0 = hi ? w - 32 : w;
        int j = 2 * il + (hi ? 1 : 0);
        float sc, mn;
        scale_min_k4(j, b + 4, sc, mn);
        float dd = __fmul_rn(dall, sc), mm = __fmul_rn(dmin, mn);
        const uint8_t *qs = b + (QT == VKF_DEQUANT_Q4_K ? 16 : 48);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            unsigned q = qs[32 * il + l0 + i];
            q = hi ? (q >> 4) : (q & 0xFu);
            if constexpr (QT == VKF_DEQUANT_Q5_K) q += (b[16 + l0 + i] & (1u << j)) ? 16u : 0u;
            o[i] = __fsub_rn(__fmul_rn(dd, (float)q), mm);
        }
    } else {  // Q6_K, dequant_q6_k.glsl:28-58
        const uint8_t *ql = b, *qh = b + 128;
        const int8_t *scales = reinterpret_cast<const int8_t *>(b + 192);
        float d = h2f(b + 208);
        int ip = v0 >> 7, r = v0 & 127, s = r >> 5, il0 = r & 31;
        int sc = scales[8 * ip + (il0 >> 4) + 2 * s];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            int il = il0 + i;
            unsigned qlb = ql[64 * ip + il + 32 * (s & 1)];
            unsigned nib = (s < 2) ? (qlb & 0xFu) : (qlb >> 4);
            unsigned hb = (qh[32 * ip + il] >> (2 * s)) & 3u;
            int v = (int)(nib | (hb << 4)) - 32;
            o[i] = __fmul_rn(d, (float)(sc * v));
        }
    }
}

template <int QT, bool ALIGNED16, bool F16OUT>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t *__restrict__ src, void *__restrict__ dstv,
                                                      uint64_t nb) {
    constexpr bool SUPER = (QT == VKF_DEQUANT_Q4_K || QT == VKF_DEQUANT_Q5_K || QT == VKF_DEQUANT_Q6_K);
    constexpr int BB = (QT == VKF_DEQUANT_Q4_0) ? 18 : (QT == VKF_DEQUANT_Q4_1) ? 20 : (QT == VKF_DEQUANT_Q5_0) ? 22
                     : (QT == VKF_DEQUANT_Q8_0) ? 34 : (QT == VKF_DEQUANT_Q8_1) ? 36 : (QT == VKF_DEQUANT_Q4_K) ? 144
                     : (QT == VKF_DEQUANT_Q5_K) ? 176 : 210;
    const int lane = threadIdx.x & 31;
    const uint64_t unit = (uint64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
    float o[8];
    uint64_t block;
    int v0;
    if constexpr (SUPER) {
        block = unit;
        v0 = lane * 8;
        if (block >= nb) return;
        dq_super<QT>(src + block * BB, v0, o);
    } else {
        block = unit * 8 + (lane >> 2);
        v0 = (lane & 3) * 8;
        if (block >= nb) return;
        dq_block32<QT>(src + block * BB, v0, o);
    }
    if constexpr (F16OUT) {  // fp16 copy for the tensor-core GEMM (one rounding per value)
        __half2 h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(o[2 * i], o[2 * i + 1]);
        *reinterpret_cast<uint4 *>(reinterpret_cast<__half *>(dstv) + unit * 256 + lane * 8) =
            *reinterpret_cast<uint4 *>(h);
        return;
    }
    float *out = reinterpret_cast<float *>(dstv) + unit * 256 + lane * 8;
    if constexpr (ALIGNED16) {
        reinterpret_cast<float4 *>(out)[0] = make_float4(o[0], o[1], o[2], o[3]);
        reinterpret_cast<float4 *>(out)[1] = make_float4(o[4], o[5], o[6], o[7]);
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = o[i];
    }
}

template <int QT>
int launch_dequant(const void *src, void *dst, uint64_t nb, cudaStream_t stream, bool f16out) {
    constexpr bool SUPER = (QT == VKF_DEQUANT_Q4_K || QT == VKF_DEQUANT_Q5_K || QT == VKF_DEQUANT_Q6_K);
    uint64_t units = SUPER ? nb : (nb + 7) / 8;
    uint64_t grid = (units + 7) / 8;
    if (grid == 0) return VKF_OK;
    if (grid > 0x7fffffffULL) return VKF_ERR_INVALID;
    bool aligned = ((uintptr_t)dst & 15) == 0;
    if (f16out) {
        if (!aligned) return VKF_ERR_BADPTR;
        dequant_kernel<QT, true, true><<<(unsigned)grid, 256, 0, stream>>>((const uint8_t *)src, dst, nb);
    } else if (aligned)
        dequant_kernel<QT, true, false><<<(unsigned)grid, 256, 0, stream>>>((const uint8_t *)src, dst, nb);
    else
        dequant_kernel<QT, false, false><<<(unsigned)grid, 256, 0, stream>>>((const uint8_t *)src, dst, nb);
    return check_launch();
}

}  // namespace

int dequant_launch(const void *src, void *dst, uint64_t nb, int qtype, cudaStream_t stream, bool f16out) {
    switch (qtype) {
    case VKF_DEQUANT_Q4_0: return launch_dequant<VKF_DEQUANT_Q4_0>(src, dst, nb, stream, f16out);
    case VKF_DEQUANT_Q4_1: return launch_dequant<VKF_DEQUANT_Q4_1>(src, dst, nb, stream, f16out);
    case VKF_DEQUANT_Q8_0: return launch_dequant<VKF_DEQUANT_Q8_0>(src, dst, nb, stream, f16out);
    case VKF_DEQUANT_Q5_0: return launch_dequant<VKF_DEQUANT_Q5_0>(src, dst, nb, stream, f16out);
    case VKF_DEQUANT_Q4_K: return launch_dequant<VKF_DEQUANT_Q4_K>(src, dst, nb, stream, f16out);
    case VKF_DEQUANT_Q5_K: return launch_dequant<VKF_DEQUANT_Q5_K>(src, dst, nb, stream, f16out);
    case VKF_DEQUANT_Q6_K: return launch_dequant<VKF_DEQUANT_Q6_K>(src, dst, nb, stream, f16out);
    case VKF_DEQUANT_Q8_1: return launch_dequant<VKF_DEQUANT_Q8_1>(src, dst, nb, stream, f16out);
    default: return VKF_ERR_INVALID;
    }
}

}  // namespace vkf

extern "C" int vkflame_dispatch_dequant_async(const void *src, void *dst, uint64_t n_blocks, int quant_type,
                                              void *stream) {
    if (quant_type < 0 || quant_type >= VKF_NUM_QTYPES) return vkf::set_status(VKF_ERR_INVALID);
    if (n_blocks == 0) return vkf::set_status(VKF_OK);
    size_t in_bytes = (size_t)n_blocks * vkf_qtype_block_bytes(quant_type);
    size_t out_bytes = (size_t)n_blocks * vkf_qtype_block_values(quant_type) * sizeof(float);
    if (vkf::validate_device_range(src, in_bytes) != VKF_OK || vkf::validate_device_range(dst, out_bytes) != VKF_OK ||
        ((uintptr_t)dst & 3) || ((uintptr_t)src & 1))
        return vkf::set_status(VKF_ERR_BADPTR);
    return vkf::set_status(vkf::dequant_launch(src, dst, n_blocks, quant_type, (cudaStream_t)stream, false));
}

extern "C" int vkflame_dispatch_dequant(void *ctx, const void *src, void *dst, uint32_t n_blocks, int quant_type) {
    (void)ctx;
    return vkflame_dispatch_dequant_async(src, dst, n_blocks, quant_type, nullptr);
}
