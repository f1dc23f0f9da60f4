// q8_1.cu — on-device Q8_1 activation quantiser and Q8_1 -> fp16 widening.
//
// The reference only decodes Q8_1 (kernels/dequant_q8_1.glsl); ggml produces
// it on the device before its mul_mat_q kernels, so the B200 path provides
// the producer.  One warp per 32-value block, one value per lane: the fp32
// input is read fully coalesced and the 36-byte block written by 9 lanes.
// The arithmetic is IEEE-rounded fp32 (no fast-math), so it matches the CPU
// oracle (oracle_quantize_q8_1) bit for bit.

#include "device_common.cuh"

namespace vkf {
namespace {

// Four threads per 32-value block, eight values each (two 16-byte loads when
// x rows are 16-byte aligned): max and sum by shuffles inside the 4-lane
// group, eight codes stored as two 4-byte words (2-byte halves when y is
// only 2-byte aligned).  Same IEEE-rounded operations per value as the
// oracle.  vec bits: 1 = vector loads, 2 = y 4-byte aligned.
__global__ void __launch_bounds__(256) quantize_q8_1_kernel(const float *__restrict__ x, uint8_t *__restrict__ y,
                                                            int M, int K, int64_t ldx, int vec) {
    const int64_t t = (int64_t)blockIdx.x * 256 + threadIdx.x;
    const int qtr = threadIdx.x & 3;
    const int nbr = K / 32;
    const int64_t blk = t >> 2;
    const bool on = blk < (int64_t)M * nbr;  // whole 4-lane groups share `on`
    const int64_t m = on ? blk / nbr : 0, b = on ? blk % nbr : 0;
    float v[8];
    if (on) {
        const float *src = x + m * ldx + b * 32 + 8 * qtr;
        if (vec & 1) {
            const float4 a0 = __ldg(reinterpret_cast<const float4 *>(src)), a1 = __ldg(reinterpret_cast<const float4 *>(src) + 1);
            v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w; v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
        } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = src[i];
        }
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = 0.f;
    }
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.0f);
    // v * rn(1/d) is within 2^-23 relative (|v/d| <= 127: 1.6e-5 absolute) of
    // v / d, so it rounds to the same integer unless the quotient lies that
    // close to a half-integer; those take the IEEE division.
    const float r = d != 0.0f ? __frcp_rn(d) : 0.0f;
    int sum = 0;
    uint32_t w[2] = {0u, 0u};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        int q = 0;
        if (d != 0.0f) {
            float t = v[i] * r;
            if (fabsf(fabsf(t - truncf(t)) - 0.5f) < 6.2e-5f) t = __fdiv_rn(v[i], d);
            q = (int)roundf(t);
            q = max(-127, min(127, q));
        }
        sum += q;
        w[i >> 2] |= (uint32_t)(q & 0xFF) << (8 * (i & 3));
    }
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if (!on) return;
    uint8_t *out = y + blk * 36;
    if (vec & 2) {  // y 4-byte aligned
        uint32_t *codes = reinterpret_cast<uint32_t *>(out + 4 + 8 * qtr);
        codes[0] = w[0];
        codes[1] = w[1];
    } else {
        uint16_t *codes = reinterpret_cast<uint16_t *>(out + 4 + 8 * qtr);
#pragma unroll
        for (int i = 0; i < 4; ++i) codes[i] = (uint16_t)(w[i >> 1] >> (16 * (i & 1)));
    }
    if (qtr == 0) {
        const __half hd = __float2half_rn(d), hs = __float2half_rn(__fmul_rn(d, (float)sum));
        *reinterpret_cast<__half *>(out) = hd;
        *reinterpret_cast<__half *>(out + 2) = hs;
    }
}

// Q8_1 (M rows of K/32 blocks, row stride ldb blocks) -> fp16 M x K (row stride
// ldo).  Four threads per block, eight values each: two 4-byte loads of
// codes (blocks are 36 bytes, so their codes are 4-byte aligned), one 16-byte
// store.  Grid: (blocks of a row / 64, M).
__global__ void __launch_bounds__(256) q8_1_to_f16_kernel(const uint8_t *__restrict__ src, __half *__restrict__ dst,
                                                          int M, int K, int64_t ldb, int64_t ldo) {
    // Programmatic dependent launch: the next kernel (the GEMM) may start its
    // set-up now; src is read only after the previous kernel completed.
    asm volatile("griddepcontrol.launch_dependents;");
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int nbr = K / 32;
    const int i = blockIdx.x * 256 + threadIdx.x;  // (block, quarter) within the row
    const int b = i >> 2, qtr = i & 3;
    if (b >= nbr) return;
    const int m = blockIdx.y;
    const uint8_t *p = src + ((int64_t)m * ldb + b) * 36;
    const float d = __half2float(*reinterpret_cast<const __half *>(p));
    const uint32_t w0 = *reinterpret_cast<const uint32_t *>(p + 4 + 8 * qtr);
    const uint32_t w1 = *reinterpret_cast<const uint32_t *>(p + 8 + 8 * qtr);
    uint32_t o[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
        const uint32_t w = k < 2 ? w0 : w1;
        const int sh = 16 * (k & 1);
        const float lo = __fmul_rn(d, (float)(int8_t)(w >> sh)), hi = __fmul_rn(d, (float)(int8_t)(w >> (sh + 8)));
        const __half2 h = __floats2half2_rn(lo, hi);
        o[k] = *reinterpret_cast<const uint32_t *>(&h);
    }
    __half *q = dst + (int64_t)m * ldo + b * 32 + 8 * qtr;
    if (((uintptr_t)q & 15) == 0) {
        *reinterpret_cast<uint4 *>(q) = make_uint4(o[0], o[1], o[2], o[3]);
    } else {
#pragma unroll
        for (int k = 0; k < 4; ++k) reinterpret_cast<__half2 *>(q)[k] = *reinterpret_cast<const __half2 *>(&o[k]);
    }
}

}  // namespace

int q8_1_to_f16(const void *src, void *dst, int M, int K, int64_t ldb, int64_t ldo, cudaStream_t stream) {
    const int nbr = K / 32;
    if (M == 0 || nbr == 0) return VKF_OK;
    if (M > 65535) return VKF_ERR_UNSUPPORTED;
    const dim3 grid((unsigned)((nbr * 4 + 255) / 256), (unsigned)M);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaLaunchKernelEx(&cfg, q8_1_to_f16_kernel, (const uint8_t *)src, (__half *)dst, M, K, ldb, ldo);
    return check_launch();
}

int quantize_q8_1_launch(const float *x, void *y, int M, int K, int64_t ldx, cudaStream_t stream) {
    int64_t blocks = (int64_t)M * (K / 32);
    if (blocks == 0) return VKF_OK;
    const int vec = (((uintptr_t)x & 15) == 0 && ldx % 4 == 0 ? 1 : 0) | (((uintptr_t)y & 3) == 0 ? 2 : 0);
    quantize_q8_1_kernel<<<(unsigned)((blocks * 4 + 255) / 256), 256, 0, stream>>>(x, (uint8_t *)y, M, K, ldx, vec);
    return check_launch();
}

}  // namespace vkf

extern "C" int vkflame_quantize_q8_1(const float *x, void *y, int M, int K, int64_t ldx, void *stream) {
    if (M < 0 || K < 0 || K % 32 || ldx < K) return vkf::set_status(VKF_ERR_INVALID);
    if (M == 0 || K == 0) return vkf::set_status(VKF_OK);
    if (vkf::validate_device_range(x, ((size_t)(M - 1) * ldx + K) * 4) != VKF_OK ||
        vkf::validate_device_range(y, (size_t)M * (K / 32) * 36) != VKF_OK || ((uintptr_t)x & 3) ||
        ((uintptr_t)y & 1))
        return vkf::set_status(VKF_ERR_BADPTR);
    return vkf::set_status(vkf::quantize_q8_1_launch(x, y, M, K, ldx, (cudaStream_t)stream));
}
