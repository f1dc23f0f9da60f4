/*
 * ggml_blocks.h — byte layouts of the ggml block-quantised formats on the
 * vkflame hot path, shared by the CUDA kernels, the C-ABI and the CPU oracle.
 *
 * Layouts follow the block comments and byte offsets of the reference shaders:
 *   Q4_0  kernels/dequant_q4_0.glsl:2,25-29   [f16 d][16 B qs]                 18 B / 32 values
 *   Q4_1  kernels/dequant_q4_1.glsl:2,25-29   [f16 d][f16 m][16 B qs]          20 B / 32 values
 *   Q5_0  kernels/dequant_q5_0.glsl:2,27-33   [f16 d][4 B qh][16 B qs]         22 B / 32 values
 *   Q8_0  kernels/dequant_q8_0.glsl:2,24-26   [f16 d][32 x i8]                 34 B / 32 values
 *   Q8_1  kernels/dequant_q8_1.glsl:2,27-30   [f16 d][f16 s][32 x i8]          36 B / 32 values
 *   Q4_K  kernels/dequant_q4_k.glsl:2,35-39   [f16 d][f16 dmin][12 B sc][128 B qs]          144 B / 256
 *   Q5_K  kernels/dequant_q5_k.glsl:2,34-42   [f16 d][f16 dmin][12 B sc][32 B qh][128 B qs] 176 B / 256
 *   Q6_K  kernels/dequant_q6_k.glsl:2,25-32   [128 B ql][64 B qh][16 x i8 sc][f16 d]        210 B / 256
 *
 * Weights are stored one row per output channel: row n holds K/QK blocks,
 * rows are contiguous (row stride = K/QK * block bytes), no padding.
 * All structs are byte-packed (alignment 1 or 2): a block may start at any
 * even byte offset.  Kernels never rely on wider alignment of a block.
 *
 * The quant-type codes are the reference's VKF_DEQUANT_* values
 * (runtime/dispatch.h:14-21) so callers of vkflame_dispatch_dequant keep
 * their constants.
 */
#ifndef VKFLAME_GGML_BLOCKS_H
#define VKFLAME_GGML_BLOCKS_H

#include <stdint.h>

#define VKF_DEQUANT_Q4_0 0
#define VKF_DEQUANT_Q4_1 1
#define VKF_DEQUANT_Q8_0 2
#define VKF_DEQUANT_Q5_0 3
#define VKF_DEQUANT_Q4_K 4
#define VKF_DEQUANT_Q5_K 5
#define VKF_DEQUANT_Q6_K 6
#define VKF_DEQUANT_Q8_1 7
#define VKF_NUM_QTYPES 8

#define VKF_QK32 32
#define VKF_QK_K 256

#pragma pack(push, 1)
typedef struct { uint16_t d; uint8_t qs[16]; } vkf_block_q4_0;
typedef struct { uint16_t d; uint16_t m; uint8_t qs[16]; } vkf_block_q4_1;
typedef struct { uint16_t d; uint8_t qh[4]; uint8_t qs[16]; } vkf_block_q5_0;
typedef struct { uint16_t d; int8_t qs[32]; } vkf_block_q8_0;
typedef struct { uint16_t d; uint16_t s; int8_t qs[32]; } vkf_block_q8_1;
typedef struct { uint16_t d; uint16_t dmin; uint8_t scales[12]; uint8_t qs[128]; } vkf_block_q4_K;
typedef struct { uint16_t d; uint16_t dmin; uint8_t scales[12]; uint8_t qh[32]; uint8_t qs[128]; } vkf_block_q5_K;
typedef struct { uint8_t ql[128]; uint8_t qh[64]; int8_t scales[16]; uint16_t d; } vkf_block_q6_K;
#pragma pack(pop)

#ifdef __cplusplus
#define VKF_STATIC_ASSERT(c, m) static_assert(c, m)
#else
#define VKF_STATIC_ASSERT(c, m) _Static_assert(c, m)
#endif
VKF_STATIC_ASSERT(sizeof(vkf_block_q4_0) == 18, "Q4_0 block is 18 bytes");
VKF_STATIC_ASSERT(sizeof(vkf_block_q4_1) == 20, "Q4_1 block is 20 bytes");
VKF_STATIC_ASSERT(sizeof(vkf_block_q5_0) == 22, "Q5_0 block is 22 bytes");
VKF_STATIC_ASSERT(sizeof(vkf_block_q8_0) == 34, "Q8_0 block is 34 bytes");
VKF_STATIC_ASSERT(sizeof(vkf_block_q8_1) == 36, "Q8_1 block is 36 bytes");
VKF_STATIC_ASSERT(sizeof(vkf_block_q4_K) == 144, "Q4_K block is 144 bytes");
VKF_STATIC_ASSERT(sizeof(vkf_block_q5_K) == 176, "Q5_K block is 176 bytes");
VKF_STATIC_ASSERT(sizeof(vkf_block_q6_K) == 210, "Q6_K block is 210 bytes");

/* Values per block and bytes per block, indexed by VKF_DEQUANT_* code. */
static inline int vkf_qtype_block_values(int qtype) {
    return (qtype == VKF_DEQUANT_Q4_K || qtype == VKF_DEQUANT_Q5_K || qtype == VKF_DEQUANT_Q6_K) ? 256 : 32;
}
static inline int vkf_qtype_block_bytes(int qtype) {
    switch (qtype) {
    case VKF_DEQUANT_Q4_0: return 18;
    case VKF_DEQUANT_Q4_1: return 20;
    case VKF_DEQUANT_Q8_0: return 34;
    case VKF_DEQUANT_Q5_0: return 22;
    case VKF_DEQUANT_Q4_K: return 144;
    case VKF_DEQUANT_Q5_K: return 176;
    case VKF_DEQUANT_Q6_K: return 210;
    case VKF_DEQUANT_Q8_1: return 36;
    default: return 0;
    }
}

#endif /* VKFLAME_GGML_BLOCKS_H */
