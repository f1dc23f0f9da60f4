// tc_common.cuh — sm_100a tensor-core (tcgen05 / TMEM / TMA) helpers.
//
// Descriptor layouts follow the PTX ISA for tcgen05 (sm_100a):
//   shared-memory matrix descriptor (64 bit): start address >> 4 [0,14),
//     leading-dimension byte offset >> 4 [16,30), stride-dimension byte
//     offset >> 4 [32,46), descriptor version 1 [46,48), base offset [49,52),
//     LBO mode [52], layout [61,64) (2 = 128-byte swizzle);
//   instruction descriptor (32 bit) for kind::f16 / kind::i8: D format
//     [4,6) (1 = f32, 2 = s32), A format [7,10), B format [10,13) (f16 = 0 /
//     s8 = 1), A major [15], B major [16] (0 = K-major), N >> 3 [17,23),
//     M >> 4 [24,29).
// Operand tiles are K-major, 128 bytes of K per row, 128-byte swizzled: the
// layout a 2-D TMA load with CU_TENSOR_MAP_SWIZZLE_128B writes (8-row atoms
// of 1024 bytes, 16-byte chunk c of row r stored at chunk c ^ (r & 7)).
#pragma once

#include "device_common.cuh"

namespace vkf {
namespace tc {

__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFF) >> 4);        // start address
    d |= (uint64_t)1 << 16;                          // LBO (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;                // SBO: 8-row atom stride
    d |= (uint64_t)1 << 46;                          // descriptor version
    d |= (uint64_t)2 << 61;                          // 128-byte swizzle
    return d;
}

// Operand kinds: f16 x f16 -> f32 (kind::f16), s8 x s8 -> s32 (kind::i8),
// tf32 x tf32 -> f32 (kind::tf32, fp32 operands in memory).
enum Kind { KIND_F16 = 0, KIND_I8 = 1, KIND_TF32 = 2 };

// Both operands K-major.  A/B format: f16 = 0, tf32 = 2 (kind::f16 family);
// s8 = 1 (kind::i8).  D format: f32 = 1, s32 = 2.
__host__ __device__ constexpr uint32_t instr_desc(int kind, int M, int N) {
    return (uint32_t)((kind == KIND_I8 ? 2u : 1u) << 4) |
           (uint32_t)((kind == KIND_I8 ? 1u : kind == KIND_TF32 ? 2u : 0u) << 7) |
           (uint32_t)((kind == KIND_I8 ? 1u : kind == KIND_TF32 ? 2u : 0u) << 10) | (uint32_t)((N >> 3) << 17) |
           (uint32_t)((M >> 4) << 24);
}

template <int KIND>
__device__ __forceinline__ void mma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    if constexpr (KIND == KIND_I8)
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
    else if constexpr (KIND == KIND_TF32)
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
    else
        asm volatile(
            "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
            " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(tmem_d),
            "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
}

// Arrives on the mbarrier once all MMAs this thread issued have completed.
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
}

__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

// Whole warp: allocate ncols TMEM columns, base address written to *slot.
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(slot)), "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(ncols) : "memory");
}

// 32 lanes x 32 columns of 32-bit accumulators: thread l of the warp gets
// lane (taddr.lane + l), columns taddr.col .. +31.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 2-D TMA tile load (no multicast): box at (x = inner element, y = row).
__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(tmap), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// MMA with the A operand in tensor memory (M = 128 rows = lanes, K packed two
// 16-bit values per 32-bit column) and B from shared memory.
__device__ __forceinline__ void mma_f16_ta(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                           uint32_t acc) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc));
}

// Thread l of the warp writes 16 consecutive 32-bit columns of lane
// (taddr.lane + l); followed by wait::st before the data is signalled.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 2-D TMA tile store from shared memory (no multicast); elements outside the
// tensor are not written.  Completion is tracked by bulk groups.
__device__ __forceinline__ void tma_store_2d(const void *tmap, const void *src, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
                 "r"(smem_addr(src)), "r"(x), "r"(y)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups still READ their shared source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until every committed bulk group has completed (writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Orders this thread's generic-proxy shared-memory writes before later
// async-proxy (TMA / tensor core) accesses.
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

}  // namespace tc
}  // namespace vkf
