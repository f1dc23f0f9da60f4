// device_common.cuh — sm_100a device helpers shared by the kernels:
// fp16 bit helpers, mbarrier and bulk-copy (TMA) PTX wrappers with bounded
// waits, and the warp-level m16n8k16 MMA used by the decode GEMV.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "rt_internal.h"

namespace vkf {

__device__ __forceinline__ float half_bits_to_float(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

__device__ __forceinline__ uint16_t ld_u16(const uint8_t *p) {
    return *reinterpret_cast<const uint16_t *>(p);
}

// 4 bytes at a 2-byte aligned address.
__device__ __forceinline__ uint32_t ld_u32_a2(const uint8_t *p) {
    const uint16_t *q = reinterpret_cast<const uint16_t *>(p);
    return (uint32_t)q[0] | ((uint32_t)q[1] << 16);
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

// ---- mbarrier --------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile(
        "{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile(
        "{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(smem_addr(bar)),
        "r"(bytes)
        : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wall-clock limit of every bounded wait in these kernels.  A count of polls
// alone does not bound the time: each try_wait may suspend the thread for a
// hardware-defined interval, so 2^22 of them can take minutes.
constexpr uint64_t WAIT_LIMIT_NS = 1000000000ull;

// Bounded wait: gives up once WAIT_LIMIT_NS of global-timer time has passed
// (the timer is read only after the first 1024 polls, so waits that succeed
// soon never read it), ORs VKF_KERR_WAIT_TIMEOUT into *err and returns false.
// Callers then stop issuing work and exit.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned *err) {
    for (int i = 0; i < 1024; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    do {
        for (int i = 0; i < 256; ++i)
            if (mbar_try_wait(bar, parity)) return true;
    } while (globaltimer_ns() - t0 < WAIT_LIMIT_NS);
    if (err) atomicOr(err, VKF_KERR_WAIT_TIMEOUT);
    return false;
}

// ---- bulk copies (TMA, non-tensor) ---------------------------------------
// dst (shared) and src (global) 16-byte aligned, bytes a multiple of 16.
// No L2 cache-hint forms anywhere in this library: on B200 (driver 580) a
// copy carrying a createpolicy evict-first policy raised "illegal
// instruction" in a microbenchmark.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

// ---- warp MMA m16n8k16, fp16 x fp16 -> fp32 ---------------------------------
// A fragment (row-major 16x16): a[0] = (row g, k 2t..2t+1), a[1] = (row g+8, k 2t..),
// a[2] = (row g, k 2t+8..), a[3] = (row g+8, k 2t+8..); B (16x8): b[0] = (k 2t.., col g),
// b[1] = (k 2t+8.., col g); C: c[0..1] = (row g, col 2t..2t+1), c[2..3] = (row g+8, ...).
// g = lane >> 2, t = lane & 3.
// Accumulates in place (d += A*B): read-write operands avoid register copies.
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t mask, uint32_t orv) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(mask), "r"(orv));  // (a & b) | c
    return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
    uint32_t r;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
    return r;
}

__device__ __forceinline__ uint32_t half2_bits(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&h);
}

}  // namespace vkf
