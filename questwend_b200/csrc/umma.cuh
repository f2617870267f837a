// umma.cuh - 5th-generation tensor core (tcgen05) building blocks for sm_100a.
//
// Thin inline-PTX wrappers: tensor-memory (TMEM) allocation, the kind::f16 MMA with the A
// operand in TMEM or shared memory and B in shared memory, the kind::i8 MMA (both operands
// in shared memory), commit to an mbarrier,
// 32x32b TMEM loads/stores and the tcgen05 ordering fences.  Descriptor encodings follow
// the PTX ISA's "matrix descriptor" and "instruction descriptor" tables for tcgen05.mma.
//
// Shared-memory operand layout used throughout (K-major, no swizzle): the operand is a
// grid of 8-row x 16-byte "core matrices"; element (r, k) of a R-row slab of 16-bit values
// lives at   (k / 8) * (R * 16) + (r / 8) * 128 + (r % 8) * 16 + (k % 8) * 2   bytes.
// So the leading-dimension byte offset (between the two K-adjacent core matrices one
// K=16 MMA reads) is R * 16 and the stride byte offset (between 8-row groups) is 128.
//
// TMEM addresses: bits [31:16] lane, bits [15:0] 32-bit column.  An M=128 accumulator
// puts row m in lane m and column n in column n.  An A operand in TMEM puts row m in lane
// m and the 16-bit elements k = 2c, 2c+1 in column c (low half = even k).
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace qwb {
namespace umma {

// ---------------------------------------------------------------- descriptors
// kind::f16 instruction descriptor: A, B fp16, D f32, both operands K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N) {
    return (1u << 4)                          // D format: f32
           | (0u << 7) | (0u << 10)          // A, B format: f16
           | (0u << 15) | (0u << 16)         // A, B K-major
           | ((uint32_t) (N >> 3) << 17)     // N / 8
           | ((uint32_t) (M >> 4) << 24);    // M / 16
}

// Shared-memory matrix descriptor, no swizzle.  addr, lbo, sbo in bytes (16-byte units
// are encoded).
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t) ((saddr >> 4) & 0x3FFFu) | ((uint64_t) ((lbo >> 4) & 0x3FFFu) << 16) |
           ((uint64_t) ((sbo >> 4) & 0x3FFFu) << 32) | (1ull << 46);  // version 1 (sm_100)
}

// ---------------------------------------------------------------- allocation
// Executed by one full warp.  Writes the TMEM base address to *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// ---------------------------------------------------------------- fences
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- MMA
// D[tmem] (+)= A[tmem] * B[smem]^T      (issued by one thread)
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T      (issued by one thread)
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u), "r"(0u), "r"(0u), "r"(0u)
        : "memory");
}
// Arrive (once) on an mbarrier of this CTA when all MMAs issued so far by this thread
// have completed.
__device__ __forceinline__ void commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// ---------------------------------------------------------------- TMEM <-> registers
// Warp-collective.  Thread i of the warp accesses lane (taddr.lane + i) - the warp may only
// touch the 32-lane quarter (warp id % 4) - and N consecutive columns from taddr.col.
__device__ __forceinline__ void ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
          "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
          "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}
__device__ __forceinline__ void st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr), "r"(r[0]),
        "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
        : "memory");
}
__device__ __forceinline__ void st16(uint32_t taddr, const uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
        : "memory");
}

// mbarrier arrive (plain, count 1) - used by consumer threads to release a stage
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// kind::i8 instruction descriptor: A, B signed 8-bit, D signed 32-bit, both K-major, M x N.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N) {
    return (2u << 4)                         // D format: s32
           | (1u << 7) | (1u << 10)          // A, B format: signed 8-bit
           | (0u << 15) | (0u << 16)         // A, B K-major
           | ((uint32_t) (N >> 3) << 17)     // N / 8
           | ((uint32_t) (M >> 4) << 24);    // M / 16
}
// D[tmem] (+)= A[smem] * B[smem]^T, s8 x s8 -> s32, K = 32 (issued by one thread).
// Shared-memory layout of 8-bit operands (K-major, no swizzle): core matrices of 8 rows x
// 16 bytes; element (r, k) of an R-row slab at (k / 16) * (R * 16) + (r / 8) * 128 +
// (r % 8) * 16 + (k % 16): leading byte offset R * 16, stride byte offset 128.
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

}  // namespace umma

// Bounded wait.  The thread is suspended between polls until the phase completes.
__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                        qwb_status_block *st) {
    if (mbar_try_wait(bar, parity, 200000u)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity, 200000u)) return true;
        if (*abort) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) {
            *abort = 1;
            report(st, QWB_DEVERR_TIMEOUT, 0);
            return false;
        }
    }
}
// warp-uniform wait: lane 0 polls, the result is broadcast
__device__ __forceinline__ bool pf_wait_warp(uint64_t *bar, uint32_t parity, volatile int *abort,
                                             qwb_status_block *st) {
    int ok = 1;
    if ((threadIdx.x & 31) == 0) ok = pf_wait(bar, parity, abort, st);
    return __shfl_sync(0xffffffffu, ok, 0) != 0;
}
// One arrival of count 32 on behalf of the whole warp, after every lane's own memory and
// tcgen05 operations are ordered by the caller's fences.
__device__ __forceinline__ void warp_arrive(uint64_t *bar) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0)
        asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0], 32;" ::"r"(smem_u32(bar)) : "memory");
}

}  // namespace qwb
