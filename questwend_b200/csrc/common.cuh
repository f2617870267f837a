// common.cuh - device-side building blocks shared by the qwb kernels (sm_100a only).
//
// Block formats are ggml's (ggml-common.h:251-255 block_q8_0, :327-337 block_q4_K,
// :362-367 block_q6_K, :370-375 block_q8_K): same field order and byte sizes, because the
// weights are read straight out of ggml-owned buffers and expert-slot pools.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/qwb.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "qwb is built for sm_100a only"
#endif

namespace qwb {

constexpr int QK_K = 256;
constexpr int QK8_0 = 32;

constexpr int Q4K_BYTES = 144;  // d, dmin (fp16), scales[12], qs[128]
constexpr int Q6K_BYTES = 210;  // ql[128], qh[64], scales[16] (int8), d (fp16)
constexpr int Q80_BYTES = 34;   // d (fp16), qs[32]
constexpr int Q8K_BYTES = 292;  // d (f32), qs[256], bsums[16] (int16)

// Internal activation layout ("q8 planes"): the bytes of ggml's block_q8_K / block_q8_0
// rows, split into separately aligned planes so the GEMV/GEMM kernels can use wide loads:
//   qs   int8  [rows][K]
//   d    float [rows][K/blk]   (Q8_0: the fp16 scale widened to f32 - exact)
//   bsum int16 [rows][K/16]    (Q8_K only)
struct Q8Planes {
    int8_t *qs;
    float *d;
    int16_t *bsum;
    int64_t K;
};

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
__host__ __device__ inline size_t align_up(size_t a, size_t b) { return (a + b - 1) / b * b; }

inline size_t row_bytes(int type, int64_t n) {
    switch (type) {
        case QWB_TYPE_F32: case QWB_TYPE_I32: return (size_t) n * 4;
        case QWB_TYPE_F16: return (size_t) n * 2;
        case QWB_TYPE_Q8_0: return (size_t) (n / QK8_0) * Q80_BYTES;
        case QWB_TYPE_Q4_K: return (size_t) (n / QK_K) * Q4K_BYTES;
        case QWB_TYPE_Q6_K: return (size_t) (n / QK_K) * Q6K_BYTES;
        case QWB_TYPE_Q8_K: return (size_t) (n / QK_K) * Q8K_BYTES;
        default: return 0;
    }
}
inline int block_elems(int type) {
    switch (type) {
        case QWB_TYPE_Q8_0: return QK8_0;
        case QWB_TYPE_Q4_K: case QWB_TYPE_Q6_K: case QWB_TYPE_Q8_K: return QK_K;
        default: return 1;
    }
}

// --------------------------------------------------------------- conversions
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }
__device__ __forceinline__ uint16_t f2h_rn(float f) { return __half_as_ushort(__float2half_rn(f)); }

// 6-bit scale / min j of a Q4_K superblock from its 12 packed bytes (get_scale_min_k4,
// ggml-quants.c:880-887)
__device__ __forceinline__ void q4k_scale_min(int j, const uint8_t *q, int &sc, int &m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// --------------------------------------------------------------- status block
__device__ __forceinline__ void report(qwb_status_block *st, uint32_t flag, int32_t value) {
    if (!st) return;
    if (atomicAdd(&st->count, 1u) == 0u) st->bad_value = value;
    atomicOr(&st->flags, flag);
}

// ------------------------------------------------ mbarrier + bulk async copies
// Non-tensor TMA (cp.async.bulk) global -> shared copies completing on an mbarrier.
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return (uint32_t) __cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
// One poll of the barrier phase; the thread may be suspended (not spinning) for up to
// `hint_ns` while the phase is incomplete, so waiting warps do not steal issue slots.
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity, uint32_t hint_ns = 1000u) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}
// One poll without a suspend-time hint: the hardware may hold the thread for a short,
// implementation-defined window and returns as soon as the phase completes.  Used on
// pipelines whose stages turn over every few hundred cycles.
__device__ __forceinline__ bool mbar_try_wait_fast(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: polls the barrier phase until it completes or `limit_ns` of wall time
// (the GPU's global timer) have passed, then returns false.  Every wait in this library
// goes through here, so no kernel can spin forever on a copy that never lands.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint64_t limit_ns = kWaitLimitNs) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (globaltimer_ns() - t0 > limit_ns) return false;
    }
}
// 16-byte aligned src/dst, bytes % 16 == 0
__device__ __forceinline__ void bulk_g2s(void *dst_smem, const void *src_gmem, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst_smem)),
        "l"(src_gmem), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Copy the byte range [src, src + bytes) of global memory into shared memory at `dst`
// (16-byte aligned), widening it to 16-byte boundaries; returns the offset of src's first
// byte inside dst.  Issued by ONE thread; the caller accounts for the widened size
// (bulk_span_bytes) in the mbarrier's expected transaction bytes.  Splits into pieces of
// at most 64 KiB.
__host__ __device__ __forceinline__ uint32_t bulk_span_bytes(const void *src, size_t bytes) {
    const uintptr_t a = (uintptr_t) src & ~(uintptr_t) 15;
    const uintptr_t e = ((uintptr_t) src + bytes + 15) & ~(uintptr_t) 15;
    return (uint32_t) (e - a);
}
__device__ __forceinline__ uint32_t bulk_span_issue(void *dst, const void *src, size_t bytes, uint64_t *bar) {
    const uintptr_t a = (uintptr_t) src & ~(uintptr_t) 15;
    const uint32_t total = bulk_span_bytes(src, bytes);
    for (uint32_t off = 0; off < total; off += 65536u) {
        const uint32_t n = total - off < 65536u ? total - off : 65536u;
        bulk_g2s((char *) dst + off, (const void *) (a + off), n, bar);
    }
    return (uint32_t) ((uintptr_t) src - a);
}

// ------------------------------------------------------------- warp helpers
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Unaligned little-endian 32-bit load from shared memory at a 2-byte aligned address.
__device__ __forceinline__ int lds_u32_a2(const uint8_t *p) {
    const uint16_t *q = (const uint16_t *) p;
    return (int) ((uint32_t) q[0] | ((uint32_t) q[1] << 16));
}

}  // namespace qwb
