// decode_dev.cuh - device building blocks of the decode GEMV kernels (decode.cu,
// mmid_one.cu): programmatic dependent launch, SwiGLU, and the Q4_K / Q6_K superblock
// dots against a Q8_K activation superblock held in registers (exact integer sub-block
// sums on the reference's Q8_K activation bytes, fp32 combine).
#pragma once

#include "common.cuh"

namespace qwb {

// ------------------------------------------------------------------- helpers
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// silu(g) * u as ggml_vec_swiglu_f32 (vec.cpp:417-447)
__device__ __forceinline__ float swiglu_f(float g, float u) { return g / (1.0f + expf(-g)) * u; }

// unsigned 4 x u8 . signed 4 x s8 dot product accumulate
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// One Q8_K activation superblock held in registers by a lane.
template <bool KQ6>
struct ActReg {
    int q[64];      // 256 int8
    int bs[KQ6 ? 16 : 8];  // Q4_K: bsum per 32 (pairs of bsum16); Q6_K: bsum per 16
    float d;
};

// load superblock s of a q8 plane row (global or shared: qs 16-byte aligned)
template <bool KQ6>
__device__ __forceinline__ void load_act(ActReg<KQ6> &a, const int8_t *qs, const int16_t *bsum, float d) {
#pragma unroll
    for (int i = 0; i < 16; ++i) {
        const int4 v = *(const int4 *) (qs + 16 * i);
        a.q[4 * i + 0] = v.x; a.q[4 * i + 1] = v.y; a.q[4 * i + 2] = v.z; a.q[4 * i + 3] = v.w;
    }
    if (KQ6) {
#pragma unroll
        for (int i = 0; i < 16; ++i) a.bs[i] = bsum[i];
    } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) a.bs[i] = (int) bsum[2 * i] + (int) bsum[2 * i + 1];
    }
    a.d = d;
}

// Q4_K superblock (144 B, 16-byte aligned in shared memory) . activation superblock
// (ggml-cpu/quants.c:696-768): d_w*d_a*sum_j sc_j*isum_j - dmin_w*d_a*sum_j m_j*bsum32_j
__device__ __forceinline__ float dot_q4K_sb(const uint8_t *sb, const ActReg<false> &a) {
    const uint4 h = *(const uint4 *) sb;
    const float dw = h2f((uint16_t) h.x), dmw = h2f((uint16_t) (h.x >> 16));
    // the 12 packed 6-bit scales/mins -> 8 scales (s0, s1) and 8 mins (m0, m1), one byte
    // each (same unpacking as get_scale_min_k4, ggml-quants.c:880-887)
    const uint32_t s0 = h.y & 0x3f3f3f3fu;
    const uint32_t m0 = h.z & 0x3f3f3f3fu;
    const uint32_t s1 = (h.w & 0x0f0f0f0fu) | (((h.y >> 6) & 0x03030303u) << 4);
    const uint32_t m1 = ((h.w >> 4) & 0x0f0f0f0fu) | (((h.z >> 6) & 0x03030303u) << 4);
    int isum = 0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const uint4 w0 = *(const uint4 *) (sb + 16 + 32 * g);
        const uint4 w1 = *(const uint4 *) (sb + 16 + 32 * g + 16);
        const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        int il = 0, ih = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            il = dp4a_us(w[i] & 0x0f0f0f0fu, a.q[16 * g + i], il);
            ih = dp4a_us(w[i] & 0xf0f0f0f0u, a.q[16 * g + 8 + i], ih);  // 16 * hi nibbles
        }
        const uint32_t sw = g < 2 ? s0 : s1;
        const int sc_lo = (sw >> (16 * (g & 1))) & 0xff, sc_hi = (sw >> (16 * (g & 1) + 8)) & 0xff;
        isum += sc_lo * il + sc_hi * (ih >> 4);
    }
    int imin = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) imin += (int) (((j < 4 ? m0 : m1) >> (8 * (j & 3))) & 0xff) * a.bs[j];
    return __fmul_rn(dw, a.d) * (float) isum - __fmul_rn(dmw, a.d) * (float) imin;
}

// 32-bit load from a shared-memory address (volatile: never hoisted above the mbarrier
// wait that makes the bulk-copied bytes visible)
__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// Q6_K superblock (210 B, 2-byte aligned in shared memory) . activation superblock
// (ggml-cpu/quants.c:851-915): d_w*d_a*sum_g sc_g*sum_{16} (q6-32)*q8, with the -32 applied
// through the activation's bsum16.  The superblock is read as aligned 32-bit words and
// realigned with funnel shifts.
struct Q6Words {
    uint32_t b;   // shared address of the first aligned word
    uint32_t sh;  // 0 or 16
    __device__ __forceinline__ uint32_t operator[](int i) const { return lds32(b + 4u * (uint32_t) i); }
};
__device__ __forceinline__ float dot_q6K_sb(const uint8_t *sb, const ActReg<true> &a) {
    const uint32_t sa = smem_u32(sb);
    const Q6Words base{sa & ~3u, (sa & 3u) * 8u};
    const uint32_t sh = base.sh;
    int gacc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) gacc[i] = 0;
#pragma unroll
    for (int n = 0; n < 2; ++n) {
        uint32_t raw[17], hr[9];
#pragma unroll
        for (int i = 0; i < 17; ++i) raw[i] = base[16 * n + i];
#pragma unroll
        for (int i = 0; i < 9; ++i) hr[i] = base[32 + 8 * n + i];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t A = __funnelshift_r(raw[i], raw[i + 1], sh);
            const uint32_t B = __funnelshift_r(raw[8 + i], raw[9 + i], sh);
            const uint32_t Hh = __funnelshift_r(hr[i], hr[i + 1], sh);
            const uint32_t q1 = (A & 0x0f0f0f0fu) | ((Hh << 4) & 0x30303030u);
            const uint32_t q2 = (B & 0x0f0f0f0fu) | ((Hh << 2) & 0x30303030u);
            const uint32_t q3 = ((A >> 4) & 0x0f0f0f0fu) | (Hh & 0x30303030u);
            const uint32_t q4 = ((B >> 4) & 0x0f0f0f0fu) | ((Hh >> 2) & 0x30303030u);
            const int aw = 32 * n + i;  // activation word of weight n*128 + 4i
            gacc[8 * n + 0 + i / 4] = dp4a_us(q1, a.q[aw], gacc[8 * n + 0 + i / 4]);
            gacc[8 * n + 2 + i / 4] = dp4a_us(q2, a.q[aw + 8], gacc[8 * n + 2 + i / 4]);
            gacc[8 * n + 4 + i / 4] = dp4a_us(q3, a.q[aw + 16], gacc[8 * n + 4 + i / 4]);
            gacc[8 * n + 6 + i / 4] = dp4a_us(q4, a.q[aw + 24], gacc[8 * n + 6 + i / 4]);
        }
    }
    uint32_t scw[5];
#pragma unroll
    for (int i = 0; i < 5; ++i) scw[i] = base[48 + i];
    const uint32_t sc0 = __funnelshift_r(scw[0], scw[1], sh), sc1 = __funnelshift_r(scw[1], scw[2], sh);
    const uint32_t sc2 = __funnelshift_r(scw[2], scw[3], sh), sc3 = __funnelshift_r(scw[3], scw[4], sh);
    const uint32_t sc[4] = {sc0, sc1, sc2, sc3};
    const uint32_t dword = __funnelshift_r(scw[4], base[53], sh);
    int isum = 0;
#pragma unroll
    for (int g = 0; g < 16; ++g) {
        const int s = (int) (int8_t) (sc[g >> 2] >> (8 * (g & 3)));
        isum += s * (gacc[g] - 32 * a.bs[g]);
    }
    return __fmul_rn(h2f((uint16_t) dword), a.d) * (float) isum;
}

}  // namespace qwb
