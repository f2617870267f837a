// dot.cuh - quantized weight-row x Q8 activation dot products, one "unit" (32 weights)
// at a time, reading weights and activations from shared memory.
//
// Arithmetic follows the reference CPU dots exactly up to the final float summation:
//   Q4_K x Q8_K  ggml-cpu/quants.c:696-768   sum_sb d_w*d_a*sum(sc*isum) - dmin_w*d_a*sum(m*bsum)
//   Q6_K x Q8_K  ggml-cpu/quants.c:851-915   sum_sb d_w*d_a*sum(sc*isum), q6 - 32 signed
//   Q8_0 x Q8_0  ggml-cpu/quants.c:451-480   sum_b isum*(d_w*d_a)
// Integer sub-block sums are exact (dp4a); the per-unit float products and the final
// sum over units are fp32 in a different order than the CPU's, which is the only source
// of difference (~1e-7 relative).
#pragma once

#include "common.cuh"

namespace qwb {

// Activation rows staged in shared memory: token k at base + k*stride:
//   qs int8[K] | d float[dstride] | bsum int16[bstride]
struct ActSmem {
    const uint8_t *base;
    int stride;   // bytes per token
    int d_off;    // byte offset of d within a token
    int b_off;    // byte offset of bsum within a token
    __device__ __forceinline__ const int8_t *qs(int k) const { return (const int8_t *) (base + k * stride); }
    __device__ __forceinline__ const float *d(int k) const { return (const float *) (base + k * stride + d_off); }
    __device__ __forceinline__ const int16_t *bsum(int k) const { return (const int16_t *) (base + k * stride + b_off); }
};

// Q4_K unit u (superblock s = u/8, qs chunk c = u%8): 16 qs bytes = 16 low nibbles of
// sub-block 2g and 16 high nibbles of sub-block 2g+1 (g = c/2), positions
// 64g + 16(c&1) + [0,16) and +32.  Row base must be 4-byte aligned.
template <int NT>
__device__ __forceinline__ void unit_q4K(const uint8_t *row, int u, const ActSmem &A, int cnt, float *acc) {
    const int s = u >> 3, c = u & 7, g = c >> 1, h = c & 1;
    const uint8_t *sb = row + s * Q4K_BYTES;
    const uint32_t dm = *(const uint32_t *) sb;
    const float dw = h2f((uint16_t) dm), dmw = h2f((uint16_t) (dm >> 16));
    uint8_t sc8[12];
    *(uint32_t *) &sc8[0] = *(const uint32_t *) (sb + 4);
    *(uint32_t *) &sc8[4] = *(const uint32_t *) (sb + 8);
    *(uint32_t *) &sc8[8] = *(const uint32_t *) (sb + 12);
    int sc_lo, m_lo, sc_hi, m_hi;
    q4k_scale_min(2 * g, sc8, sc_lo, m_lo);
    q4k_scale_min(2 * g + 1, sc8, sc_hi, m_hi);
    const uint4 q = *(const uint4 *) (sb + 16 + 16 * c);
    const int l0 = (int) (q.x & 0x0f0f0f0fu), l1 = (int) (q.y & 0x0f0f0f0fu);
    const int l2 = (int) (q.z & 0x0f0f0f0fu), l3 = (int) (q.w & 0x0f0f0f0fu);
    const int h0 = (int) ((q.x >> 4) & 0x0f0f0f0fu), h1 = (int) ((q.y >> 4) & 0x0f0f0f0fu);
    const int h2 = (int) ((q.z >> 4) & 0x0f0f0f0fu), h3 = (int) ((q.w >> 4) & 0x0f0f0f0fu);
    const int apos = s * QK_K + 64 * g + 16 * h;
    const int bpos = s * 16 + 4 * g + h;
#pragma unroll
    for (int k = 0; k < NT; ++k) {
        if (k < cnt) {
            const int4 al = *(const int4 *) (A.qs(k) + apos);
            const int4 ah = *(const int4 *) (A.qs(k) + apos + 32);
            int il = __dp4a(l0, al.x, 0);
            il = __dp4a(l1, al.y, il);
            il = __dp4a(l2, al.z, il);
            il = __dp4a(l3, al.w, il);
            int ih = __dp4a(h0, ah.x, 0);
            ih = __dp4a(h1, ah.y, ih);
            ih = __dp4a(h2, ah.z, ih);
            ih = __dp4a(h3, ah.w, ih);
            const int16_t *bs = A.bsum(k);
            const int isc = sc_lo * il + sc_hi * ih;
            const int imn = m_lo * (int) bs[bpos] + m_hi * (int) bs[bpos + 2];
            const float da = A.d(k)[s];
            acc[k] += __fmul_rn(dw, da) * (float) isc - __fmul_rn(dmw, da) * (float) imn;
        }
    }
}

// Q6_K unit u (superblock s = u/8, half hf = (u%8)/4, l-quarter q = u%4, l0 = 8q):
// weights at hf*128 + l0 + [0,8) + {0, 32, 64, 96}.  Row base must be 2-byte aligned.
template <int NT>
__device__ __forceinline__ void unit_q6K(const uint8_t *row, int u, const ActSmem &A, int cnt, float *acc) {
    const int s = u >> 3, v = u & 7, hf = v >> 2, l0 = 8 * (v & 3);
    const uint8_t *sb = row + s * Q6K_BYTES;
    const uint8_t *qla = sb + 64 * hf + l0, *qlb = qla + 32, *qh = sb + 128 + 32 * hf + l0;
    const int8_t *scp = (const int8_t *) (sb + 192) + 8 * hf + (l0 >> 4);
    const int sc0 = scp[0], sc1 = scp[2], sc2 = scp[4], sc3 = scp[6];
    const float dw = h2f(*(const uint16_t *) (sb + 208));
    int w[4][2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const uint32_t a = (uint32_t) lds_u32_a2(qla + 4 * i), b = (uint32_t) lds_u32_a2(qlb + 4 * i);
        const uint32_t hb = (uint32_t) lds_u32_a2(qh + 4 * i);
        w[0][i] = (int) __vsub4((a & 0x0f0f0f0fu) | ((hb << 4) & 0x30303030u), 0x20202020u);
        w[1][i] = (int) __vsub4((b & 0x0f0f0f0fu) | ((hb << 2) & 0x30303030u), 0x20202020u);
        w[2][i] = (int) __vsub4(((a >> 4) & 0x0f0f0f0fu) | (hb & 0x30303030u), 0x20202020u);
        w[3][i] = (int) __vsub4(((b >> 4) & 0x0f0f0f0fu) | ((hb >> 2) & 0x30303030u), 0x20202020u);
    }
    const int apos = s * QK_K + 128 * hf + l0;
#pragma unroll
    for (int k = 0; k < NT; ++k) {
        if (k < cnt) {
            const int8_t *aq = A.qs(k) + apos;
            const int2 a0 = *(const int2 *) (aq), a1 = *(const int2 *) (aq + 32);
            const int2 a2 = *(const int2 *) (aq + 64), a3 = *(const int2 *) (aq + 96);
            const int i0 = __dp4a(w[0][1], a0.y, __dp4a(w[0][0], a0.x, 0));
            const int i1 = __dp4a(w[1][1], a1.y, __dp4a(w[1][0], a1.x, 0));
            const int i2 = __dp4a(w[2][1], a2.y, __dp4a(w[2][0], a2.x, 0));
            const int i3 = __dp4a(w[3][1], a3.y, __dp4a(w[3][0], a3.x, 0));
            const int isum = sc0 * i0 + sc1 * i1 + sc2 * i2 + sc3 * i3;
            acc[k] += __fmul_rn(dw, A.d(k)[s]) * (float) isum;
        }
    }
}

// Q8_0 unit u = block u (34 bytes: fp16 d, 32 int8).  Row base must be 2-byte aligned.
template <int NT>
__device__ __forceinline__ void unit_q80(const uint8_t *row, int u, const ActSmem &A, int cnt, float *acc) {
    const uint8_t *b = row + u * Q80_BYTES;
    const float dw = h2f(*(const uint16_t *) b);
    int w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = lds_u32_a2(b + 2 + 4 * i);
#pragma unroll
    for (int k = 0; k < NT; ++k) {
        if (k < cnt) {
            const int4 a0 = *(const int4 *) (A.qs(k) + 32 * u);
            const int4 a1 = *(const int4 *) (A.qs(k) + 32 * u + 16);
            int is = __dp4a(w[0], a0.x, 0);
            is = __dp4a(w[1], a0.y, is);
            is = __dp4a(w[2], a0.z, is);
            is = __dp4a(w[3], a0.w, is);
            is = __dp4a(w[4], a1.x, is);
            is = __dp4a(w[5], a1.y, is);
            is = __dp4a(w[6], a1.z, is);
            is = __dp4a(w[7], a1.w, is);
            acc[k] += (float) is * __fmul_rn(dw, A.d(k)[u]);
        }
    }
}

template <int TYPE, int NT>
__device__ __forceinline__ void unit_dot(const uint8_t *row, int u, const ActSmem &A, int cnt, float *acc) {
    if (TYPE == QWB_TYPE_Q4_K) unit_q4K<NT>(row, u, A, cnt, acc);
    else if (TYPE == QWB_TYPE_Q6_K) unit_q6K<NT>(row, u, A, cnt, acc);
    else unit_q80<NT>(row, u, A, cnt, acc);
}

// silu(g) * u as ggml_vec_swiglu_f32 (vec.cpp:417-447): g / (1 + exp(-g)) * u
__device__ __forceinline__ float swiglu1(float g, float u) { return g / (1.0f + expf(-g)) * u; }

}  // namespace qwb
