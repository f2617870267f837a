// dot.cuh - quantized weight-row x Q8 activation dot products, one "unit" (32 weights)
// at a time, reading weights from shared memory and activations either from shared
// memory (ActSmem) or in place from the q8 planes in global memory (ActRows).
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
    __device__ __forceinline__ const int8_t *sbq(int k, int s) const { return qs(k) + s * QK_K; }
    __device__ __forceinline__ const int16_t *sbb(int k, int s) const { return bsum(k) + s * 16; }
    __device__ __forceinline__ float sbd(int k, int s) const { return d(k)[s]; }
    __device__ __forceinline__ const int8_t *blk(int k, int u) const { return qs(k) + 32 * u; }
    __device__ __forceinline__ float bd(int k, int u) const { return d(k)[u]; }
};

// Activation rows staged in shared memory with bank padding: each group of `upq` 32-byte
// blocks of qs (a Q8_K superblock, or four Q8_0 blocks) is followed by 16 spare bytes,
// and each superblock's 16 bsums by 16 spare bytes, so lanes reading consecutive groups
// hit different banks.  Token k at base + k*stride; d plane at d_off, bsum plane at b_off.
struct ActStage {
    const uint8_t *base;
    int stride, d_off, b_off;
    int upq_shift;  // log2(blocks per qs group): 3 (Q8_K), 2 (Q8_0)
    __device__ __forceinline__ const int8_t *blk(int k, int u) const {
        const int gsz = (32 << upq_shift) + 16;
        return (const int8_t *) (base + k * stride + (u >> upq_shift) * gsz + (u & ((1 << upq_shift) - 1)) * 32);
    }
    __device__ __forceinline__ const int8_t *sbq(int k, int s) const {
        return (const int8_t *) (base + k * stride + s * (QK_K + 16));
    }
    __device__ __forceinline__ const int16_t *sbb(int k, int s) const {
        return (const int16_t *) (base + k * stride + b_off + s * 48);
    }
    __device__ __forceinline__ float sbd(int k, int s) const { return ((const float *) (base + k * stride + d_off))[s]; }
    __device__ __forceinline__ float bd(int k, int u) const { return ((const float *) (base + k * stride + d_off))[u]; }
};

// Activation rows read in place from the q8 planes (global memory, cached in L1): token k
// of the current group is plane row ar[k].
struct ActRows {
    const int8_t *qs_;
    const float *d_;
    const int16_t *b_;
    int64_t K;
    int dstride, bstride;
    int ar[8];
    __device__ __forceinline__ const int8_t *qs(int k) const { return qs_ + (int64_t) ar[k] * K; }
    __device__ __forceinline__ const float *d(int k) const { return d_ + (int64_t) ar[k] * dstride; }
    __device__ __forceinline__ const int16_t *bsum(int k) const { return b_ + (int64_t) ar[k] * bstride; }
    __device__ __forceinline__ const int8_t *sbq(int k, int s) const { return qs(k) + s * QK_K; }
    __device__ __forceinline__ const int16_t *sbb(int k, int s) const { return bsum(k) + s * 16; }
    __device__ __forceinline__ float sbd(int k, int s) const { return d(k)[s]; }
    __device__ __forceinline__ const int8_t *blk(int k, int u) const { return qs(k) + 32 * u; }
    __device__ __forceinline__ float bd(int k, int u) const { return d(k)[u]; }
};

// Q4_K unit u (superblock s = u/8, qs chunk c = u%8): 16 qs bytes = 16 low nibbles of
// sub-block 2g and 16 high nibbles of sub-block 2g+1 (g = c/2), positions
// 64g + 16(c&1) + [0,16) and +32.  Row base must be 4-byte aligned.
template <int NT, class Act>
__device__ __forceinline__ void unit_q4K(const uint8_t *row, int u, const Act &A, int cnt, float *acc) {
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
template <int NT, class Act>
__device__ __forceinline__ void unit_q6K(const uint8_t *row, int u, const Act &A, int cnt, float *acc) {
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
template <int NT, class Act>
__device__ __forceinline__ void unit_q80(const uint8_t *row, int u, const Act &A, int cnt, float *acc) {
    const uint8_t *b = row + u * Q80_BYTES;
    const float dw = h2f(*(const uint16_t *) b);
    int w[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = lds_u32_a2(b + 2 + 4 * i);
#pragma unroll
    for (int k = 0; k < NT; ++k) {
        if (k < cnt) {
            const int4 a0 = *(const int4 *) A.blk(k, u);
            const int4 a1 = *(const int4 *) (A.blk(k, u) + 16);
            int is = __dp4a(w[0], a0.x, 0);
            is = __dp4a(w[1], a0.y, is);
            is = __dp4a(w[2], a0.z, is);
            is = __dp4a(w[3], a0.w, is);
            is = __dp4a(w[4], a1.x, is);
            is = __dp4a(w[5], a1.y, is);
            is = __dp4a(w[6], a1.z, is);
            is = __dp4a(w[7], a1.w, is);
            acc[k] += (float) is * __fmul_rn(dw, A.bd(k, u));
        }
    }
}

// ---------------------------------------------------------------- superblock dots
// One whole superblock s of a weight row against up to NT activation rows, with the
// superblock's scales decoded once and each 64- (Q4_K) or 32-element (Q6_K) slice of
// weights unpacked once for all tokens.  Same integer sums as the unit dots; the fp32
// combine is one term per superblock, as in the reference CPU dots.

// 32 bytes at a 2-byte aligned shared-memory address as 8 little-endian words
// (4-byte aligned loads, funnel-shifted when the address is 2 mod 4)
__device__ __forceinline__ void lds_words8_a2(const uint8_t *p, uint32_t *w) {
    const uint32_t *q = (const uint32_t *) ((uintptr_t) p & ~(uintptr_t) 3);
    const uint32_t sh = (uint32_t) ((uintptr_t) p & 3) * 8u;
    uint32_t x[9];
#pragma unroll
    for (int i = 0; i < 9; ++i) x[i] = (i < 8 || sh) ? q[i] : 0u;
#pragma unroll
    for (int i = 0; i < 8; ++i) w[i] = __funnelshift_r(x[i], x[i + 1], sh);
}

// Q4_K superblock (144 bytes, 16-byte aligned): ggml-cpu/quants.c q4_K x q8_K.
// isum = sum_j sc_j * (q . a)_j, summ = sum_j m_j * bsum_j over the 8 sub-blocks of 32,
// acc += d_w*d_a*isum - dmin_w*d_a*summ.
template <int NT, class Act>
__device__ __forceinline__ void sb_q4K(const uint8_t *sb, int s, const Act &A, int cnt, float *acc) {
    const uint4 h = *(const uint4 *) sb;  // d, dmin | 12 packed scale bytes
    const float dw = h2f((uint16_t) h.x), dmw = h2f((uint16_t) (h.x >> 16));
    // get_scale_min_k4 (ggml-quants.c:880-887) on four bytes at once
    const uint32_t sc_lo = h.y & 0x3f3f3f3fu, m_lo = h.z & 0x3f3f3f3fu;
    const uint32_t sc_hi = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t m_hi = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u);
    int isum[NT];
#pragma unroll
    for (int k = 0; k < NT; ++k) isum[k] = 0;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
        const uint32_t scw = g < 2 ? sc_lo : sc_hi;
        const int sa = (int) ((scw >> (16 * (g & 1))) & 0xffu), sbh = (int) ((scw >> (16 * (g & 1) + 8)) & 0xffu);
        const uint4 q0 = *(const uint4 *) (sb + 16 + 32 * g), q1 = *(const uint4 *) (sb + 32 + 32 * g);
        const uint32_t qw[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        int lo[8], hi[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            lo[i] = (int) (qw[i] & 0x0f0f0f0fu);
            hi[i] = (int) ((qw[i] >> 4) & 0x0f0f0f0fu);
        }
#pragma unroll
        for (int k = 0; k < NT; ++k) {
            if (k < cnt) {
                const int8_t *aq = A.sbq(k, s) + 64 * g;
                const int4 a0 = *(const int4 *) aq, a1 = *(const int4 *) (aq + 16);
                const int4 a2 = *(const int4 *) (aq + 32), a3 = *(const int4 *) (aq + 48);
                int il = __dp4a(lo[0], a0.x, 0);
                il = __dp4a(lo[1], a0.y, il);
                il = __dp4a(lo[2], a0.z, il);
                il = __dp4a(lo[3], a0.w, il);
                il = __dp4a(lo[4], a1.x, il);
                il = __dp4a(lo[5], a1.y, il);
                il = __dp4a(lo[6], a1.z, il);
                il = __dp4a(lo[7], a1.w, il);
                int ih = __dp4a(hi[0], a2.x, 0);
                ih = __dp4a(hi[1], a2.y, ih);
                ih = __dp4a(hi[2], a2.z, ih);
                ih = __dp4a(hi[3], a2.w, ih);
                ih = __dp4a(hi[4], a3.x, ih);
                ih = __dp4a(hi[5], a3.y, ih);
                ih = __dp4a(hi[6], a3.z, ih);
                ih = __dp4a(hi[7], a3.w, ih);
                isum[k] += sa * il + sbh * ih;
            }
        }
    }
#pragma unroll
    for (int k = 0; k < NT; ++k) {
        if (k < cnt) {
            const int4 b0 = *(const int4 *) A.sbb(k, s), b1 = *(const int4 *) (A.sbb(k, s) + 8);
            const int bw[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
            int summ = 0;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                // bsum of sub-block j = the two int16 sums of its halves
                const int pair = (int) (int16_t) (bw[j] & 0xffff) + (bw[j] >> 16);
                const uint32_t mw = j < 4 ? m_lo : m_hi;
                summ += (int) ((mw >> (8 * (j & 3))) & 0xffu) * pair;
            }
            const float da = A.sbd(k, s);
            acc[k] += __fmul_rn(dw, da) * (float) isum[k] - __fmul_rn(dmw, da) * (float) summ;
        }
    }
}

// Q6_K superblock (210 bytes, 2-byte aligned): ggml-cpu/quants.c q6_K x q8_K.
// Element 128*hf + 32*i + l has ql nibble (ql[64hf + 32(i&1) + l], high nibble when i >= 2)
// and qh bits 2i..2i+1 of qh[32hf + l]; scale sc[8hf + 2i + l/16]; isum = sum sc*(q6-32).a.
template <int NT, class Act>
__device__ __forceinline__ void sb_q6K(const uint8_t *sb, int s, const Act &A, int cnt, float *acc) {
    const float dw = h2f(*(const uint16_t *) (sb + 208));
    int isum[NT];
#pragma unroll
    for (int k = 0; k < NT; ++k) isum[k] = 0;
#pragma unroll
    for (int hf = 0; hf < 2; ++hf) {
        uint32_t qa[8], qb[8], qh[8];
        lds_words8_a2(sb + 64 * hf, qa);
        lds_words8_a2(sb + 64 * hf + 32, qb);
        lds_words8_a2(sb + 128 + 32 * hf, qh);
        const int8_t *scp = (const int8_t *) (sb + 192) + 8 * hf;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            int w[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const uint32_t ql = (i & 1) ? qb[m] : qa[m];
                const uint32_t nib = i < 2 ? (ql & 0x0f0f0f0fu) : ((ql >> 4) & 0x0f0f0f0fu);
                const uint32_t hb = ((qh[m] >> (2 * i)) & 0x03030303u) << 4;
                w[m] = (int) __vsub4(nib | hb, 0x20202020u);
            }
            const int s0 = scp[2 * i], s1 = scp[2 * i + 1];
#pragma unroll
            for (int k = 0; k < NT; ++k) {
                if (k < cnt) {
                    const int8_t *aq = A.sbq(k, s) + 128 * hf + 32 * i;
                    const int4 a0 = *(const int4 *) aq, a1 = *(const int4 *) (aq + 16);
                    int i0 = __dp4a(w[0], a0.x, 0);
                    i0 = __dp4a(w[1], a0.y, i0);
                    i0 = __dp4a(w[2], a0.z, i0);
                    i0 = __dp4a(w[3], a0.w, i0);
                    int i1 = __dp4a(w[4], a1.x, 0);
                    i1 = __dp4a(w[5], a1.y, i1);
                    i1 = __dp4a(w[6], a1.z, i1);
                    i1 = __dp4a(w[7], a1.w, i1);
                    isum[k] += s0 * i0 + s1 * i1;
                }
            }
        }
    }
#pragma unroll
    for (int k = 0; k < NT; ++k)
        if (k < cnt) acc[k] += __fmul_rn(dw, A.sbd(k, s)) * (float) isum[k];
}

template <int TYPE, int NT, class Act>
__device__ __forceinline__ void unit_dot(const uint8_t *row, int u, const Act &A, int cnt, float *acc) {
    if constexpr (TYPE == QWB_TYPE_Q4_K) unit_q4K<NT>(row, u, A, cnt, acc);
    else if constexpr (TYPE == QWB_TYPE_Q6_K) unit_q6K<NT>(row, u, A, cnt, acc);
    else unit_q80<NT>(row, u, A, cnt, acc);
}

// silu(g) * u as ggml_vec_swiglu_f32 (vec.cpp:417-447): g / (1 + exp(-g)) * u
__device__ __forceinline__ float swiglu1(float g, float u) { return g / (1.0f + expf(-g)) * u; }

}  // namespace qwb
