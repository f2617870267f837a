// quant_dev.cuh - warp-level activation quantizers (device functions), bit-exact with
// the reference CPU backend's from_float; see quantize.cu for the exactness argument.
#pragma once

#include "common.cuh"
#include "kernels.cuh"

namespace qwb {

// Lane `lane`'s 8 consecutive inputs x[8*lane .. 8*lane+8).  With a norm weight nw the
// values are first RMS-normalised exactly as ggml's fused rms_norm * weight on the CPU
// (ggml-cpu/ops.cpp:4161: y = x * scale * w, two rounded products).
__device__ __forceinline__ void load8_normed(const float *x, float nscale, const float *nw, int lane, float v[8]) {
    const float4 a = *(const float4 *) (x + 8 * lane);
    const float4 b = *(const float4 *) (x + 8 * lane + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
    if (nw) {
        const float4 c = *(const float4 *) (nw + 8 * lane);
        const float4 e = *(const float4 *) (nw + 8 * lane + 4);
        const float w[8] = {c.x, c.y, c.z, c.w, e.x, e.y, e.z, e.w};
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], nscale), w[i]);
    }
}

// One warp quantizes one 256-value Q8_K block; lane l owns values [8l, 8l+8).
// Outputs (any may be null): packed block_q8_K, or plane qs/d/bsum.
__device__ __forceinline__ void q8K_block_vals(const float v[8], uint8_t *packed, int8_t *pqs, float *pd,
                                               int16_t *pbsum);
__device__ __forceinline__ void q8K_block_warp(const float *x, uint8_t *packed, int8_t *pqs, float *pd,
                                               int16_t *pbsum, float nscale = 1.f, const float *nw = nullptr) {
    float v[8];
    load8_normed(x, nscale, nw, threadIdx.x & 31, v);
    q8K_block_vals(v, packed, pqs, pd, pbsum);
}
// Same, on values already loaded: lane l holds values [8l, 8l+8) of the block.
__device__ __forceinline__ void q8K_block_vals(const float v[8], uint8_t *packed, int8_t *pqs, float *pd,
                                               int16_t *pbsum) {
    const int lane = threadIdx.x & 31;
    // local first-max of |x|
    float lam = 0.f, lmx = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float ax = fabsf(v[i]);
        if (ax > lam) { lam = ax; lmx = v[i]; }
    }
    float amax = lam;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    // lowest lane holding amax (values within a lane are in index order, so its local
    // first-max is the global first-max)
    const unsigned hit = __ballot_sync(0xffffffffu, lam == amax && amax > 0.f);
    const int src = hit ? __ffs(hit) - 1 : 0;
    const float mx = __shfl_sync(0xffffffffu, lmx, src);

    int q[8];
    float d = 0.f;
    if (amax == 0.f) {
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = 0;
    } else {
        const float iscale = __fdiv_rn(-127.f, mx);
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = min(127, __float2int_rn(__fmul_rn(iscale, v[i])));
        d = __fdiv_rn(1.f, iscale);
    }
    int s = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) s += q[i];
    s += __shfl_xor_sync(0xffffffffu, s, 1);  // lanes 2g, 2g+1 cover bsum group g
    const uint32_t w0 = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((uint32_t) (q[3] & 0xff) << 24);
    const uint32_t w1 = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((uint32_t) (q[7] & 0xff) << 24);
    if (packed) {
        uint32_t *qw = (uint32_t *) (packed + 4 + 8 * lane);
        qw[0] = w0;
        qw[1] = w1;
        if ((lane & 1) == 0) *(int16_t *) (packed + 4 + 256 + lane) = (int16_t) s;
        if (lane == 0) *(float *) packed = d;
    }
    if (pqs) *(uint2 *) (pqs + 8 * lane) = make_uint2(w0, w1);
    if (pbsum && (lane & 1) == 0) pbsum[lane >> 1] = (int16_t) s;
    if (pd && lane == 0) *pd = d;
}

// One warp quantizes 8 Q8_0 blocks (256 values); lane l owns values [8l, 8l+8) of block l/4.
__device__ __forceinline__ void q80_8blocks_warp(const float *x, int variant, uint8_t *packed, int8_t *pqs,
                                                 float *pd, float nscale = 1.f, const float *nw = nullptr) {
    const int lane = threadIdx.x & 31;
    float v[8];
    load8_normed(x, nscale, nw, lane, v);
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(v[i]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
    const float d = __fdiv_rn(amax, 127.f);
    const uint16_t dh = f2h_rn(d);
    int q[8];
    if (variant == QWB_Q8_0_REF) {
        const float id = d != 0.f ? __fdiv_rn(1.f, d) : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = (int) roundf(__fmul_rn(v[i], id));
    } else {
        const float id = amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) q[i] = __float2int_rn(__fmul_rn(v[i], id));
    }
    const uint32_t w0 = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((uint32_t) (q[3] & 0xff) << 24);
    const uint32_t w1 = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((uint32_t) (q[7] & 0xff) << 24);
    const int blk = lane >> 2, sub = lane & 3;
    if (packed) {
        uint8_t *b = packed + Q80_BYTES * blk;
        uint16_t *qh = (uint16_t *) (b + 2 + 8 * sub);
        qh[0] = (uint16_t) w0; qh[1] = (uint16_t) (w0 >> 16);
        qh[2] = (uint16_t) w1; qh[3] = (uint16_t) (w1 >> 16);
        if (sub == 0) *(uint16_t *) b = dh;
    }
    if (pqs) *(uint2 *) (pqs + 8 * lane) = make_uint2(w0, w1);
    if (pd && sub == 0) pd[blk] = h2f(dh);
}

// Quantize one 256-value chunk (row r, columns [c0, c0+256) of a row of length K) of
// f32 activations at x into q8 planes.  kind: 0 = Q8_K, 1 = Q8_0 cpu, 2 = Q8_0 ref.
__device__ __forceinline__ void quantize_chunk_warp(int kind, const float *x, const Q8Planes &pl, int64_t r,
                                                    int64_t c0, int64_t K, float nscale = 1.f,
                                                    const float *nw = nullptr) {
    if (kind == 0) {
        q8K_block_warp(x, nullptr, pl.qs + r * K + c0, pl.d + r * plane_d_stride(K, QK_K) + c0 / QK_K,
                       pl.bsum + r * plane_bsum_stride(K) + c0 / 16, nscale, nw);
    } else {
        q80_8blocks_warp(x, kind == 2 ? QWB_Q8_0_REF : QWB_Q8_0_CPU, nullptr, pl.qs + r * K + c0,
                         pl.d + r * plane_d_stride(K, QK8_0) + c0 / QK8_0, nscale, nw);
    }
}

}  // namespace qwb
