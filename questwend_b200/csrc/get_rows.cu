// get_rows.cu - GGML_OP_GET_ROWS for the embedding table and the expert-slot remap.
//
// Semantics (ggml.c:3975-3996, CPU ggml-cpu/ops.cpp:5204-5240 get_rows_q and :5371):
//   src0 [ne0, ne01, ne02, ne03], idx [n, ne11 = ne02, ne12 = ne03] I32,
//   dst  [ne0, n, ne11, ne12]:  dst[:, i10, i11, i12] = row(src0[:, idx[i10,i11,i12], i11, i12])
// Quantized rows are dequantized with the reference's formulas (ggml-quants.c:1530-1552
// Q4_K, :1940-1969 Q6_K, :553 Q8_0).  Each output is bit-identical to the CPU's: the
// products d*sc*q (Q4_K/Q6_K) and d*q (Q8_0) are exact in fp32, so only Q4_K's final
// subtraction rounds, once, in both implementations; F16 widening and F32/I32 copies are
// exact.  Ids outside [0, ne01) produce a zero row and a QWB_DEVERR_ROW_RANGE record
// (the CPU backend asserts).
#include "common.cuh"
#include "kernels.cuh"

namespace qwb {

struct GetRowsArgs {
    const uint8_t *src;
    size_t nb01, nb02, nb03;
    int64_t ne0, ne01;
    const uint8_t *idx;
    size_t ib0, ib1, ib2;  // idx strides (bytes)
    int64_t n, ne11, ne12;
    uint8_t *dst;
    size_t db1, db2, db3;
    qwb_status_block *st;
};

// 8 consecutive outputs starting at p (p % 8 == 0) of a quantized / F16 / F32 row
template <int TYPE>
__device__ __forceinline__ void dequant8(const uint8_t *row, int64_t p, float out[8]) {
    if (TYPE == QWB_TYPE_Q4_K) {
        const uint8_t *sb = row + (p >> 8) * Q4K_BYTES;
        const int w = (int) (p & 255), g = w >> 6, hi = (w >> 5) & 1, l = w & 31;
        const uint32_t dm = *(const uint32_t *) sb;
        const float d = h2f((uint16_t) dm), dmin = h2f((uint16_t) (dm >> 16));
        uint8_t sc8[12];
        *(uint32_t *) &sc8[0] = *(const uint32_t *) (sb + 4);
        *(uint32_t *) &sc8[4] = *(const uint32_t *) (sb + 8);
        *(uint32_t *) &sc8[8] = *(const uint32_t *) (sb + 12);
        int sc, m;
        q4k_scale_min(2 * g + hi, sc8, sc, m);
        const float d1 = __fmul_rn(d, (float) sc), m1 = __fmul_rn(dmin, (float) m);
        const uint32_t q0 = *(const uint32_t *) (sb + 16 + 32 * g + l);
        const uint32_t q1 = *(const uint32_t *) (sb + 16 + 32 * g + l + 4);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int a = (int) ((q0 >> (8 * i + 4 * hi)) & 0xF), b = (int) ((q1 >> (8 * i + 4 * hi)) & 0xF);
            out[i] = __fsub_rn(__fmul_rn(d1, (float) a), m1);
            out[4 + i] = __fsub_rn(__fmul_rn(d1, (float) b), m1);
        }
    } else if (TYPE == QWB_TYPE_Q6_K) {
        const uint8_t *sb = row + (p >> 8) * Q6K_BYTES;
        const int w = (int) (p & 255), n = w >> 7, t = w & 127, grp = t >> 5, l = t & 31;
        const uint8_t *ql = sb + 64 * n + ((grp & 1) ? 32 : 0) + l;
        const uint8_t *qh = sb + 128 + 32 * n + l;
        const int sc = (int) (int8_t) sb[192 + 8 * n + (l >> 4) + 2 * grp];
        const float d = h2f(*(const uint16_t *) (sb + 208));
        const float dsc = __fmul_rn(d, (float) sc);
        const uint32_t qlw0 = (uint32_t) lds_u32_a2(ql), qlw1 = (uint32_t) lds_u32_a2(ql + 4);
        const uint32_t qhw0 = (uint32_t) lds_u32_a2(qh), qhw1 = (uint32_t) lds_u32_a2(qh + 4);
        const int lsh = grp >= 2 ? 4 : 0, hsh = 2 * grp;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const int a = (int) (((qlw0 >> (8 * i + lsh)) & 0xF) | (((qhw0 >> (8 * i + hsh)) & 3) << 4)) - 32;
            const int b = (int) (((qlw1 >> (8 * i + lsh)) & 0xF) | (((qhw1 >> (8 * i + hsh)) & 3) << 4)) - 32;
            out[i] = __fmul_rn(dsc, (float) a);
            out[4 + i] = __fmul_rn(dsc, (float) b);
        }
    } else if (TYPE == QWB_TYPE_Q8_0) {
        const uint8_t *b = row + (p >> 5) * Q80_BYTES;
        const int o = (int) (p & 31);
        const float d = h2f(*(const uint16_t *) b);
        const uint32_t w0 = (uint32_t) lds_u32_a2(b + 2 + o), w1 = (uint32_t) lds_u32_a2(b + 2 + o + 4);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            out[i] = __fmul_rn((float) (int8_t) (w0 >> (8 * i)), d);
            out[4 + i] = __fmul_rn((float) (int8_t) (w1 >> (8 * i)), d);
        }
    } else if (TYPE == QWB_TYPE_F16) {
        const uint16_t *h = (const uint16_t *) row + p;
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = h2f(h[i]);
    } else {  // F32 / I32: raw 32-bit words
        const uint32_t *f = (const uint32_t *) row + p;
#pragma unroll
        for (int i = 0; i < 8; ++i) out[i] = __uint_as_float(f[i]);
    }
}

// one CTA per output row, 8 outputs per thread per step (ne0 % 8 == 0)
template <int TYPE>
__global__ void __launch_bounds__(128) get_rows_vec_kernel(GetRowsArgs a) {
    const int64_t r = blockIdx.x;  // flattened (i10, i11, i12)
    const int64_t i10 = r % a.n, i11 = (r / a.n) % a.ne11, i12 = r / (a.n * a.ne11);
    const int32_t i01 = *(const int32_t *) (a.idx + i10 * a.ib0 + i11 * a.ib1 + i12 * a.ib2);
    float *drow = (float *) (a.dst + i10 * a.db1 + i11 * a.db2 + i12 * a.db3);
    if (i01 < 0 || i01 >= a.ne01) {
        if (threadIdx.x == 0) report(a.st, QWB_DEVERR_ROW_RANGE, i01);
        for (int64_t p = 8 * threadIdx.x; p < a.ne0; p += 8 * blockDim.x) {
            *(float4 *) (drow + p) = make_float4(0.f, 0.f, 0.f, 0.f);
            *(float4 *) (drow + p + 4) = make_float4(0.f, 0.f, 0.f, 0.f);
        }
        return;
    }
    const uint8_t *row = a.src + (size_t) i01 * a.nb01 + i11 * a.nb02 + i12 * a.nb03;
    for (int64_t p = 8 * threadIdx.x; p < a.ne0; p += 8 * blockDim.x) {
        float v[8];
        dequant8<TYPE>(row, p, v);
        *(float4 *) (drow + p) = make_float4(v[0], v[1], v[2], v[3]);
        *(float4 *) (drow + p + 4) = make_float4(v[4], v[5], v[6], v[7]);
    }
}

// any ne0, F32 / I32 / F16 sources: one thread per output element (covers the I32
// [1, n_expert] slot tables of the in-graph remap)
__global__ void get_rows_elem_kernel(GetRowsArgs a, int type, int64_t total) {
    const int64_t e = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (e >= total) return;
    const int64_t c = e % a.ne0, r = e / a.ne0;
    const int64_t i10 = r % a.n, i11 = (r / a.n) % a.ne11, i12 = r / (a.n * a.ne11);
    const int32_t i01 = *(const int32_t *) (a.idx + i10 * a.ib0 + i11 * a.ib1 + i12 * a.ib2);
    uint32_t *d = (uint32_t *) (a.dst + i10 * a.db1 + i11 * a.db2 + i12 * a.db3) + c;
    if (i01 < 0 || i01 >= a.ne01) {
        if (c == 0) report(a.st, QWB_DEVERR_ROW_RANGE, i01);
        *d = 0u;
        return;
    }
    const uint8_t *row = a.src + (size_t) i01 * a.nb01 + i11 * a.nb02 + i12 * a.nb03;
    if (type == QWB_TYPE_F16) *d = __float_as_uint(h2f(((const uint16_t *) row)[c]));
    else *d = ((const uint32_t *) row)[c];
}

}  // namespace qwb

using namespace qwb;

extern "C" QWB_API qwb_status qwb_get_rows(const qwb_tensor *src0, const qwb_tensor *idx, const qwb_tensor *dst,
                                           qwb_status_block *d_status, qwb_stream_t stream) {
    if (!src0 || !idx || !dst) return QWB_ERR_INVALID_ARG;
    const int t = src0->type;
    if (t != QWB_TYPE_Q4_K && t != QWB_TYPE_Q6_K && t != QWB_TYPE_Q8_0 && t != QWB_TYPE_F16 && t != QWB_TYPE_F32 &&
        t != QWB_TYPE_I32)
        return QWB_ERR_UNSUPPORTED_TYPE;
    if (idx->type != QWB_TYPE_I32) return QWB_ERR_UNSUPPORTED_TYPE;
    if (dst->type != (t == QWB_TYPE_I32 ? QWB_TYPE_I32 : QWB_TYPE_F32)) return QWB_ERR_UNSUPPORTED_TYPE;
    for (int i = 0; i < 4; ++i)
        if (src0->ne[i] < 0 || idx->ne[i] < 0 || dst->ne[i] < 0) return QWB_ERR_INVALID_ARG;
    if (src0->ne[2] != idx->ne[1] || src0->ne[3] != idx->ne[2] || idx->ne[3] != 1) return QWB_ERR_SHAPE;
    if (dst->ne[0] != src0->ne[0] || dst->ne[1] != idx->ne[0] || dst->ne[2] != idx->ne[1] ||
        dst->ne[3] != idx->ne[2])
        return QWB_ERR_SHAPE;
    const int64_t ne0 = src0->ne[0];
    const int blk = block_elems(t);
    if (ne0 % blk) return QWB_ERR_SHAPE;
    const int64_t nrows_out = idx->ne[0] * idx->ne[1] * idx->ne[2];
    if (nrows_out == 0 || ne0 == 0) return QWB_OK;
    if (!src0->data || !idx->data || !dst->data) return QWB_ERR_INVALID_ARG;
    if (dst->nb[0] != 4) return QWB_ERR_LAYOUT;
    const size_t esz = t == QWB_TYPE_F16 ? 2 : (blk == 1 ? 4 : 0);
    if (esz && src0->nb[0] != esz) return QWB_ERR_LAYOUT;
    if (!esz && src0->nb[0] != row_bytes(t, blk)) return QWB_ERR_LAYOUT;
    if (idx->nb[0] % 4 || (uintptr_t) idx->data % 4) return QWB_ERR_ALIGNMENT;

    GetRowsArgs a;
    a.src = (const uint8_t *) src0->data;
    a.nb01 = src0->nb[1]; a.nb02 = src0->nb[2]; a.nb03 = src0->nb[3];
    a.ne0 = ne0; a.ne01 = src0->ne[1];
    a.idx = (const uint8_t *) idx->data;
    a.ib0 = idx->nb[0]; a.ib1 = idx->nb[1]; a.ib2 = idx->nb[2];
    a.n = idx->ne[0]; a.ne11 = idx->ne[1]; a.ne12 = idx->ne[2];
    a.dst = (uint8_t *) dst->data;
    a.db1 = dst->nb[1]; a.db2 = dst->nb[2]; a.db3 = dst->nb[3];
    a.st = d_status;
    cudaStream_t s = (cudaStream_t) stream;

    const uintptr_t salign = (uintptr_t) src0->data | src0->nb[1] | src0->nb[2] | src0->nb[3];
    const uintptr_t dalign = (uintptr_t) dst->data | dst->nb[1] | dst->nb[2] | dst->nb[3];
    const bool vec = ne0 % 8 == 0 && dalign % 16 == 0 &&
                     ((t == QWB_TYPE_Q4_K && salign % 4 == 0) || (t == QWB_TYPE_Q6_K && salign % 2 == 0) ||
                      (t == QWB_TYPE_Q8_0 && salign % 2 == 0) || (t == QWB_TYPE_F16 && salign % 2 == 0) ||
                      ((t == QWB_TYPE_F32 || t == QWB_TYPE_I32) && salign % 4 == 0));
    if (!vec) {
        if (blk != 1) return QWB_ERR_ALIGNMENT;  // quantized rows need the vector path
        if (salign % esz || dalign % 4) return QWB_ERR_ALIGNMENT;
        const int64_t total = nrows_out * ne0;
        get_rows_elem_kernel<<<(unsigned) ceil_div(total, 256), 256, 0, s>>>(a, t, total);
        return cudaGetLastError() == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
    }
    if (nrows_out > 0x7fffffff) return QWB_ERR_LIMIT;
    const unsigned grid = (unsigned) nrows_out;
    switch (t) {
        case QWB_TYPE_Q4_K: get_rows_vec_kernel<QWB_TYPE_Q4_K><<<grid, 128, 0, s>>>(a); break;
        case QWB_TYPE_Q6_K: get_rows_vec_kernel<QWB_TYPE_Q6_K><<<grid, 128, 0, s>>>(a); break;
        case QWB_TYPE_Q8_0: get_rows_vec_kernel<QWB_TYPE_Q8_0><<<grid, 128, 0, s>>>(a); break;
        case QWB_TYPE_F16: get_rows_vec_kernel<QWB_TYPE_F16><<<grid, 128, 0, s>>>(a); break;
        default: get_rows_vec_kernel<QWB_TYPE_F32><<<grid, 128, 0, s>>>(a); break;
    }
    return cudaGetLastError() == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
}
