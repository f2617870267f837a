// quantize.cu - activation quantizers, bit-exact with the reference CPU backend.
//
//   Q8_K : quantize_row_q8_K_ref (ggml-quants.c:2769-2806), which is what the x86 CPU
//          backend's quantize_row_q8_K calls (ggml-cpu/arch/x86/quants.c:505).
//   Q8_0 : the x86 CPU backend's quantize_row_q8_0 (ggml-cpu/arch/x86/quants.c:302-360),
//          or quantize_row_q8_0_ref (ggml-quants.c:276-300) on request.
//
// Exactness: every float operation the reference performs is reproduced with an IEEE
// round-to-nearest intrinsic (no contraction into FMA): the reciprocal scales are IEEE
// divisions, x*iscale one rounded multiply, nearest_int() == cvt.rni (ties to even, as the
// reference's 1.5*2^23 trick for |v| < 2^22), the fp16 scale a cvt.rn.f16.f32.
// The first index holding the largest |x| wins ties, as in the reference's strict '>' scan.
//
// Two output layouts: ggml's packed blocks (the public entry points) and the split "q8
// planes" the MoE kernels consume (same bytes, separately aligned).
#include "common.cuh"
#include "kernels.cuh"
#include "quant_dev.cuh"

namespace qwb {

// One warp per 256-value chunk; warps are numbered row-major over (row, chunk).
template <int KIND>  // 0 = Q8_K, 1 = Q8_0 cpu, 2 = Q8_0 ref
__global__ void quantize_rows_kernel(const float *__restrict__ x, int64_t x_stride, int64_t n_rows, int64_t K,
                                     uint8_t *__restrict__ packed, Q8Planes pl, const int32_t *row_map) {
    const int64_t gw = ((int64_t) blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t nck = K / 256;
    const int64_t r = gw / nck, c = gw - r * nck;
    if (r >= n_rows) return;
    const int64_t src_row = row_map ? row_map[r] : r;
    const float *xr = x + src_row * x_stride + c * 256;
    if (KIND == 0) {
        uint8_t *pk = packed ? packed + (r * (K / QK_K) + c) * Q8K_BYTES : nullptr;
        int8_t *pqs = pl.qs ? pl.qs + r * K + c * 256 : nullptr;
        float *pd = pl.d ? pl.d + r * plane_d_stride(K, QK_K) + c : nullptr;
        int16_t *pb = pl.bsum ? pl.bsum + r * plane_bsum_stride(K) + c * 16 : nullptr;
        q8K_block_warp(xr, pk, pqs, pd, pb);
    } else {
        uint8_t *pk = packed ? packed + (r * (K / QK8_0) + c * 8) * Q80_BYTES : nullptr;
        int8_t *pqs = pl.qs ? pl.qs + r * K + c * 256 : nullptr;
        float *pd = pl.d ? pl.d + r * plane_d_stride(K, QK8_0) + c * 8 : nullptr;
        q80_8blocks_warp(xr, KIND == 2 ? QWB_Q8_0_REF : QWB_Q8_0_CPU, pk, pqs, pd);
    }
}

// Q8_0 rows whose length is not a multiple of 256: one thread per 32-block (rare: only
// used when K % 256 != 0).
__global__ void quantize_q80_tail_kernel(const float *__restrict__ x, int64_t x_stride, int64_t n_rows, int64_t K,
                                         int variant, uint8_t *__restrict__ packed, Q8Planes pl,
                                         const int32_t *row_map) {
    const int64_t nb = K / QK8_0;
    const int64_t gi = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t r = gi / nb, b = gi - r * nb;
    if (r >= n_rows) return;
    const int64_t src_row = row_map ? row_map[r] : r;
    const float *xr = x + src_row * x_stride + b * QK8_0;
    float amax = 0.f;
    for (int i = 0; i < QK8_0; ++i) amax = fmaxf(amax, fabsf(xr[i]));
    const float d = __fdiv_rn(amax, 127.f);
    const uint16_t dh = f2h_rn(d);
    const float id = variant == QWB_Q8_0_REF ? (d != 0.f ? __fdiv_rn(1.f, d) : 0.f)
                                             : (amax != 0.f ? __fdiv_rn(127.f, amax) : 0.f);
    uint8_t *pk = packed ? packed + (r * nb + b) * Q80_BYTES : nullptr;
    for (int i = 0; i < QK8_0; ++i) {
        const float t = __fmul_rn(xr[i], id);
        const int q = variant == QWB_Q8_0_REF ? (int) roundf(t) : __float2int_rn(t);
        if (pk) pk[2 + i] = (uint8_t) q;
        if (pl.qs) pl.qs[r * K + b * QK8_0 + i] = (int8_t) q;
    }
    if (pk) { pk[0] = (uint8_t) dh; pk[1] = (uint8_t) (dh >> 8); }
    if (pl.d) pl.d[r * plane_d_stride(K, QK8_0) + b] = h2f(dh);
}

cudaError_t launch_quantize_rows(int kind, const float *x, int64_t x_stride, int64_t n_rows, int64_t K,
                                 uint8_t *packed, Q8Planes pl, const int32_t *row_map, cudaStream_t s) {
    if (n_rows == 0 || K == 0) return cudaSuccess;
    if (kind != 0 && K % 256 != 0) {
        const int64_t total = n_rows * (K / QK8_0);
        quantize_q80_tail_kernel<<<(unsigned) ceil_div(total, 128), 128, 0, s>>>(
            x, x_stride, n_rows, K, kind == 2 ? QWB_Q8_0_REF : QWB_Q8_0_CPU, packed, pl, row_map);
        return cudaGetLastError();
    }
    const int warps = 8;
    const unsigned grid = (unsigned) ceil_div(n_rows * (K / 256), warps);
    switch (kind) {
        case 0: quantize_rows_kernel<0><<<grid, warps * 32, 0, s>>>(x, x_stride, n_rows, K, packed, pl, row_map); break;
        case 1: quantize_rows_kernel<1><<<grid, warps * 32, 0, s>>>(x, x_stride, n_rows, K, packed, pl, row_map); break;
        default: quantize_rows_kernel<2><<<grid, warps * 32, 0, s>>>(x, x_stride, n_rows, K, packed, pl, row_map); break;
    }
    return cudaGetLastError();
}

}  // namespace qwb

using namespace qwb;

extern "C" QWB_API qwb_status qwb_quantize_row_q8_K(const float *x, void *y, int64_t n_rows, int64_t k,
                                                    int64_t x_row_stride, qwb_stream_t stream) {
    if (n_rows < 0 || k < 0 || x_row_stride < k) return QWB_ERR_INVALID_ARG;
    if (n_rows == 0 || k == 0) return QWB_OK;
    if (!x || !y) return QWB_ERR_INVALID_ARG;
    if (k % QK_K) return QWB_ERR_SHAPE;
    if (((uintptr_t) x % 16) || (x_row_stride % 4)) return QWB_ERR_ALIGNMENT;
    if ((uintptr_t) y % 4) return QWB_ERR_ALIGNMENT;
    if (n_rows > (1ll << 31) / (k / 32 + 1)) return QWB_ERR_LIMIT;
    Q8Planes none{nullptr, nullptr, nullptr, k};
    return launch_quantize_rows(0, x, x_row_stride, n_rows, k, (uint8_t *) y, none, nullptr, (cudaStream_t) stream)
                   == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
}

extern "C" QWB_API qwb_status qwb_quantize_row_q8_0(const float *x, void *y, int64_t n_rows, int64_t k,
                                                    int64_t x_row_stride, int variant, qwb_stream_t stream) {
    if (n_rows < 0 || k < 0 || x_row_stride < k) return QWB_ERR_INVALID_ARG;
    if (variant != QWB_Q8_0_CPU && variant != QWB_Q8_0_REF) return QWB_ERR_INVALID_ARG;
    if (n_rows == 0 || k == 0) return QWB_OK;
    if (!x || !y) return QWB_ERR_INVALID_ARG;
    if (k % QK8_0) return QWB_ERR_SHAPE;
    if (((uintptr_t) x % 16) || (x_row_stride % 4)) return QWB_ERR_ALIGNMENT;
    if ((uintptr_t) y % 2) return QWB_ERR_ALIGNMENT;
    if (n_rows > (1ll << 31) / (k / 32 + 1)) return QWB_ERR_LIMIT;
    Q8Planes none{nullptr, nullptr, nullptr, k};
    return launch_quantize_rows(variant == QWB_Q8_0_REF ? 2 : 1, x, x_row_stride, n_rows, k, (uint8_t *) y, none,
                                nullptr, (cudaStream_t) stream) == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
}
