// prefill.cu - MUL_MAT_ID with many tokens per expert as a grouped GEMM on tcgen05.
//
// Semantics are ggml_compute_forward_mul_mat_id (ggml-cpu.c:1474-1736) with the weights'
// vec_dot type Q8_K: dst[:, j, t] = as[:, :, ids[j, t]] . q8K(b[:, j % n_b, t]).  The CPU
// computes each superblock exactly in integers and combines superblocks in f32
// (ggml_vec_dot_q4_K_q8_K: d_a*d_w*sum(sc*isum) - d_a*dmin_w*sum(m*bsum)).  The tensor-core
// formulation keeps that exactness:
//
//   A[m, k] = fp16(sc * q)        (sc <= 63, q <= 15: sc*q <= 945, an exact fp16 integer)
//   B[n, k] = fp16(q8)            (|q8| <= 127, exact)
//   plus 32 extra K positions per superblock for the min term:
//   A[m, 256 + i] = hi / lo fp16 parts of -(dmin/d) * m_{i/2},  B[n, 256 + i] = bsum16[i]
//
// so one f32 TMEM accumulator holds isum - (dmin/d) * sum(m*bsum) for one superblock
// (integer products, exactly accumulated), and the epilogue adds d_w * d_a * acc.
// Superblocks whose dmin/d ratio is too large for an fp16 min coefficient (d ~ 0) use
// dmin as the row scale instead (see pf_row_mode).
//
// Work item = (token tile of one expert, 128 weight rows).  One persistent CTA per SM,
// warp-specialised:
//   warp 0      producer: bulk copies of the raw Q4_K rows and of the fp16 B tiles
//   warp 1      TMEM allocation and the MMA-issuing thread
//   warps 4-7   dequantisation of the raw rows into TMEM (A operand), one row per thread
//   warps 8-15  epilogue: TMEM accumulator -> registers, per-superblock scale, store
// Every wait is bounded; a timeout sets QWB_DEVERR_TIMEOUT and all roles drain and exit.
#include "prefill.cuh"

#include <algorithm>

#include "kernels.cuh"
#include "umma.cuh"

namespace qwb {

// K position p (0..127) of the fp16 B/A tiles inside half h of a superblock -> element
// index in the superblock.  The order is the one the dequantiser produces from Q4_K's
// nibble packing (four 32-bit words -> 16 columns of packed pairs), and the gather kernel
// places the activation values in the same order.
__host__ __device__ inline int pf_elem_of_pos(int h, int p) {
    const int col = p >> 1, t = p & 1;
    const int jj = col >> 5, w = (col & 31) >> 2, kind = col & 3;
    return 64 * (2 * h + jj) + 32 * (kind >> 1) + 4 * w + (kind & 1) + 2 * t;
}

// ------------------------------------------------------------------ gather
// grid (max_tiles, K/256), 256 threads: one superblock of one token tile.
constexpr int kGatherRow = 260;  // smem row stride in bytes (65 words: conflict-free 4-byte reads)

__global__ void __launch_bounds__(256) pf_gather_kernel(Q8Planes act, int64_t K, const int4 *__restrict__ tiles,
                                                        const int *__restrict__ n_tiles,
                                                        const int *__restrict__ pairs, int n_used, int n_b,
                                                        uint8_t *__restrict__ btiles, float *__restrict__ da) {
    const int tile = blockIdx.x;
    if (tile >= *n_tiles) return;
    const int s = blockIdx.y;
    const int nsb = (int) (K / QK_K);
    const int4 tl = tiles[tile];
    const int cnt = tl.z, Nt = (cnt + 15) & ~15;
    __shared__ __align__(16) uint8_t q[kPfTileN * kGatherRow];
    __shared__ __align__(16) int16_t bs[kPfTileN][16];
    const int tid = threadIdx.x;
    const int64_t dstride = plane_d_stride(K, QK_K), bstride = plane_bsum_stride(K);

    // load the tile's rows (quantized values of superblock s, block sums, scale)
    for (int c = tid; c < Nt * 16; c += 256) {
        const int n = c >> 4, v = c & 15;
        uint4 x = make_uint4(0, 0, 0, 0);
        if (n < cnt) {
            const int p = pairs[tl.y + n];
            const int t = p / n_used, j = p - t * n_used;
            const int64_t r = (int64_t) t * n_b + (j % n_b);
            x = *(const uint4 *) (act.qs + r * K + (int64_t) s * QK_K + 16 * v);
        }
        uint32_t *d = (uint32_t *) (q + n * kGatherRow + 16 * v);
        d[0] = x.x; d[1] = x.y; d[2] = x.z; d[3] = x.w;
    }
    for (int c = tid; c < Nt * 2; c += 256) {
        const int n = c >> 1, v = c & 1;
        uint4 x = make_uint4(0, 0, 0, 0);
        if (n < cnt) {
            const int p = pairs[tl.y + n];
            const int t = p / n_used, j = p - t * n_used;
            const int64_t r = (int64_t) t * n_b + (j % n_b);
            x = *(const uint4 *) (act.bsum + r * bstride + (int64_t) s * 16 + 8 * v);
        }
        *(uint4 *) &bs[n][8 * v] = x;
    }
    for (int n = tid; n < kPfTileN; n += 256) {
        float v = 0.f;
        if (n < cnt) {
            const int p = pairs[tl.y + n];
            const int t = p / n_used, j = p - t * n_used;
            const int64_t r = (int64_t) t * n_b + (j % n_b);
            v = act.d[r * dstride + s];
        }
        da[((size_t) tile * nsb + s) * kPfTileN + n] = v;
    }
    __syncthreads();

    // write both half-superblock stages in the core-matrix layout:
    // element (n, p) at (p / 8) * Nt * 16 + n * 16 + (p % 8) * 2
    uint8_t *tb = btiles + (size_t) tile * pf_btile_stride(K) + (size_t) (2 * s) * Nt * kPfHalfK * 2;
    const int chunks = 2 * 18 * Nt;
    for (int c = tid; c < chunks; c += 256) {
        const int n = c % Nt, rest = c / Nt;
        const int pc = rest % 18, h = rest / 18;
        uint32_t o[4];
        if (pc < 16) {
            // positions 8pc..8pc+7 = columns 4pc..4pc+3: elements base+4w+{0,2,1,3} and
            // base+32+4w+{0,2,1,3} with w = pc % 8, base = 64 * (2h + pc / 8)
            const int base = 64 * (2 * h + (pc >> 3)) + 4 * (pc & 7);
            const uint32_t wa = *(const uint32_t *) (q + n * kGatherRow + base);
            const uint32_t wb = *(const uint32_t *) (q + n * kGatherRow + base + 32);
            auto cvt = [](uint32_t w, int byte) -> uint32_t {
                return (uint32_t) __half_as_ushort(__int2half_rn((int) (int8_t) (w >> (8 * byte))));
            };
            o[0] = cvt(wa, 0) | (cvt(wa, 2) << 16);
            o[1] = cvt(wa, 1) | (cvt(wa, 3) << 16);
            o[2] = cvt(wb, 0) | (cvt(wb, 2) << 16);
            o[3] = cvt(wb, 1) | (cvt(wb, 3) << 16);
        } else {
            const int i0 = 8 * (pc - 16);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t lo = __half_as_ushort(__int2half_rn((int) bs[n][i0 + 2 * i]));
                const uint32_t hi = __half_as_ushort(__int2half_rn((int) bs[n][i0 + 2 * i + 1]));
                o[i] = lo | (hi << 16);
            }
        }
        *(uint4 *) (tb + (size_t) h * Nt * kPfHalfK * 2 + (size_t) pc * Nt * 16 + (size_t) n * 16) =
            make_uint4(o[0], o[1], o[2], o[3]);
    }
}

cudaError_t launch_pf_gather(Q8Planes act, int64_t K, const int4 *tiles, const int *n_tiles, int max_tiles,
                             const int *pairs, int n_used, int n_b, uint8_t *btiles, float *da, cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    dim3 grid((unsigned) max_tiles, (unsigned) (K / QK_K));
    pf_gather_kernel<<<grid, 256, 0, s>>>(act, K, tiles, n_tiles, pairs, n_used, n_b, btiles, da);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ GEMM
constexpr int kPfThreads = 512;
constexpr int kPfRawStages = 2, kPfBStages = 4, kPfAStages = 3;
constexpr int kPfRawBytes = kPfTileM * Q4K_BYTES;      // 18432
constexpr int kPfBBytes = kPfTileN * kPfHalfK * 2;     // 36864
constexpr uint32_t kPfACols = 72;                      // 64 value columns + 8 min columns
constexpr uint32_t kPfAccCols = 128;
constexpr uint32_t kPfTmemCols = 512;                  // [0,256) accumulators, [256,472) A stages
constexpr int kPfOffB = kPfRawStages * kPfRawBytes;
constexpr int kPfOffBar = kPfOffB + kPfBStages * kPfBBytes;
constexpr int kPfSmem = kPfOffBar + 256;

struct PfBars {
    uint64_t raw_full[kPfRawStages], raw_empty[kPfRawStages];
    uint64_t b_full[kPfBStages], b_empty[kPfBStages];
    uint64_t a_full[kPfAStages], a_empty[kPfAStages];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t drain;
    uint32_t tmem;
    int abort;
};
static_assert(sizeof(PfBars) <= 256, "barrier block");

__device__ __forceinline__ bool pf_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                        qwb_status_block *st) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
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

struct PfItem {
    int tile, mt, p0, cnt, Nt, rows;
    int64_t slot;  // -1: invalid expert id / slot
};
__device__ __forceinline__ PfItem pf_item(const PrefillArgs &a, int it) {
    PfItem x;
    x.tile = it / a.m_tiles;
    x.mt = it - x.tile * a.m_tiles;
    const int4 t = a.tiles[x.tile];
    x.p0 = t.y;
    x.cnt = t.z;
    x.Nt = (t.z + 15) & ~15;
    x.rows = (int) min((int64_t) kPfTileM, a.M - (int64_t) x.mt * kPfTileM);
    x.slot = -1;
    if (t.x >= 0 && t.x < a.n_ids) {
        const int64_t sl = a.remap ? (int64_t) a.remap[t.x] : (int64_t) t.x;
        if (sl >= 0 && sl < a.n_slots) x.slot = sl;
    }
    return x;
}

// Row scale mode of one Q4_K superblock.  0: S = d, min coefficient -(dmin/d)*m (|dmin/d|
// <= 1000 keeps it inside fp16); 1: S = dmin, values scaled by d/dmin, min coefficient -m;
// 2: S = 0 (d = dmin = 0).
__device__ __forceinline__ int pf_row_mode(float d, float dmin) {
    if (d != 0.f && fabsf(dmin) <= 1000.f * fabsf(d)) return 0;
    if (dmin != 0.f) return 1;
    return 2;
}
__device__ __forceinline__ float pf_row_scale(float d, float dmin) {
    const int mode = pf_row_mode(d, dmin);
    return mode == 0 ? d : (mode == 1 ? dmin : 0.f);
}

__device__ __forceinline__ uint32_t hfma2_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ uint32_t hmul2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
__device__ __forceinline__ uint32_t h2_splat(float v) {
    const uint32_t h = f2h_rn(v);
    return h | (h << 16);
}

__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm_q4k_kernel(const PrefillArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *raw = smem;
    uint8_t *bst = smem + kPfOffB;
    PfBars *bars = (PfBars *) (smem + kPfOffBar);
    volatile int *abort = &bars->abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int total = *a.n_tiles * a.m_tiles;
    if ((int) blockIdx.x >= total) return;
    const int nsb = (int) (a.K / QK_K);

    if (tid == 0) {
        for (int i = 0; i < kPfRawStages; ++i) {
            mbar_init(&bars->raw_full[i], 1);
            mbar_init(&bars->raw_empty[i], 128);
        }
        for (int i = 0; i < kPfBStages; ++i) {
            mbar_init(&bars->b_full[i], 1);
            mbar_init(&bars->b_empty[i], 1);
        }
        for (int i = 0; i < kPfAStages; ++i) {
            mbar_init(&bars->a_full[i], 128);
            mbar_init(&bars->a_empty[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&bars->acc_full[i], 1);
            mbar_init(&bars->acc_empty[i], 256);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        umma::tmem_alloc(&bars->tmem, kPfTmemCols);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tbase = bars->tmem;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        uint32_t ra_i = 0, b_i = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
            const PfItem x = pf_item(a, it);
            if (x.slot < 0 && lane == 0 && x.mt == 0) report(a.st, QWB_DEVERR_ID_RANGE, a.tiles[x.tile].x);
            const uint8_t *wb = x.slot >= 0 ? a.W + (size_t) x.slot * a.nb2 + (size_t) x.mt * kPfTileM * a.nb1 : nullptr;
            const uint8_t *bt = a.btiles + (size_t) x.tile * pf_btile_stride(a.K);
            const uint32_t bbytes = (uint32_t) x.Nt * kPfHalfK * 2;
            for (int s = 0; s < nsb && ok; ++s) {
                const int ra = ra_i % kPfRawStages;
                if (!(ok = pf_wait_warp(&bars->raw_empty[ra], ((ra_i / kPfRawStages) & 1) ^ 1, abort, a.st))) break;
                if (lane == 0) mbar_arrive_expect_tx(&bars->raw_full[ra], wb ? (uint32_t) x.rows * Q4K_BYTES : 0u);
                __syncwarp();
                if (wb)
                    for (int r = lane; r < x.rows; r += 32)
                        bulk_g2s(raw + ra * kPfRawBytes + r * Q4K_BYTES, wb + (size_t) r * a.nb1 + (size_t) s * Q4K_BYTES,
                                 Q4K_BYTES, &bars->raw_full[ra]);
                ++ra_i;
                for (int h = 0; h < 2; ++h) {
                    const int bs = b_i % kPfBStages;
                    if (!(ok = pf_wait_warp(&bars->b_empty[bs], ((b_i / kPfBStages) & 1) ^ 1, abort, a.st))) break;
                    if (lane == 0) {
                        mbar_arrive_expect_tx(&bars->b_full[bs], bbytes);
                        bulk_g2s(bst + bs * kPfBBytes, bt + (size_t) (2 * s + h) * bbytes, bbytes, &bars->b_full[bs]);
                    }
                    ++b_i;
                }
            }
        }
        // wait for this warp's copies still in flight (only after an abort can there be any)
        if (lane == 0) {
            for (int k = 0; k < kPfRawStages; ++k)
                if (ra_i > (uint32_t) k) {
                    const uint32_t last = ra_i - 1 - ((ra_i - 1 - k) % kPfRawStages);
                    mbar_wait(&bars->raw_full[k], (last / kPfRawStages) & 1);
                }
            for (int k = 0; k < kPfBStages; ++k)
                if (b_i > (uint32_t) k) {
                    const uint32_t last = b_i - 1 - ((b_i - 1 - k) % kPfBStages);
                    mbar_wait(&bars->b_full[k], (last / kPfBStages) & 1);
                }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t b_i = 0, a_i = 0, acc_i = 0;
            bool ok = true;
            for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
                const PfItem x = pf_item(a, it);
                const uint32_t idesc = umma::idesc_f16(kPfTileM, x.Nt);
                const uint32_t lbo = (uint32_t) x.Nt * 16;
                for (int s = 0; s < nsb && ok; ++s) {
                    const int ab = acc_i & 1;
                    if (!(ok = pf_wait(&bars->acc_empty[ab], ((acc_i >> 1) & 1) ^ 1, abort, a.st))) break;
                    umma::fence_after_sync();
                    const uint32_t d_t = tbase + (uint32_t) ab * kPfAccCols;
                    for (int h = 0; h < 2; ++h) {
                        const int bs = b_i % kPfBStages, as = a_i % kPfAStages;
                        if (!(ok = pf_wait(&bars->b_full[bs], (b_i / kPfBStages) & 1, abort, a.st))) break;
                        if (!(ok = pf_wait(&bars->a_full[as], (a_i / kPfAStages) & 1, abort, a.st))) break;
                        umma::fence_after_sync();
                        const uint32_t b_s = smem_u32(bst + bs * kPfBBytes);
                        const uint32_t a_t = tbase + 2 * kPfAccCols + (uint32_t) as * kPfACols;
#pragma unroll
                        for (int ks = 0; ks < 8; ++ks)
                            umma::mma_f16_ts(d_t, a_t + ks * 8, umma::sdesc(b_s + ks * 2 * lbo, lbo, 128), idesc,
                                             (h | ks) != 0);
                        umma::mma_f16_ts(d_t, a_t + 64, umma::sdesc(b_s + 16 * lbo, lbo, 128), idesc, 1u);
                        umma::commit(&bars->b_empty[bs]);
                        umma::commit(&bars->a_empty[as]);
                        ++b_i;
                        ++a_i;
                    }
                    if (!ok) break;
                    umma::commit(&bars->acc_full[ab]);
                    ++acc_i;
                }
            }
            // all MMAs issued by this thread have completed before TMEM is released
            umma::commit(&bars->drain);
            mbar_wait(&bars->drain, 0);
        }
        __syncwarp();
    } else if (warp >= 4 && warp < 8) {
        // ------------------------------------------------------------ dequantiser
        const int qd = warp - 4, m = qd * 32 + lane;
        const uint32_t lane_base = (uint32_t) (qd * 32) << 16;
        uint32_t ra_i = 0, a_i = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
            const PfItem x = pf_item(a, it);
            const bool live = x.slot >= 0 && m < x.rows;
            for (int s = 0; s < nsb && ok; ++s) {
                const int ra = ra_i % kPfRawStages;
                if (!(ok = pf_wait_warp(&bars->raw_full[ra], (ra_i / kPfRawStages) & 1, abort, a.st))) break;
                uint32_t w[36];
                if (live) {
                    const uint4 *src = (const uint4 *) (raw + ra * kPfRawBytes + m * Q4K_BYTES);
#pragma unroll
                    for (int i = 0; i < 9; ++i) {
                        const uint4 v = src[i];
                        w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 36; ++i) w[i] = 0;
                }
                umma::mbar_arrive(&bars->raw_empty[ra]);
                ++ra_i;
                const float d = h2f((uint16_t) (w[0] & 0xFFFF)), dmin = h2f((uint16_t) (w[0] >> 16));
                const int mode = pf_row_mode(d, dmin);
                uint8_t sb[12];
#pragma unroll
                for (int i = 0; i < 12; ++i) sb[i] = (uint8_t) (w[1 + i / 4] >> (8 * (i % 4)));
                int sc[8], mn[8];
#pragma unroll
                for (int j = 0; j < 8; ++j) {
                    if (j < 4) {
                        sc[j] = sb[j] & 63;
                        mn[j] = sb[j + 4] & 63;
                    } else {
                        sc[j] = (sb[j + 4] & 0xF) | ((sb[j - 4] >> 6) << 4);
                        mn[j] = (sb[j + 4] >> 4) | ((sb[j] >> 6) << 4);
                    }
                }
                const float r = mode == 0 ? dmin / d : (mode == 1 ? d / dmin : 0.f);
                const uint32_t k2 = mode == 1 ? h2_splat(r) : 0u;
                for (int h = 0; h < 2 && ok; ++h) {
                    const int as = a_i % kPfAStages;
                    if (!(ok = pf_wait_warp(&bars->a_empty[as], ((a_i / kPfAStages) & 1) ^ 1, abort, a.st))) break;
                    umma::fence_after_sync();
                    const uint32_t a_t = tbase + lane_base + 2 * kPfAccCols + (uint32_t) as * kPfACols;
#pragma unroll
                    for (int jj = 0; jj < 2; ++jj) {
                        const int j = 2 * h + jj;
                        const uint32_t slo = h2_splat((float) sc[2 * j]), blo = h2_splat(-1024.f * (float) sc[2 * j]);
                        const uint32_t shi = h2_splat((float) sc[2 * j + 1]),
                                       bhi = h2_splat(-1024.f * (float) sc[2 * j + 1]);
#pragma unroll
                        for (int g = 0; g < 2; ++g) {
                            uint32_t o[16];
#pragma unroll
                            for (int ww = 0; ww < 4; ++ww) {
                                const uint32_t xw = w[4 + 8 * j + 4 * g + ww];
                                o[4 * ww + 0] = hfma2_u((xw & 0x000F000Fu) | 0x64006400u, slo, blo);
                                o[4 * ww + 1] = hfma2_u(((xw >> 8) & 0x000F000Fu) | 0x64006400u, slo, blo);
                                o[4 * ww + 2] = hfma2_u(((xw >> 4) & 0x000F000Fu) | 0x64006400u, shi, bhi);
                                o[4 * ww + 3] = hfma2_u(((xw >> 12) & 0x000F000Fu) | 0x64006400u, shi, bhi);
                            }
                            if (mode != 0) {
#pragma unroll
                                for (int i = 0; i < 16; ++i) o[i] = hmul2_u(o[i], k2);
                            }
                            umma::st16(a_t + (uint32_t) (jj * 32 + g * 16), o);
                        }
                    }
                    uint32_t o8[8];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        float hi = 0.f, lo = 0.f;
                        if (mode == 0) {
                            const float v = -r * (float) mn[c];
                            hi = __half2float(__float2half_rn(v));
                            lo = v - hi;
                        } else if (mode == 1) {
                            hi = -(float) mn[c];
                        }
                        o8[c] = h2_splat(h == 0 ? hi : lo);
                    }
                    umma::st8(a_t + 64, o8);
                    umma::wait_st();
                    umma::fence_before_sync();
                    umma::mbar_arrive(&bars->a_full[as]);
                    ++a_i;
                }
            }
        }
    } else if (warp >= 8) {
        // ------------------------------------------------------------ epilogue
        const int qd = warp & 3, g = (warp - 8) >> 2, m = qd * 32 + lane;
        const uint32_t lane_base = (uint32_t) (qd * 32) << 16;
        uint32_t acc_i = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
            const PfItem x = pf_item(a, it);
            const bool live = x.slot >= 0 && m < x.rows;
            const uint8_t *hdr =
                live ? a.W + (size_t) x.slot * a.nb2 + ((size_t) x.mt * kPfTileM + m) * a.nb1 : nullptr;
            const float *dap = a.da + (size_t) x.tile * nsb * kPfTileN + 64 * g;
            float out[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) out[i] = 0.f;
            for (int s = 0; s < nsb && ok; ++s) {
                float S = 0.f;
                if (hdr) {
                    const uint32_t hw = __ldg((const unsigned int *) (hdr + (size_t) s * Q4K_BYTES));
                    S = pf_row_scale(h2f((uint16_t) (hw & 0xFFFF)), h2f((uint16_t) (hw >> 16)));
                }
                const int ab = acc_i & 1;
                if (!(ok = pf_wait_warp(&bars->acc_full[ab], (acc_i >> 1) & 1, abort, a.st))) break;
                umma::fence_after_sync();
                const uint32_t d_t = tbase + lane_base + (uint32_t) ab * kPfAccCols + 64 * g;
                const float *ds = dap + (size_t) s * kPfTileN;
#pragma unroll
                for (int c = 0; c < 4; ++c) {
                    if (64 * g + 16 * c < x.Nt) {  // warp-uniform
                        uint32_t v[16];
                        umma::ld16(d_t + 16 * c, v);
                        umma::wait_ld();
#pragma unroll
                        for (int i = 0; i < 16; i += 4) {
                            const float4 dv = __ldg((const float4 *) (ds + 16 * c + i));
                            out[16 * c + i + 0] = fmaf(S * dv.x, __uint_as_float(v[i + 0]), out[16 * c + i + 0]);
                            out[16 * c + i + 1] = fmaf(S * dv.y, __uint_as_float(v[i + 1]), out[16 * c + i + 1]);
                            out[16 * c + i + 2] = fmaf(S * dv.z, __uint_as_float(v[i + 2]), out[16 * c + i + 2]);
                            out[16 * c + i + 3] = fmaf(S * dv.w, __uint_as_float(v[i + 3]), out[16 * c + i + 3]);
                        }
                    }
                }
                umma::fence_before_sync();
                umma::mbar_arrive(&bars->acc_empty[ab]);
                ++acc_i;
            }
            if (!ok) break;
            if (m < x.rows) {
                const int64_t row = (int64_t) x.mt * kPfTileM + m;
#pragma unroll
                for (int i = 0; i < 64; ++i) {
                    const int n = 64 * g + i;
                    if (n < x.cnt) {
                        const int p = __ldg(a.pairs + x.p0 + n);
                        const int t = p / a.n_used, j = p - t * a.n_used;
                        float *o = (float *) ((char *) a.dst + (size_t) j * a.dnb1 + (size_t) t * a.dnb2);
                        o[row] = out[i];
                    }
                }
            }
        }
    }

    umma::fence_before_sync();
    __syncthreads();
    if (warp == 1) {
        umma::fence_after_sync();
        umma::tmem_dealloc(tbase, kPfTmemCols);
    }
}

cudaError_t launch_pf_gemm_q4k(const PrefillArgs &a, cudaStream_t s) {
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(pf_gemm_q4k_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfSmem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    pf_gemm_q4k_kernel<<<num_sms(), kPfThreads, kPfSmem, s>>>(a);
    return cudaGetLastError();
}

bool pf_eligible(int type, int64_t K, int64_t M, int64_t P, int64_t n_as) {
    if (type != QWB_TYPE_Q4_K || K % QK_K || K < QK_K || M < 1) return false;
    const int64_t used = std::min<int64_t>(P, n_as);
    return used > 0 && P >= 32 * used;
}

}  // namespace qwb
