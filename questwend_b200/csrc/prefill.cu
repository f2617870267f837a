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
// warp-specialised (18 warps):
//   warps 0-7   dequantisation of the raw rows into TMEM (A operand), one row per thread,
//               one warpgroup per half superblock; each thread fetches its own row bytes
//               with 16-byte async copies (cp.async) several superblocks ahead
//   warps 8-15  epilogue: TMEM accumulator -> per-superblock scale -> running sums -> store
//   warp 16     producer: L2 prefetch of the next item's weight rows; bulk copies of the
//               B stages and the activation scales
//   warp 17     TMEM allocation and the MMA-issuing thread
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
    const int cnt = tl.z, Nt = pf_tile_cols(cnt);
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
// Optional pipeline timestamps (compiled in only with -DQWB_PF_TRACE; no effect on the
// default build): CTA 0 records the global timer per role and per superblock.
#ifdef QWB_PF_TRACE
__device__ unsigned long long g_pf_trace[32][256];
#define PF_TRACE(role, idx)                                                                          \
    do {                                                                                            \
        if (blockIdx.x < 2 && (idx) < 256u) g_pf_trace[(role) + 16 * blockIdx.x][idx] = globaltimer_ns(); \
    } while (0)
#else
#define PF_TRACE(role, idx) \
    do {                    \
    } while (0)
#endif

constexpr int kPfThreads = 576;  // 18 warps
constexpr int kPfBStages = 4, kPfAStages = 3, kPfEpStages = 4;
// raw weight bytes: each dequantiser thread copies (cp.async) its row's 16-byte header and
// the 64 bytes of its half superblock, kPfPre superblocks ahead, into a private slot
constexpr int kPfPre = 3;
constexpr int kPfSlot = 80;
constexpr int kPfRawStage = 256 * kPfSlot;                 // 20480 per superblock
constexpr int kPfBBytes = kPfTileN * kPfHalfK * 2;         // 36864: one half-superblock B stage
constexpr uint32_t kPfACols = 72;                          // 64 value columns + 8 min columns
constexpr uint32_t kPfAccCols = 128;
constexpr uint32_t kPfTmemCols = 512;                      // [0,256) accumulators, [256,472) A stages
constexpr int kPfOffB = kPfPre * kPfRawStage;
// epilogue ring, one slot per superblock: activation scales of the token tile (bulk copy)
// and the weight rows' superblock scales (written by the dequantiser)
constexpr int kPfOffEp = kPfOffB + kPfBStages * kPfBBytes;
constexpr int kPfEpBytes = 2 * kPfTileN * 4;
constexpr int kPfOffBar = kPfOffEp + kPfEpStages * kPfEpBytes;
constexpr int kPfSmem = kPfOffBar + 512;

struct PfBars {
    uint64_t b_full[kPfBStages], b_empty[kPfBStages];
    uint64_t a_full[kPfAStages], a_empty[kPfAStages];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t ep_full[kPfEpStages], ep_empty[kPfEpStages];
    uint64_t drain;
    uint32_t tmem;
    int abort;
};
static_assert(sizeof(PfBars) <= 512, "barrier block");

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
    x.Nt = pf_tile_cols(t.z);
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
__device__ __forceinline__ uint32_t hsub2_u(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
// fp16x2 {v, v} of an integer 0 <= v < 1024 without a conversion instruction: the bits
// 0x6400 | v encode 1024 + v, and subtracting 1024 is exact.
__device__ __forceinline__ uint32_t h2_int(uint32_t v) {
    return hsub2_u((v * 0x10001u) | 0x64006400u, 0x64006400u);
}
// f32 value of an integer 0 <= v < 2^23 without a conversion instruction
__device__ __forceinline__ float f_int(uint32_t v) { return __fsub_rn(__uint_as_float(0x4B000000u | v), 8388608.f); }
// fp16x2 {v, v} (one packed conversion)
__device__ __forceinline__ uint32_t h2_pack(float v) {
    uint32_t d;
    asm("cvt.rn.f16x2.f32 %0, %1, %1;" : "=r"(d) : "f"(v));
    return d;
}
constexpr uint32_t kH2Neg1024 = 0xE400E400u, kH2Sixteenth = 0x2C002C00u, kH2Neg64 = 0xD400D400u;

// 16-byte async copy global -> shared (L2 only); src_bytes 0 zero-fills the destination
__device__ __forceinline__ void cp_async16(void *dst, const void *src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Warp roles (18 warps).  TMEM lane quarter = warp % 4 for every role that touches TMEM.
constexpr int kPfWarpEpi = 8;    // warps 8..15: epilogue (column half (warp - 8) / 4)
constexpr int kPfWarpProd = 16;  // producer
constexpr int kPfWarpMma = 17;   // TMEM allocation + MMA issue
// warps 0..3 / 4..7: dequantiser groups for superblock halves 0 / 1

__global__ void __launch_bounds__(kPfThreads, 1) pf_gemm_q4k_kernel(const PrefillArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    uint8_t *raw = smem;
    uint8_t *bst = smem + kPfOffB;
    float *ep = (float *) (smem + kPfOffEp);  // [slot][0..127] activation scales, [slot][128..255] row scales
    PfBars *bars = (PfBars *) (smem + kPfOffBar);
    volatile int *abort = &bars->abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int total = *a.n_tiles * a.m_tiles;  // work items: (token tile, 128-row weight tile)
    if ((int) blockIdx.x >= total) return;
    const int nsb = (int) (a.K / QK_K);

    if (tid == 0) {
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
        for (int i = 0; i < kPfEpStages; ++i) {
            mbar_init(&bars->ep_full[i], 1 + 128);  // producer (scales copy) + dequantiser group 0
            mbar_init(&bars->ep_empty[i], 256);
        }
        mbar_init(&bars->drain, 1);
        bars->abort = 0;
        fence_mbar_init();
    }
    if (warp == kPfWarpMma) {
        umma::tmem_alloc(&bars->tmem, kPfTmemCols);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tbase = bars->tmem;

    if (warp == kPfWarpProd) {
        // ------------------------------------------------------------ producer
        // Per item, the whole warp first asks L2 to prefetch the NEXT item's weight rows as
        // contiguous row-long runs (one bulk prefetch per row).  Then lane 0 issues, per
        // superblock, the token tile's activation scales and the two B stages (bulk copies).
        const uint32_t rb = (uint32_t) (a.K / QK_K) * Q4K_BYTES;
        auto prefetch_rows = [&](int it) {
            if (it >= total) return;
            const PfItem y = pf_item(a, it);
            if (y.slot < 0) return;
            const uint8_t *base = a.W + (size_t) y.slot * a.nb2 + (size_t) y.mt * kPfTileM * a.nb1;
            for (int r = lane; r < y.rows; r += 32)
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(base + (size_t) r * a.nb1), "r"(rb)
                             : "memory");
        };
        prefetch_rows(blockIdx.x);
        uint32_t b_i = 0, ep_i = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
            prefetch_rows(it + gridDim.x);
            if (lane == 0) {
                const PfItem x = pf_item(a, it);
                if (x.slot < 0 && x.mt == 0) report(a.st, QWB_DEVERR_ID_RANGE, a.tiles[x.tile].x);
                const float *dat = a.da + (size_t) x.tile * nsb * kPfTileN;
                const uint32_t bbytes = (uint32_t) x.Nt * kPfHalfK * 2;
                const uint8_t *bt = a.btiles + (size_t) x.tile * pf_btile_stride(a.K);
                for (int s = 0; s < nsb && ok; ++s) {
                    const int es = ep_i % kPfEpStages;
                    if (!(ok = pf_wait(&bars->ep_empty[es], ((ep_i / kPfEpStages) & 1) ^ 1, abort, a.st))) break;
                    PF_TRACE(0, ep_i);
                    mbar_arrive_expect_tx(&bars->ep_full[es], (uint32_t) x.Nt * 4);
                    bulk_g2s(ep + es * 2 * kPfTileN, dat + (size_t) s * kPfTileN, (uint32_t) x.Nt * 4, &bars->ep_full[es]);
                    ++ep_i;
                    for (int h = 0; h < 2; ++h) {
                        const int bs = b_i % kPfBStages;
                        if (!(ok = pf_wait(&bars->b_empty[bs], ((b_i / kPfBStages) & 1) ^ 1, abort, a.st))) break;
                        mbar_arrive_expect_tx(&bars->b_full[bs], bbytes);
                        bulk_g2s(bst + bs * kPfBBytes, bt + (size_t) (2 * s + h) * bbytes, bbytes, &bars->b_full[bs]);
                        ++b_i;
                    }
                    PF_TRACE(1, ep_i - 1);
                }
            }
            ok = __shfl_sync(0xffffffffu, (int) ok, 0) != 0;
        }
        if (lane == 0) {
            // wait for copies still in flight (only after an abort can there be any)
            for (int k = 0; k < kPfBStages; ++k)
                if (b_i > (uint32_t) k) {
                    const uint32_t last = b_i - 1 - ((b_i - 1 - k) % kPfBStages);
                    mbar_wait(&bars->b_full[k], (last / kPfBStages) & 1);
                }
            for (int k = 0; k < kPfEpStages; ++k)
                if (ep_i > (uint32_t) k) {
                    const uint32_t last = ep_i - 1 - ((ep_i - 1 - k) % kPfEpStages);
                    mbar_wait(&bars->ep_full[k], (last / kPfEpStages) & 1);
                }
        }
        __syncwarp();
    } else if (warp == kPfWarpMma) {
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
                    PF_TRACE(4, acc_i);
                    umma::fence_after_sync();
                    const uint32_t d_t = tbase + (uint32_t) ab * kPfAccCols;
                    for (int h = 0; h < 2; ++h) {
                        const int bs = b_i % kPfBStages, as = a_i % kPfAStages;
                        if (!(ok = pf_wait(&bars->b_full[bs], (b_i / kPfBStages) & 1, abort, a.st))) break;
                        if (h == 0) PF_TRACE(11, acc_i);
                        if (!(ok = pf_wait(&bars->a_full[as], (a_i / kPfAStages) & 1, abort, a.st))) break;
                        PF_TRACE(h == 0 ? 13 : 14, acc_i);
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
                    PF_TRACE(5, acc_i);
                    ++acc_i;
                }
            }
            // all MMAs issued by this thread have completed before TMEM is released
            umma::commit(&bars->drain);
            mbar_wait(&bars->drain, 0);
        }
        __syncwarp();
    } else if (warp < kPfWarpEpi) {
        // ------------------------------------------------------------ dequantisers
        // group grp turns half grp of every superblock (Q4_K chunks 2grp, 2grp+1: 64 bytes
        // of nibbles) into 64 TMEM columns of packed fp16(sc*q) pairs plus 8 min columns
        // (group 0: fp16 high parts of -(dmin/d)*m, group 1: the low parts).
        const int grp = warp >> 2, qd = warp & 3, m = qd * 32 + lane;
        const uint32_t lane_base = (uint32_t) (qd * 32) << 16;
        uint8_t *mine = raw + (size_t) (grp * 128 + m) * kPfSlot;
        // this CTA's superblocks in order: f -> (item f / nsb, superblock f % nsb); the row
        // pointer of the item being fetched is cached (null: invalid slot or row past M)
        const int n_sb = (total - (int) blockIdx.x + (int) gridDim.x - 1) / (int) gridDim.x * nsb;
        int f_item = -1;
        const uint8_t *f_row = nullptr;
        auto fetch = [&](int f) {
            if (f < n_sb) {
                const int k = f / nsb, s = f - k * nsb;
                if (k != f_item) {
                    const PfItem y = pf_item(a, (int) blockIdx.x + k * (int) gridDim.x);
                    f_row = (y.slot >= 0 && m < y.rows)
                                ? a.W + (size_t) y.slot * a.nb2 + ((size_t) y.mt * kPfTileM + m) * a.nb1
                                : nullptr;
                    f_item = k;
                }
                const bool v = f_row != nullptr;
                const uint8_t *src = v ? f_row + (size_t) s * Q4K_BYTES : a.W;
                uint8_t *dst = mine + (f % kPfPre) * kPfRawStage;
                const uint32_t n = v ? 16u : 0u;  // 0: zero-fill
                cp_async16(dst, src, n);
#pragma unroll
                for (int i = 0; i < 4; ++i) cp_async16(dst + 16 + 16 * i, src + 16 + 64 * grp + 16 * i, n);
            }
            cp_async_commit();
        };
#pragma unroll 1
        for (int f = 0; f < kPfPre; ++f) fetch(f);
        uint32_t sb_i = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
            for (int s = 0; s < nsb && ok; ++s, ++sb_i) {
                cp_async_wait<kPfPre - 1>();  // superblock sb_i has landed
                if (tid == 0) PF_TRACE(2, sb_i);
                // header + scales (16 bytes) and this half's 64 bytes of nibbles
                uint32_t hw[4], w[16];
                {
                    const uint4 *src = (const uint4 *) (mine + (sb_i % kPfPre) * kPfRawStage);
                    const uint4 h4 = src[0];
                    hw[0] = h4.x; hw[1] = h4.y; hw[2] = h4.z; hw[3] = h4.w;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint4 v = src[1 + i];
                        w[4 * i] = v.x; w[4 * i + 1] = v.y; w[4 * i + 2] = v.z; w[4 * i + 3] = v.w;
                    }
                }
                fetch((int) sb_i + kPfPre);  // into the slot just read
                if (tid == 0) PF_TRACE(8, sb_i);
                const float d = h2f((uint16_t) (hw[0] & 0xFFFF)), dmin = h2f((uint16_t) (hw[0] >> 16));
                const int mode = pf_row_mode(d, dmin);
                if (grp == 0) {
                    const int es = sb_i % kPfEpStages;
                    if (!(ok = pf_wait_warp(&bars->ep_empty[es], ((sb_i / kPfEpStages) & 1) ^ 1, abort, a.st))) break;
                    ep[es * 2 * kPfTileN + kPfTileN + m] = mode == 0 ? d : (mode == 1 ? dmin : 0.f);
                    warp_arrive(&bars->ep_full[es]);
                }
                // 6-bit scale / min of sub-block j (get_scale_min_k4, ggml-quants.c:880-887)
                auto sbyte = [&](int i) -> uint32_t { return (hw[1 + i / 4] >> (8 * (i % 4))) & 0xFFu; };
                auto scale_of = [&](int j) -> uint32_t {
                    return j < 4 ? (sbyte(j) & 63u) : ((sbyte(j + 4) & 0xFu) | ((sbyte(j - 4) >> 6) << 4));
                };
                auto min_of = [&](int j) -> uint32_t {
                    return j < 4 ? (sbyte(j + 4) & 63u) : ((sbyte(j + 4) >> 4) | ((sbyte(j) >> 6) << 4));
                };
                const float r = mode == 0 ? dmin / d : (mode == 1 ? d / dmin : 0.f);
                const uint32_t k2 = mode == 1 ? h2_pack(r) : 0u;
                const uint32_t a_i = 2 * sb_i + (uint32_t) grp;  // A stages are used in turn by the halves
                const int as = a_i % kPfAStages;
                if (tid == 0) PF_TRACE(12, sb_i);
                if (!(ok = pf_wait_warp(&bars->a_empty[as], ((a_i / kPfAStages) & 1) ^ 1, abort, a.st))) break;
                if (tid == 0) PF_TRACE(10, sb_i);
                umma::fence_after_sync();
                const uint32_t a_t = tbase + lane_base + 2 * kPfAccCols + (uint32_t) as * kPfACols;
#pragma unroll
                for (int jj = 0; jj < 2; ++jj) {
                    // chunk j = 2grp + jj: low nibbles -> sub-block 2j, high nibbles -> 2j+1.
                    // Low nibble q: fp16 bits 0x6400|q = 1024+q, times sc minus 1024*sc.
                    // High nibble in place: 0x6400|(q<<4) = 1024+16q, times sc/16 minus 64*sc.
                    // Both fused multiply-adds are exact (results are integers <= 945).
                    const int j = 2 * grp + jj;
                    const uint32_t slo = h2_int(scale_of(2 * j)), blo = hmul2_u(slo, kH2Neg1024);
                    const uint32_t sh1 = h2_int(scale_of(2 * j + 1));
                    const uint32_t shi = hmul2_u(sh1, kH2Sixteenth), bhi = hmul2_u(sh1, kH2Neg64);
#pragma unroll
                    for (int g = 0; g < 2; ++g) {
                        uint32_t o[16];
#pragma unroll
                        for (int ww = 0; ww < 4; ++ww) {
                            const uint32_t xw = w[8 * jj + 4 * g + ww], yw = xw >> 8;
                            o[4 * ww + 0] = hfma2_u((xw & 0x000F000Fu) | 0x64006400u, slo, blo);
                            o[4 * ww + 1] = hfma2_u((yw & 0x000F000Fu) | 0x64006400u, slo, blo);
                            o[4 * ww + 2] = hfma2_u((xw & 0x00F000F0u) | 0x64006400u, shi, bhi);
                            o[4 * ww + 3] = hfma2_u((yw & 0x00F000F0u) | 0x64006400u, shi, bhi);
                        }
                        if (mode != 0) {
#pragma unroll
                            for (int i = 0; i < 16; ++i) o[i] = hmul2_u(o[i], k2);
                        }
                        umma::st16(a_t + (uint32_t) (jj * 32 + g * 16), o);
                    }
                }
                // min coefficients -(dmin/d)*m as hi + lo: Veltkamp split (factor 2^13 + 1)
                // leaves 11 significant bits in hi, so hi is an fp16 value and lo = full - hi
                // is exact; fp16(lo) then carries the next 11 bits.
                uint32_t o8[8];
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const float mc = f_int(min_of(c));
                    float v = 0.f;
                    if (mode == 0) {
                        const float full = __fmul_rn(-r, mc);
                        const float t = __fmul_rn(full, 8193.f);
                        const float hi = __fsub_rn(t, __fsub_rn(t, full));
                        v = grp == 0 ? hi : __fsub_rn(full, hi);
                    } else if (mode == 1) {
                        v = grp == 0 ? -mc : 0.f;
                    }
                    o8[c] = h2_pack(v);
                }
                umma::st8(a_t + 64, o8);
                umma::wait_st();
                umma::fence_before_sync();
                warp_arrive(&bars->a_full[as]);
                if (tid == 0) PF_TRACE(9, sb_i);
                if (tid == 128) PF_TRACE(3, sb_i);
            }
        }
    } else if (warp < kPfWarpProd) {
        // ------------------------------------------------------------ epilogue
        // one thread per (weight row, half of the token columns): 64 running sums in registers
        const int qd = warp & 3, g = (warp - kPfWarpEpi) >> 2, m = qd * 32 + lane;
        const uint32_t lane_base = (uint32_t) (qd * 32) << 16;
        uint32_t acc_i = 0;
        bool ok = true;
        for (int it = blockIdx.x; it < total && ok; it += gridDim.x) {
            const PfItem x = pf_item(a, it);
            // output row offsets (in floats, < 2^32 checked on the host) of columns
            // 64g + lane and 64g + 32 + lane
            uint32_t off[2] = {0, 0};
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const int n = 64 * g + 32 * u + lane;
                if (n < x.cnt) {
                    const int p = __ldg(a.pairs + x.p0 + n);
                    const int t = p / a.n_used, j = p - t * a.n_used;
                    off[u] = (uint32_t) (((size_t) j * a.dnb1 + (size_t) t * a.dnb2) >> 2);
                }
            }
            float out[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) out[i] = 0.f;
            for (int s = 0; s < nsb && ok; ++s, ++acc_i) {
                const int es = acc_i % kPfEpStages;
                if (!(ok = pf_wait_warp(&bars->ep_full[es], (acc_i / kPfEpStages) & 1, abort, a.st))) break;
                const float *eps = ep + es * 2 * kPfTileN;
                const float S = eps[kPfTileN + m];
                const int ab = acc_i & 1;
                if (!(ok = pf_wait_warp(&bars->acc_full[ab], (acc_i >> 1) & 1, abort, a.st))) break;
                if (tid == kPfWarpEpi * 32) PF_TRACE(6, acc_i);
                umma::fence_after_sync();
                const uint32_t d_t = tbase + lane_base + (uint32_t) ab * kPfAccCols + 64 * g;
#pragma unroll
                for (int c = 0; c < 8; ++c) {
                    const int c0 = 64 * g + 8 * c;
                    if (c0 < x.Nt) {  // warp-uniform
                        uint32_t v[8];
                        umma::ld8(d_t + 8 * c, v);
                        umma::wait_ld();
                        const float4 da0 = *(const float4 *) (eps + c0), da1 = *(const float4 *) (eps + c0 + 4);
                        float *o = out + 8 * c;
                        o[0] = fmaf(S * da0.x, __uint_as_float(v[0]), o[0]);
                        o[1] = fmaf(S * da0.y, __uint_as_float(v[1]), o[1]);
                        o[2] = fmaf(S * da0.z, __uint_as_float(v[2]), o[2]);
                        o[3] = fmaf(S * da0.w, __uint_as_float(v[3]), o[3]);
                        o[4] = fmaf(S * da1.x, __uint_as_float(v[4]), o[4]);
                        o[5] = fmaf(S * da1.y, __uint_as_float(v[5]), o[5]);
                        o[6] = fmaf(S * da1.z, __uint_as_float(v[6]), o[6]);
                        o[7] = fmaf(S * da1.w, __uint_as_float(v[7]), o[7]);
                    }
                }
                umma::fence_before_sync();
                warp_arrive(&bars->acc_empty[ab]);
                warp_arrive(&bars->ep_empty[es]);
                if (tid == kPfWarpEpi * 32) PF_TRACE(7, acc_i);
            }
            if (!ok) break;
            // rows of an invalid expert slot come out as zeros (row scale 0)
            const int64_t row = (int64_t) x.mt * kPfTileM + m;
#pragma unroll
            for (int i = 0; i < 64; ++i) {
                const uint32_t o = __shfl_sync(0xffffffffu, off[i >> 5], i & 31);
                if (m < x.rows && 64 * g + i < x.cnt) a.dst[(size_t) o + row] = out[i];
            }
        }
    }

    umma::fence_before_sync();
    __syncthreads();
    if (warp == kPfWarpMma) {
        umma::fence_after_sync();
        umma::tmem_dealloc(tbase, kPfTmemCols);
    }
}

cudaError_t launch_pf_gemm_q4k(const PrefillArgs &a, cudaStream_t s) {
    static DeviceSmemLimit limit;
    cudaError_t e = ensure_dyn_smem(pf_gemm_q4k_kernel, (size_t) kPfSmem, limit);
    if (e != cudaSuccess) return e;
    pf_gemm_q4k_kernel<<<num_sms(), kPfThreads, kPfSmem, s>>>(a);
    return cudaGetLastError();
}

#ifdef QWB_PF_TRACE
}  // namespace qwb
extern "C" QWB_API int qwb_debug_pf_trace(void *host, size_t bytes) {
    return cudaMemcpyFromSymbol(host, qwb::g_pf_trace, bytes) == cudaSuccess ? 0 : 1;
}
namespace qwb {
#endif

bool pf_eligible(int type, int64_t K, int64_t M, int64_t P, int64_t n_as) {
    if (type != QWB_TYPE_Q4_K || K % QK_K || K < QK_K || M < 1) return false;
    const int64_t used = std::min<int64_t>(P, n_as);
    return used > 0 && P >= 32 * used;
}

}  // namespace qwb
