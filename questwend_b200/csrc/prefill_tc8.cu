// prefill_tc8.cu - MUL_MAT_ID on Q6_K experts with many tokens per expert as a grouped
// GEMM on the 5th-generation tensor cores (tcgen05.mma kind::i8: s8 x s8 -> s32
// accumulators in tensor memory).
//
// Reference arithmetic (ggml_compute_forward_mul_mat_id, ggml-cpu/ggml-cpu.c:1554-1736;
// Q6_K x Q8_K, ggml-cpu/quants.c:851-915): for every superblock of 256,
//     sumf += (d_w * d_a) * (float) sum_s sc_s * isum_s   over its 16 sub-blocks of 16,
//     isum_s = sum (q6 - 32) * q_a, sc_s the sub-block's int8 scale.
// The integer superblock sum is kept exact: the sub-block scale is folded into the
// weights, v = sc * (q - 32) in [-4064, 4096], written as two int8 planes
// v = 64 * a1 + a0 (a0 in [-32, 31], a1 in [-63, 64]); two MMAs per K=32 (planes a1 and
// a0, same activations) accumulate sum a1 * q_a and sum a0 * q_a over the superblock, and
// 64 * acc1 + acc0 is the reference's integer superblock sum (|.| < 2^31).  The epilogue
// adds (d_w * d_a) * (float) sum, once per 256 K.
//
// Q8_0 (pf_tc8q_kernel below): the rank-1 block scale d_w * d_a changes every 32 K, so the
// integer dot of every 32-element block gets its own tensor-memory accumulator region:
// per 128-K step four MMAs of K = 32 into four regions (two per accumulator buffer, the
// buffers alternating), and the epilogue adds (d_w * d_a) * (float) isum per block.  The
// epilogue of one half-step runs while the MMAs of the next fill the other buffer, so no
// per-block load / scale / refill chain lies on the critical path.
//
// Work item = (token tile of <= 128 (token, slot) pairs of one expert, 128 weight rows);
// one persistent CTA per SM takes items blockIdx.x, + gridDim.x, ...  Warp roles:
//   warps 0-3   producers, one thread per weight row: 16-byte cp.async of the raw
//               superblocks (widened to 16-byte boundaries) and one bulk copy per step of
//               the tile's activation codes and scales, gathered beforehand into the B
//               operand's core-matrix layout (tc8_gather_kernel: the bulk copies keep far
//               more bytes in flight per SM than 16-byte copies of scattered rows); then
//               the repack of the codes into the A operand's two planes and the step's
//               scales; one mbarrier arrival per step
//   warp 4      TMEM allocation and the MMA-issuing thread
//   warps 5-12  epilogue: two warpgroups (token columns 0-63 / 64-127), one weight row
//               per thread, the item's sums in registers
// Pipeline step = 128 K elements (half a superblock); A/B operand stages are
// triple-buffered, the two superblock accumulators (a1 and a0 planes, 256 columns each)
// double-buffered in the 512 tensor-memory columns.  Every wait is bounded; a timeout sets
// QWB_DEVERR_TIMEOUT and all roles drain and exit.
#include <algorithm>

#include "common.cuh"
#include "dot.cuh"
#include "kernels.cuh"
#include "mmid.cuh"
#include "umma.cuh"

namespace qwb {

namespace {

constexpr int kT8M = 128;        // weight rows per item
constexpr int kT8N = 128;        // token pairs per item (index tile)
constexpr int kT8Step = 128;     // K per pipeline step
constexpr int kT8Stages = 3;     // A/B operand stages
constexpr int kT8EpStages = 4;   // scale slots (one per step)
constexpr int kT8Threads = 13 * 32;
constexpr int kT8WarpMma = 4;
constexpr int kT8WarpEpi = 5;    // 5..12
constexpr int kT8A = 2 * kT8M * kT8Step;  // 32768: A stage bytes (planes a1 | a0)
constexpr int kT8B = kT8N * kT8Step;      // 16384: B stage bytes
constexpr int kT8RawRow = 240;            // raw bytes per row per superblock (widened)
constexpr uint32_t kT8Lbo = 128 * 16;     // leading byte offset of a 128-row operand slab
constexpr uint32_t kT8TmemCols = 512;
constexpr uint32_t kT8DaBytes = 4 * kT8N;  // activation scales per step of a tile
constexpr int kQ8Blk = kT8Step / 32;           // Q8_0 blocks per step
constexpr int kQ8RawRow = 8 * Q80_BYTES;       // 272: raw bytes of an 8-block group (two steps)
constexpr uint32_t kQ8DaBytes = 4 * kQ8Blk * kT8N;  // Q8_0 activation scales per step of a tile
// Q8_0 kernel: 4 producer warps, the MMA warp, 16 epilogue warps (four warpgroups of 32
// token columns each: the per-element block scaling is the kernel's main work)
constexpr int kQ8EpiWarps = 16;
constexpr int kQ8Threads = (kT8WarpEpi + kQ8EpiWarps) * 32;

// scales of one superblock: d of weight row m and d_a of token n
struct T8Ep {
    float dw[kT8M];
    float da[kT8N];
};

struct T8Smem {
    uint8_t a[kT8Stages][kT8A];
    uint8_t b[kT8Stages][kT8B];
    uint8_t raw[2][kT8M * kT8RawRow];
    T8Ep ep[kT8EpStages];
    float dstage[kT8Stages][kT8N];  // activation scales of the step (bulk copy)
    int raw_off[2][kT8M];           // offset of the superblock inside its widened row bytes
    uint64_t full[kT8Stages], empty[kT8Stages], bfull[kT8Stages];
    uint64_t acc_full[2], acc_empty[2];
    uint64_t ep_full[kT8EpStages], ep_empty[kT8EpStages];
    uint64_t drain;
    uint32_t tmem;
    int abort;
};
static_assert(sizeof(T8Smem) <= 232448, "one CTA per SM: at most 227 KB of shared memory");

struct T8Item {
    int tile, mt, p0, cnt, Nt, rows;
    int64_t slot;  // -1: invalid expert id
};
__device__ __forceinline__ T8Item t8_item(const I8PrefillArgs &a, int m_tiles, int it) {
    T8Item x;
    x.tile = it / m_tiles;
    x.mt = it - x.tile * m_tiles;
    const int4 t = a.tiles[x.tile];
    x.p0 = t.y;
    x.cnt = t.z;
    x.Nt = (t.z + 15) & ~15;
    x.rows = (int) min((int64_t) kT8M, a.M - (int64_t) x.mt * kT8M);
    x.slot = (t.x >= 0 && t.x < a.n_as) ? (int64_t) t.x : -1;
    return x;
}

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// barrier among the 128 producer threads only
__device__ __forceinline__ void producers_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// byte offset of operand element (row r, k) in a 128-row stage (k < 128)
__device__ __forceinline__ uint32_t t8_off(int r, int k) {
    return (uint32_t) (k >> 4) * kT8Lbo + (uint32_t) (r >> 3) * 128u + (uint32_t) (r & 7) * 16u + (uint32_t) (k & 15);
}

// 4 codes q (0..63, one per byte of w) of sub-block scale sc -> int8 planes a1, a0 with
// sc * (q - 32) = 64 * a1 + a0.  Two 16-bit lanes per 32-bit word: with sc' = sc + 128 in
// [0, 255], z = q * sc' - 128 q + (4128 - 32 sc) = sc (q - 32) + 4128 lies in [64, 8224]
// and no lane borrows from or carries into its neighbour; then a0 + 32 = z & 63 and
// a1 + 64 = z >> 6.
__device__ __forceinline__ void q6_planes(uint32_t w, int sc, uint32_t &a1, uint32_t &a0) {
    const uint32_t scp = (uint32_t) (sc + 128);
    const uint32_t bias = (uint32_t) (4096 - 32 * sc + 32) * 0x10001u;
    const uint32_t x01 = __byte_perm(w, 0, 0x4140), x23 = __byte_perm(w, 0, 0x4342);
    const uint32_t z01 = x01 * scp + bias - (x01 << 7), z23 = x23 * scp + bias - (x23 << 7);
    const uint32_t lo01 = z01 & 0x003F003Fu, lo23 = z23 & 0x003F003Fu;
    const uint32_t hi01 = (z01 >> 6) & 0x03FF03FFu, hi23 = (z23 >> 6) & 0x03FF03FFu;
    a0 = __vsub4(__byte_perm(lo01, lo23, 0x6420), 0x20202020u);
    a1 = __vsub4(__byte_perm(hi01, hi23, 0x6420), 0x40404040u);
}

// Gathered activations: per tile and 128-K step, the B operand stage exactly as the MMA
// reads it (token n's codes k at t8_off(n, k)) and the superblock's activation scales.
// Grid (max_tiles, steps); tiles past the index's count exit.
// Q8_0 activations (q80): four scales per step and token (blocks of 32), stored
// [block][token]; Q8_K: one per superblock (two steps).
template <bool Q80>
__global__ void __launch_bounds__(256) tc8_gather_kernel(Q8Planes act, int act_dstride, int64_t K,
                                                         const int4 *__restrict__ tiles, const int *__restrict__ n_tiles,
                                                         const int *__restrict__ pairs, int n_used, int n_b,
                                                         uint8_t *__restrict__ btiles, float *__restrict__ bda) {
    const int tile = blockIdx.x, s = blockIdx.y, nsteps = (int) gridDim.y;
    if (tile >= *n_tiles) return;
    const int4 t = tiles[tile];
    __shared__ int64_t arow[kT8N];
    for (int n = threadIdx.x; n < kT8N; n += blockDim.x) {
        int64_t r = -1;
        if (n < t.z) {
            const int p = pairs[t.y + n];
            const int tt = p / n_used, j = p - tt * n_used;
            r = (int64_t) tt * n_b + j % n_b;
        }
        arow[n] = r;
    }
    __syncthreads();
    uint8_t *dst = btiles + ((size_t) tile * nsteps + s) * kT8B;
    // chunk c: token n = c % 128, 16-byte column kc = c / 128 (consecutive threads write
    // consecutive 16-byte pieces of one core-matrix column)
    for (int c = threadIdx.x; c < kT8N * 8; c += blockDim.x) {
        const int n = c & (kT8N - 1), kc = c >> 7;
        uint4 v = make_uint4(0, 0, 0, 0);
        if (arow[n] >= 0) v = *(const uint4 *) (act.qs + arow[n] * K + (int64_t) s * kT8Step + 16 * kc);
        *(uint4 *) (dst + t8_off(n, 16 * kc)) = v;
    }
    if (Q80) {
        float *da = bda + ((size_t) tile * nsteps + s) * (kQ8DaBytes / 4);
        for (int c = threadIdx.x; c < kQ8Blk * kT8N; c += blockDim.x) {
            const int b = c >> 7, n = c & (kT8N - 1);
            da[c] = arow[n] >= 0 ? act.d[arow[n] * act_dstride + (int64_t) s * kQ8Blk + b] : 0.f;
        }
    } else {
        float *da = bda + ((size_t) tile * nsteps + s) * (kT8DaBytes / 4);
        for (int n = threadIdx.x; n < kT8N; n += blockDim.x)
            da[n] = arow[n] >= 0 ? act.d[arow[n] * act_dstride + (s >> 1)] : 0.f;
    }
}

__global__ void __launch_bounds__(kT8Threads, 1) pf_tc8_kernel(const I8PrefillArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    T8Smem &S = *(T8Smem *) smem_raw;
    volatile int *abort = &S.abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m_tiles = (int) ceil_div(a.M, kT8M);
    const int total = *a.n_tiles * m_tiles;
    if ((int) blockIdx.x >= total) return;
    const int nsteps = (int) (a.K / kT8Step);
    const int n_items = (total - (int) blockIdx.x + (int) gridDim.x - 1) / (int) gridDim.x;
    const int gsteps = n_items * nsteps;  // this CTA's steps over all its items

    if (tid == 0) {
        for (int i = 0; i < kT8Stages; ++i) {
            mbar_init(&S.full[i], 128);
            mbar_init(&S.empty[i], 1);
            mbar_init(&S.bfull[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&S.acc_full[i], 1);
            mbar_init(&S.acc_empty[i], 256);
        }
        for (int i = 0; i < kT8EpStages; ++i) {
            mbar_init(&S.ep_full[i], 128);
            mbar_init(&S.ep_empty[i], 256);
        }
        mbar_init(&S.drain, 1);
        S.abort = 0;
        fence_mbar_init();
    }
    if (warp == kT8WarpMma) {
        umma::tmem_alloc(&S.tmem, kT8TmemCols);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tbase = S.tmem;

    if (warp < kT8WarpMma) {
        // ------------------------------------------------------------ producers
        const int r = tid;  // weight row / token row of this thread (repack, scales)
        // item state cached per item index (k = CTA-local item)
        int c_item = -1, c_tile = 0, c_rows = 0;
        int n_issued = 0, n_seen = 0;  // steps whose bulk copies were issued / waited for
        const uint8_t *wbase = nullptr;  // row 0 of the item's 128 weight rows (null: invalid expert)
        auto item_state = [&](int k) {
            if (k == c_item) return;
            c_item = k;
            const T8Item x = t8_item(a, m_tiles, (int) blockIdx.x + k * (int) gridDim.x);
            wbase = x.slot >= 0 ? a.W + (size_t) x.slot * a.nb2 + (size_t) x.mt * kT8M * a.nb1 : nullptr;
            c_rows = x.rows;
            c_tile = x.tile;
        };
        // copies of global step g: the B codes of the step and their scales and, on even
        // steps, the raw bytes of the superblock it starts; one cp.async group per step
        auto issue = [&](int g) {
            if (g < gsteps) {
                const int k = g / nsteps, s = g - k * nsteps, st = g % kT8Stages;
                item_state(k);
                if (g >= kT8Stages) {
                    // the stage's previous MMAs are done (the MMA thread commits it)
                    if (!pf_wait_warp(&S.empty[st], ((g / kT8Stages) & 1) ^ 1, abort, a.st)) {
                        cp_async_commit();
                        return false;
                    }
                }
                // B and its scales: the tile's gathered stage, two bulk copies on bfull[st]
                if (r == 0) {
                    const size_t ts = (size_t) c_tile * nsteps + s;
                    mbar_arrive_expect_tx(&S.bfull[st], (uint32_t) kT8B + kT8DaBytes);
                    bulk_g2s(S.b[st], a.btiles + ts * kT8B, (uint32_t) kT8B, &S.bfull[st]);
                    bulk_g2s(S.dstage[st], a.bda + ts * (kT8DaBytes / 4), kT8DaBytes, &S.bfull[st]);
                }
                n_issued = g + 1;
                if ((s & 1) == 0) {
                    // the 210-byte superblock widened to 16-byte boundaries (<= 15 pieces)
                    const int u = s >> 1, rs = (g >> 1) & 1;
                    const uint8_t *wrow = wbase && r < c_rows ? wbase + (size_t) r * a.nb1 : nullptr;
                    const uintptr_t s0 = (uintptr_t) (wrow ? wrow : a.W) + (uintptr_t) u * Q6K_BYTES;
                    const uintptr_t a0 = s0 & ~(uintptr_t) 15;
                    S.raw_off[rs][r] = (int) (s0 - a0);
                    for (int c = 0; c < 15; ++c) {
                        const bool in = wrow && (a0 + 16 * c < s0 + Q6K_BYTES);
                        cp_async16(&S.raw[rs][r * kT8RawRow + 16 * c], (const void *) (in ? a0 + 16 * c : a0), in);
                    }
                }
            }
            cp_async_commit();
            return true;
        };
        bool ok = issue(0);
        ok = ok && issue(1);
        // Every producer thread runs all gsteps iterations (the named barriers need all
        // 128 of them); after a timeout anywhere the iterations do no work.
        for (int g = 0; g < gsteps; ++g) {
            producers_sync();  // step g - 1 repacked by every producer: its raw unit may be refilled
            if (ok && !*abort) ok = issue(g + 2);
            cp_async_wait<2>();  // this thread's copies of step g
            producers_sync();    // everyone's
            if (!ok || *abort) {
                ok = false;
                continue;
            }
            const int k = g / nsteps, s = g - k * nsteps, st = g % kT8Stages, rs = (g >> 1) & 1;
            item_state(k);
            // scale slot of this step
            const int es = g % kT8EpStages;
            if (!(ok = pf_wait_warp(&S.ep_empty[es], ((g / kT8EpStages) & 1) ^ 1, abort, a.st))) continue;
            if (!(ok = pf_wait_warp(&S.bfull[st], (g / kT8Stages) & 1, abort, a.st))) continue;  // the step's scales
            n_seen = g + 1;
            auto &ep = S.ep[es];
            uint8_t *A = S.a[st];
            // half h = s & 1 of the superblock: elements 128 h + 32 i + l of sub-lanes
            // i = 0..3 (ql at 64 h + 32 (i & 1), high nibbles when i >= 2; qh bits 2i, 2i+1)
            const uint8_t *sb = S.raw[rs] + r * kT8RawRow + S.raw_off[rs][r];
            const int h = s & 1;
            uint32_t qh[8];
            lds_words8_a2(sb + 128 + 32 * h, qh);
#pragma unroll 1
            for (int i = 0; i < 4; ++i) {
                uint32_t qa[8];
                lds_words8_a2(sb + 64 * h + 32 * (i & 1), qa);
                const int8_t *scp = (const int8_t *) (sb + 192) + 8 * h + 2 * i;
                const int sc0 = scp[0], sc1 = scp[1];  // sub-blocks of l = 0..15 and 16..31
                uint32_t p1[8], p0[8];
#pragma unroll
                for (int m = 0; m < 8; ++m) {
                    const uint32_t nib = i < 2 ? (qa[m] & 0x0f0f0f0fu) : ((qa[m] >> 4) & 0x0f0f0f0fu);
                    const uint32_t q = nib | (((qh[m] >> (2 * i)) & 0x03030303u) << 4);
                    q6_planes(q, m < 4 ? sc0 : sc1, p1[m], p0[m]);
                }
                // elements l = 0..31 of sub-lane i are k = 32 i .. 32 i + 31 within the half:
                // two 16-byte core-matrix rows per plane (a warp's 32 rows store 512
                // contiguous bytes per instruction: no bank conflicts)
                *(uint4 *) (A + t8_off(r, 32 * i)) = make_uint4(p1[0], p1[1], p1[2], p1[3]);
                *(uint4 *) (A + t8_off(r, 32 * i + 16)) = make_uint4(p1[4], p1[5], p1[6], p1[7]);
                *(uint4 *) (A + kT8M * kT8Step + t8_off(r, 32 * i)) = make_uint4(p0[0], p0[1], p0[2], p0[3]);
                *(uint4 *) (A + kT8M * kT8Step + t8_off(r, 32 * i + 16)) = make_uint4(p0[4], p0[5], p0[6], p0[7]);
            }
            if (h == 1) {  // the superblock's scales, once both halves are in
                ep.dw[r] = h2f(*(const uint16_t *) (sb + 208));
                ep.da[r] = S.dstage[st][r];
            }
            fence_proxy_async_smem();  // the operands are read by the tensor cores
            // one arrival per thread on both: operands and scales of step g are in place
            asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&S.full[st])) : "memory");
            asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&S.ep_full[es])) : "memory");
        }
        cp_async_wait<0>();  // no copy stays in flight past the kernel
        if (r == 0) {
            // bulk copies issued for steps this loop did not consume (only after an abort)
            for (int g = n_seen; g < n_issued; ++g) mbar_wait(&S.bfull[g % kT8Stages], (g / kT8Stages) & 1);
        }
    } else if (warp == kT8WarpMma) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t acc_i = 0;
            bool ok = true;
            for (int g = 0; g < gsteps && ok; ++g) {
                const int k = g / nsteps, s = g - k * nsteps, st = g % kT8Stages;
                const T8Item x = t8_item(a, m_tiles, (int) blockIdx.x + k * (int) gridDim.x);
                const uint32_t idesc = umma::idesc_i8(kT8M, x.Nt);
                if (!(ok = pf_wait(&S.full[st], (g / kT8Stages) & 1, abort, a.st))) break;
                if (!(ok = pf_wait(&S.bfull[st], (g / kT8Stages) & 1, abort, a.st))) break;
                umma::fence_after_sync();
                const uint32_t a_s = smem_u32(S.a[st]), b_s = smem_u32(S.b[st]);
                const int h = s & 1, rg = (int) (acc_i & 1);
                if (h == 0) {
                    if (!(ok = pf_wait(&S.acc_empty[rg], ((acc_i >> 1) & 1) ^ 1, abort, a.st))) break;
                    umma::fence_after_sync();
                }
                const uint32_t d1 = tbase + (uint32_t) rg * 256, d0 = d1 + 128;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const uint64_t bd = umma::sdesc(b_s + 2 * b * kT8Lbo, kT8Lbo, 128);
                    const uint32_t acc = (h | b) != 0;
                    umma::mma_i8_ss(d1, umma::sdesc(a_s + 2 * b * kT8Lbo, kT8Lbo, 128), bd, idesc, acc);
                    umma::mma_i8_ss(d0, umma::sdesc(a_s + kT8M * kT8Step + 2 * b * kT8Lbo, kT8Lbo, 128), bd, idesc,
                                    acc);
                }
                umma::commit(&S.empty[st]);
                if (h == 1) {
                    umma::commit(&S.acc_full[rg]);
                    ++acc_i;
                }
            }
            // every MMA issued by this thread has completed before TMEM is released
            umma::commit(&S.drain);
            mbar_wait(&S.drain, 0);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        const int qd = warp & 3, g = (warp - kT8WarpEpi) >> 2, m = qd * 32 + lane;
        const uint32_t lane_base = (uint32_t) (qd * 32) << 16;
        uint32_t acc_i = 0;
        bool ok = true;
        int gstep = 0;
        for (int k = 0; k < n_items && ok; ++k) {
            const T8Item x = t8_item(a, m_tiles, (int) blockIdx.x + k * (int) gridDim.x);
            // output offsets (floats) of token columns 64 g + lane and 64 g + 32 + lane
            uint32_t off[2] = {0, 0};
#pragma unroll
            for (int uu = 0; uu < 2; ++uu) {
                const int n = 64 * g + 32 * uu + lane;
                if (n < x.cnt) {
                    const int p = __ldg(a.pairs + x.p0 + n);
                    const int t = p / a.n_used, j = p - t * a.n_used;
                    off[uu] = (uint32_t) (((size_t) j * a.dnb1 + (size_t) t * a.dnb2) >> 2);
                }
            }
            const int nch = max(0, min(2, (x.Nt - 64 * g + 31) / 32));  // 32-column chunks with tokens
            float out[64];
#pragma unroll
            for (int i = 0; i < 64; ++i) out[i] = 0.f;
            for (int s = 0; s < nsteps && ok; ++s, ++gstep) {
                const int es = gstep % kT8EpStages;
                if (!(ok = pf_wait_warp(&S.ep_full[es], (gstep / kT8EpStages) & 1, abort, a.st))) break;
                const auto &ep = S.ep[es];
                if (s & 1) {
                    const int rg = (int) (acc_i & 1);
                    if (!(ok = pf_wait_warp(&S.acc_full[rg], (acc_i >> 1) & 1, abort, a.st))) break;
                    umma::fence_after_sync();
                    const float dw = ep.dw[m];
                    const uint32_t d1 = tbase + lane_base + (uint32_t) rg * 256 + 64 * g;
#pragma unroll
                    for (int c = 0; c < 4; ++c) {
                        if (16 * c < 32 * nch) {  // warp-uniform: 16-column pieces with tokens
                            uint32_t v1[16], v0[16];
                            umma::ld16(d1 + 16 * c, v1);
                            umma::ld16(d1 + 128 + 16 * c, v0);
                            umma::wait_ld();
#pragma unroll
                            for (int i = 0; i < 16; ++i) {
                                const int col = 64 * g + 16 * c + i;
                                const int isum = 64 * (int) v1[i] + (int) v0[i];
                                out[16 * c + i] = __fmaf_rn(__fmul_rn(dw, ep.da[col]), (float) isum, out[16 * c + i]);
                            }
                        }
                    }
                    umma::fence_before_sync();
                    warp_arrive(&S.acc_empty[rg]);
                    ++acc_i;
                }
                warp_arrive(&S.ep_empty[es]);
            }
            if (!ok) break;
            // rows of an invalid expert id come out as zeros (their weights were zero-filled)
            const int64_t row = (int64_t) x.mt * kT8M + m;
#pragma unroll
            for (int i = 0; i < 64; ++i) {
                const uint32_t o = __shfl_sync(0xffffffffu, off[i >> 5], i & 31);
                if (m < x.rows && 64 * g + i < x.cnt) a.dst[(size_t) o + row] = out[i];
            }
            if (x.slot < 0 && x.mt == 0 && m == 0 && g == 0) report(a.st, QWB_DEVERR_ID_RANGE, a.tiles[x.tile].x);
        }
    }

    umma::fence_before_sync();
    __syncthreads();
    if (warp == kT8WarpMma) {
        umma::fence_after_sync();
        umma::tmem_dealloc(tbase, kT8TmemCols);
    }
}

// ---------------------------------------------------------------- Q8_0
// Optional per-step timestamps of CTA 0's roles (compiled in only with -DQWB_DECODE_TRACE):
// [0] producers' operands in place, [1] MMAs issued, [2] epilogue done, [3] copies landed.
#ifdef QWB_DECODE_TRACE
__device__ unsigned long long g_tc8_trace[4][512];
#define T8TRACE(role, step)                                                         \
    do {                                                                            \
        if (blockIdx.x == 0 && (step) < 512) g_tc8_trace[role][step] = globaltimer_ns(); \
    } while (0)
#else
#define T8TRACE(role, step) \
    do {                    \
    } while (0)
#endif

// scales of one step: d of weight row m and d_a of token n, per block of 32
struct Q8Ep {
    float dw[kQ8Blk][kT8M];
    float da[kQ8Blk][kT8N];
};

struct Q8Smem {
    uint8_t a[kT8Stages][kT8M * kT8Step];
    uint8_t b[kT8Stages][kT8B];
    uint8_t raw[2][kT8M * kQ8RawRow];
    Q8Ep ep[kT8EpStages];
    float dstage[kT8Stages][kQ8Blk * kT8N];  // activation scales of the step (bulk copy)
    uint64_t full[kT8Stages], empty[kT8Stages], bfull[kT8Stages];
    uint64_t acc_full[2], acc_empty[2];  // two accumulator buffers of two 128-column regions
    uint64_t ep_full[kT8EpStages], ep_empty[kT8EpStages];
    uint64_t drain;
    uint32_t tmem;
    int abort;
};
static_assert(sizeof(Q8Smem) <= 232448, "one CTA per SM: at most 227 KB of shared memory");

// Repack blocks 4 H .. 4 H + 3 of a row's raw 8-block group (272 bytes at rowp, 16-byte
// aligned) into the A stage: each block's 32 codes start at the 2-byte aligned offset
// 34 b + 2; they are read as three 16-byte words from the 16-byte floor (conflict-free at
// the 272-byte row stride) and realigned with funnel shifts (compile-time offsets).
template <int H>
__device__ __forceinline__ void q8_repack_half(const uint8_t *rowp, uint8_t *A, int r, float (*dw)[kT8M]) {
#pragma unroll
    for (int bb = 0; bb < kQ8Blk; ++bb) {
        const int q = Q80_BYTES * (4 * H + bb) + 2;  // compile-time after unrolling
        const uint4 *src = (const uint4 *) (rowp + (q & ~15));
        const uint4 c0 = src[0], c1 = src[1], c2 = src[2];
        const uint32_t x[12] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w, c2.x, c2.y, c2.z, c2.w};
        const int ws = (q & 15) >> 2;
        const uint32_t bs = (uint32_t) (q & 3) * 8u;
        uint32_t w[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) w[i] = __funnelshift_r(x[ws + i], x[ws + i + 1], bs);
        *(uint4 *) (A + t8_off(r, 32 * bb)) = make_uint4(w[0], w[1], w[2], w[3]);
        *(uint4 *) (A + t8_off(r, 32 * bb + 16)) = make_uint4(w[4], w[5], w[6], w[7]);
        // the block's fp16 scale: the 2 bytes before its codes
        dw[bb][r] = h2f(*(const uint16_t *) (rowp + q - 2));
    }
}

// Q8_0 x Q8_0 (ggml-cpu/quants.c:451: sumf += (d_w * d_a) * isum over the blocks of 32).
// Work items, operand stages and bounded waits as pf_tc8_kernel; the A stage is one plane
// of int8 codes.  Per 128-K step the MMA thread issues, for each half-step (blocks 2 hs,
// 2 hs + 1), two K = 32 MMAs into the two 128-column regions of accumulator buffer
// (half-step count & 1), then commits it; sixteen epilogue warps (four warpgroups of 32
// token columns) read both regions and add (d_w * d_a) * (float) isum per block into the
// item's register sums.
__global__ void __launch_bounds__(kQ8Threads, 1) pf_tc8q_kernel(const I8PrefillArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    Q8Smem &S = *(Q8Smem *) smem_raw;
    volatile int *abort = &S.abort;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int m_tiles = (int) ceil_div(a.M, kT8M);
    const int total = *a.n_tiles * m_tiles;
    if ((int) blockIdx.x >= total) return;
    const int nsteps = (int) (a.K / kT8Step);
    const int n_items = (total - (int) blockIdx.x + (int) gridDim.x - 1) / (int) gridDim.x;
    const int gsteps = n_items * nsteps;

    if (tid == 0) {
        for (int i = 0; i < kT8Stages; ++i) {
            mbar_init(&S.full[i], 128);
            mbar_init(&S.empty[i], 1);
            mbar_init(&S.bfull[i], 1);
        }
        for (int i = 0; i < 2; ++i) {
            mbar_init(&S.acc_full[i], 1);
            mbar_init(&S.acc_empty[i], 32 * kQ8EpiWarps);
        }
        for (int i = 0; i < kT8EpStages; ++i) {
            mbar_init(&S.ep_full[i], 128);
            mbar_init(&S.ep_empty[i], 32 * kQ8EpiWarps);
        }
        mbar_init(&S.drain, 1);
        S.abort = 0;
        fence_mbar_init();
    }
    if (warp == kT8WarpMma) {
        umma::tmem_alloc(&S.tmem, kT8TmemCols);
        umma::tmem_relinquish();
    }
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tbase = S.tmem;

    if (warp < kT8WarpMma) {
        // ------------------------------------------------------------ producers
        const int r = tid;  // weight row / token row of this thread (repack, scales)
        int c_item = -1, c_tile = 0, c_rows = 0;
        int n_issued = 0, n_seen = 0;
        const uint8_t *wbase = nullptr;  // row 0 of the item's 128 weight rows (null: invalid expert)
        auto item_state = [&](int k) {
            if (k == c_item) return;
            c_item = k;
            const T8Item x = t8_item(a, m_tiles, (int) blockIdx.x + k * (int) gridDim.x);
            wbase = x.slot >= 0 ? a.W + (size_t) x.slot * a.nb2 + (size_t) x.mt * kT8M * a.nb1 : nullptr;
            c_rows = x.rows;
            c_tile = x.tile;
        };
        // copies of global step g: the step's B codes and scales (bulk) and, on even steps,
        // the raw 8-block group (272 bytes, 16-byte aligned) of every row the step starts:
        // chunk c = row * 17 + piece, thread t taking chunks t, t + 128, ... (consecutive
        // lanes read consecutive pieces of a row: a warp touches ~3 rows per copy, not 32)
        auto issue = [&](int g) {
            if (g < gsteps) {
                const int k = g / nsteps, s = g - k * nsteps, st = g % kT8Stages;
                item_state(k);
                if (g >= kT8Stages) {
                    if (!pf_wait_warp(&S.empty[st], ((g / kT8Stages) & 1) ^ 1, abort, a.st)) {
                        cp_async_commit();
                        return false;
                    }
                }
                if (r == 0) {
                    const size_t ts = (size_t) c_tile * nsteps + s;
                    mbar_arrive_expect_tx(&S.bfull[st], (uint32_t) kT8B + kQ8DaBytes);
                    bulk_g2s(S.b[st], a.btiles + ts * kT8B, (uint32_t) kT8B, &S.bfull[st]);
                    bulk_g2s(S.dstage[st], a.bda + ts * (kQ8DaBytes / 4), kQ8DaBytes, &S.bfull[st]);
                }
                n_issued = g + 1;
                if ((s & 1) == 0) {
                    const int u = s >> 1, rs = (g >> 1) & 1;
                    constexpr int kPieces = kQ8RawRow / 16;  // 17
#pragma unroll
                    for (int it = 0; it < kPieces; ++it) {
                        const int c = it * 128 + r, row = c / kPieces, pc = c - row * kPieces;
                        const bool in = wbase && row < c_rows;
                        const uint8_t *src = in ? wbase + (size_t) row * a.nb1 + (size_t) u * kQ8RawRow + 16 * pc : a.W;
                        cp_async16(&S.raw[rs][c * 16], src, in);
                    }
                }
            }
            cp_async_commit();
            return true;
        };
        bool ok = issue(0);
        ok = ok && issue(1);
        for (int g = 0; g < gsteps; ++g) {
            producers_sync();  // step g - 1 repacked by every producer: its raw group may be refilled
            if (ok && !*abort) ok = issue(g + 2);
            cp_async_wait<2>();
            producers_sync();
            if (!ok || *abort) {
                ok = false;
                continue;
            }
            const int k = g / nsteps, s = g - k * nsteps, st = g % kT8Stages, rs = (g >> 1) & 1;
            item_state(k);
            if (r == 0) T8TRACE(3, g);
            const int es = g % kT8EpStages;
            if (!(ok = pf_wait_warp(&S.ep_empty[es], ((g / kT8EpStages) & 1) ^ 1, abort, a.st))) continue;
            if (!(ok = pf_wait_warp(&S.bfull[st], (g / kT8Stages) & 1, abort, a.st))) continue;
            n_seen = g + 1;
            auto &ep = S.ep[es];
            uint8_t *A = S.a[st];
            // blocks 4 h .. 4 h + 3 of the group: 2-byte aligned codes -> two 16-byte
            // core-matrix rows each (a warp's 32 rows store 512 contiguous bytes)
            const uint8_t *rowp = S.raw[rs] + r * kQ8RawRow;
            if (s & 1) q8_repack_half<1>(rowp, A, r, ep.dw);
            else q8_repack_half<0>(rowp, A, r, ep.dw);
#pragma unroll
            for (int bb = 0; bb < kQ8Blk; ++bb) ep.da[bb][r] = S.dstage[st][bb * kT8N + r];
            if (r == 0) T8TRACE(0, g);
            fence_proxy_async_smem();
            asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&S.full[st])) : "memory");
            asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(&S.ep_full[es])) : "memory");
        }
        cp_async_wait<0>();
        if (r == 0) {
            for (int g = n_seen; g < n_issued; ++g) mbar_wait(&S.bfull[g % kT8Stages], (g / kT8Stages) & 1);
        }
    } else if (warp == kT8WarpMma) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            uint32_t acc_i = 0;
            bool ok = true;
            for (int g = 0; g < gsteps && ok; ++g) {
                const int k = g / nsteps, st = g % kT8Stages;
                const T8Item x = t8_item(a, m_tiles, (int) blockIdx.x + k * (int) gridDim.x);
                const uint32_t idesc = umma::idesc_i8(kT8M, x.Nt);
                if (!(ok = pf_wait(&S.full[st], (g / kT8Stages) & 1, abort, a.st))) break;
                if (!(ok = pf_wait(&S.bfull[st], (g / kT8Stages) & 1, abort, a.st))) break;
                umma::fence_after_sync();
                const uint32_t a_s = smem_u32(S.a[st]), b_s = smem_u32(S.b[st]);
                // half-step hs (blocks 2 hs, 2 hs + 1) into accumulator buffer (count & 1)
                for (int hs = 0; hs < 2 && ok; ++hs) {
                    const int rg = (int) (acc_i & 1);
                    if (!(ok = pf_wait(&S.acc_empty[rg], ((acc_i >> 1) & 1) ^ 1, abort, a.st))) break;
                    umma::fence_after_sync();
#pragma unroll
                    for (int bb = 0; bb < 2; ++bb) {
                        const int b = 2 * hs + bb;
                        umma::mma_i8_ss(tbase + (uint32_t) rg * 256 + (uint32_t) bb * 128,
                                        umma::sdesc(a_s + 2 * b * kT8Lbo, kT8Lbo, 128),
                                        umma::sdesc(b_s + 2 * b * kT8Lbo, kT8Lbo, 128), idesc, 0u);
                    }
                    umma::commit(&S.acc_full[rg]);
                    ++acc_i;
                }
                if (ok) umma::commit(&S.empty[st]);
                T8TRACE(1, g);
            }
            umma::commit(&S.drain);
            mbar_wait(&S.drain, 0);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        // warp w reads TMEM lanes 32 (w % 4) .. + 31 (weight rows); warpgroup g = token
        // columns 32 g .. 32 g + 31
        const int qd = warp & 3, g = (warp - kT8WarpEpi) >> 2, m = qd * 32 + lane;
        const uint32_t lane_base = (uint32_t) (qd * 32) << 16;
        uint32_t acc_i = 0;
        bool ok = true;
        int gstep = 0;
        for (int k = 0; k < n_items && ok; ++k) {
            const T8Item x = t8_item(a, m_tiles, (int) blockIdx.x + k * (int) gridDim.x);
            // output offset (floats) of token column 32 g + lane
            uint32_t off = 0;
            {
                const int n = 32 * g + lane;
                if (n < x.cnt) {
                    const int p = __ldg(a.pairs + x.p0 + n);
                    const int t = p / a.n_used, j = p - t * a.n_used;
                    off = (uint32_t) (((size_t) j * a.dnb1 + (size_t) t * a.dnb2) >> 2);
                }
            }
            const bool cols = 32 * g < x.Nt;  // warp-uniform: this warpgroup has tokens
            float out[32];
#pragma unroll
            for (int i = 0; i < 32; ++i) out[i] = 0.f;
            for (int s = 0; s < nsteps && ok; ++s, ++gstep) {
                const int es = gstep % kT8EpStages;
                if (!(ok = pf_wait_warp(&S.ep_full[es], (gstep / kT8EpStages) & 1, abort, a.st))) break;
                const auto &ep = S.ep[es];
                for (int hs = 0; hs < 2; ++hs) {
                    const int rg = (int) (acc_i & 1);
                    if (!(ok = pf_wait_warp(&S.acc_full[rg], (acc_i >> 1) & 1, abort, a.st))) break;
                    umma::fence_after_sync();
                    if (cols) {
#pragma unroll
                        for (int bb = 0; bb < 2; ++bb) {
                            const int b = 2 * hs + bb;
                            const float dw = ep.dw[b][m];
                            const float2 dw2 = make_float2(dw, dw);
                            const float2 *da2 = (const float2 *) &ep.da[b][32 * g];
                            // the block's 32 columns in one load and one wait
                            uint32_t v[32];
                            umma::ld32(tbase + lane_base + (uint32_t) rg * 256 + (uint32_t) bb * 128 + 32 * g, v);
                            umma::wait_ld();
                            // out += (d_w * d_a) * (float) isum, two columns per packed f32x2
                            // instruction; (float) isum as the exact bit trick
                            // (1.5 * 2^23 + isum) - 1.5 * 2^23, |isum| <= 32 * 127 * 128 < 2^22
#pragma unroll
                            for (int i = 0; i < 32; i += 2) {
                                float2 f = make_float2(__int_as_float((int) v[i] + 0x4B400000),
                                                       __int_as_float((int) v[i + 1] + 0x4B400000));
                                f = __fadd2_rn(f, make_float2(-12582912.f, -12582912.f));
                                const float2 sc = __fmul2_rn(dw2, da2[i / 2]);
                                float2 o = make_float2(out[i], out[i + 1]);
                                o = __ffma2_rn(sc, f, o);
                                out[i] = o.x;
                                out[i + 1] = o.y;
                            }
                        }
                    }
                    umma::fence_before_sync();
                    warp_arrive(&S.acc_empty[rg]);
                    ++acc_i;
                }
                if (!ok) break;
                warp_arrive(&S.ep_empty[es]);
                if (warp == kT8WarpEpi && lane == 0) T8TRACE(2, gstep);
            }
            if (!ok) break;
            const int64_t row = (int64_t) x.mt * kT8M + m;
#pragma unroll
            for (int i = 0; i < 32; ++i) {
                const uint32_t o = __shfl_sync(0xffffffffu, off, i);
                if (m < x.rows && 32 * g + i < x.cnt) a.dst[(size_t) o + row] = out[i];
            }
            if (x.slot < 0 && x.mt == 0 && m == 0 && g == 0) report(a.st, QWB_DEVERR_ID_RANGE, a.tiles[x.tile].x);
        }
    }

    umma::fence_before_sync();
    __syncthreads();
    if (warp == kT8WarpMma) {
        umma::fence_after_sync();
        umma::tmem_dealloc(tbase, kT8TmemCols);
    }
}

}  // namespace

size_t tc8_btile_stride(int64_t K) { return (size_t) (K / kT8Step) * kT8B; }
size_t tc8_da_stride(int type, int64_t K) {
    return (size_t) (K / kT8Step) * (type == QWB_TYPE_Q8_0 ? kQ8DaBytes : kT8DaBytes);
}

cudaError_t launch_tc8_gather(int type, Q8Planes act, int act_dstride, int64_t K, const int4 *tiles,
                              const int *n_tiles, int max_tiles, const int *pairs, int n_used, int n_b,
                              uint8_t *btiles, float *bda, cudaStream_t s) {
    if (max_tiles <= 0) return cudaSuccess;
    dim3 grid((unsigned) max_tiles, (unsigned) (K / kT8Step));
    if (type == QWB_TYPE_Q8_0)
        tc8_gather_kernel<true><<<grid, 256, 0, s>>>(act, act_dstride, K, tiles, n_tiles, pairs, n_used, n_b, btiles, bda);
    else
        tc8_gather_kernel<false><<<grid, 256, 0, s>>>(act, act_dstride, K, tiles, n_tiles, pairs, n_used, n_b, btiles, bda);
    return cudaGetLastError();
}

cudaError_t launch_pf_tc8(int type, const I8PrefillArgs &a, cudaStream_t s) {
    if (type == QWB_TYPE_Q8_0) {
        const size_t smem = sizeof(Q8Smem);
        static DeviceSmemLimit limit;
        cudaError_t e = ensure_dyn_smem(pf_tc8q_kernel, smem, limit);
        if (e != cudaSuccess) return e;
        pf_tc8q_kernel<<<num_sms(), kQ8Threads, smem, s>>>(a);
        return cudaGetLastError();
    }
    const size_t smem = sizeof(T8Smem);
    static DeviceSmemLimit limit;
    cudaError_t e = ensure_dyn_smem(pf_tc8_kernel, smem, limit);
    if (e != cudaSuccess) return e;
    pf_tc8_kernel<<<num_sms(), kT8Threads, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace qwb

#ifdef QWB_DECODE_TRACE
extern "C" QWB_API int qwb_debug_tc8_trace(void *host, size_t bytes) {
    return cudaMemcpyFromSymbol(host, qwb::g_tc8_trace, bytes) == cudaSuccess ? 0 : 1;
}
#endif
