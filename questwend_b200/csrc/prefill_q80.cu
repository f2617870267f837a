// prefill_q80.cu - MUL_MAT_ID on Q8_0 experts with many tokens per expert (prefill) on
// the integer tensor cores.
//
// Reference arithmetic: ggml_vec_dot_q8_0_q8_0 (ggml-cpu/quants.c:451-480), used by
// ggml_compute_forward_mul_mat_id (ggml-cpu/ggml-cpu.c:1554-1736) with the activations
// quantized to Q8_0 (CPU variant): for every 32-element block j,
//     sumf += (float) isum_j * (d_w,j * d_a,j)      isum_j = sum q_w * q_a (exact int32)
// One `mma.sync.m16n8k32.s32.s8.s8` is exactly that block's integer dot for a 16-row x
// 8-token fragment; the epilogue of each block scales it by d_w * d_a in fp32 and adds it
// to the running sums in block order, as the CPU does.
//
// Work item = (expert tile of <= 64 routed (token, slot) pairs, 128 weight rows); one
// persistent CTA per SM takes items from a counter the index kernel zeroed.  8 warps, each
// a 32-row x 32-token tile (2 x 4 fragments).  Per K step of 256 (8 blocks):
//   * cp.async (16 B per thread, double-buffered) brings the 128 weight rows' raw 272-byte
//     block groups and the tile's 64 activation rows (qs + per-block scales) to shared
//     memory; no spin waits (cp.async groups + block barriers);
//   * the raw Q8_0 blocks (2-byte scale + 32 codes, 34 B) are repacked into codes only, in
//     a bank-padded layout (272-byte row stride) for ldmatrix, and fp32 weight scales;
//   * 8 blocks x 8 MMAs per warp, each followed by its scale-and-add epilogue.
#include <algorithm>

#include "common.cuh"
#include "dot.cuh"
#include "kernels.cuh"
#include "mmid.cuh"

namespace qwb {

namespace {

constexpr int kQ8TM = 128;        // weight rows per item
constexpr int kQ8TN = 64;         // token pairs per item (index tile size)
constexpr int kQ8KS = 256;        // K per step (8 Q8_0 blocks)
constexpr int kQ8Raw = 272;       // raw bytes per row per step (8 x 34)
constexpr int kQ8Row = 272;       // padded code row stride in shared memory (256 + 16)
constexpr int kQ8Threads = 256;

struct Q8Smem {
    uint8_t raw[2][kQ8TM][kQ8Raw];      // raw weight block groups (cp.async)
    uint8_t wq[kQ8TM][kQ8Row];          // repacked weight codes
    uint8_t aq[2][kQ8TN][kQ8Row];       // activation codes (cp.async straight from the planes)
    float dw[kQ8TM][8];                 // weight scales of the step
    float da[2][kQ8TN][8];              // activation scales (cp.async)
    long long tok_o[kQ8TN];             // output byte offset of each pair (-1: none)
    int tok_ar[kQ8TN];                  // activation plane row of each pair
    int item;
};

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait0() { asm volatile("cp.async.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void mma_s8(int *c, const uint32_t *a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Issue the copies of K step `ks` of the current item into buffer `buf`.
__device__ __forceinline__ void q80_issue(const Q8PrefillArgs &a, Q8Smem &S, int buf, int ks, const uint8_t *wbase,
                                          int nrows, int ntok) {
    const int tid = threadIdx.x;
    // weights: 128 rows x 17 pieces of 16 B
    for (int i = tid; i < kQ8TM * (kQ8Raw / 16); i += kQ8Threads) {
        const int r = i / (kQ8Raw / 16), c = i - r * (kQ8Raw / 16);
        const bool ok = r < nrows;
        const uint8_t *src = wbase + (size_t) (ok ? r : 0) * a.nb1 + (size_t) ks * kQ8Raw + 16 * c;
        cp_async16(&S.raw[buf][r][16 * c], src, ok);
    }
    // activation codes: 64 tokens x 16 pieces; scales: 64 tokens x 2 pieces
    for (int i = tid; i < kQ8TN * 18; i += kQ8Threads) {
        const int k = i / 18, c = i - k * 18;
        const bool ok = k < ntok;
        const int64_t ar = ok ? S.tok_ar[k] : 0;
        if (c < 16) {
            cp_async16(&S.aq[buf][k][16 * c], a.act.qs + ar * a.K + (int64_t) ks * kQ8KS + 16 * c, ok);
        } else {
            cp_async16(&S.da[buf][k][4 * (c - 16)], a.act.d + ar * a.act_dstride + (int64_t) ks * 8 + 4 * (c - 16), ok);
        }
    }
    cp_async_commit();
}

__global__ void __launch_bounds__(kQ8Threads, 1) pf_q80_kernel(const Q8PrefillArgs a) {
    extern __shared__ __align__(128) uint8_t smem_raw[];
    Q8Smem &S = *(Q8Smem *) smem_raw;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp & 3, wn = warp >> 2;  // warp tile: rows 32*wm.., tokens 32*wn..
    const int n_rb = (int) ceil_div(a.M, kQ8TM);
    const int64_t n_items = (int64_t) (*a.n_tiles) * n_rb;
    const int nks = (int) (a.K / kQ8KS);

    for (int64_t item = blockIdx.x;;) {
        if (item >= n_items) break;
        const int4 t = a.tiles[item / n_rb];  // (expert, first pair, pair count)
        const int rb = (int) (item % n_rb);
        const int64_t r0 = (int64_t) rb * kQ8TM;
        const int nrows = (int) min((int64_t) kQ8TM, a.M - r0);
        const int ntok = t.z;
        const int64_t e = (t.x >= 0 && t.x < a.n_as) ? t.x : -1;
        __syncthreads();  // the previous item's buffers are no longer read
        if (tid < kQ8TN) {
            if (tid < ntok) {
                const int p = a.pairs[t.y + tid];
                const int tt = p / a.n_used, j = p - tt * a.n_used;
                S.tok_ar[tid] = tt * a.n_b + j % a.n_b;
                S.tok_o[tid] = (long long) ((size_t) j * a.dnb1 + (size_t) tt * a.dnb2);
            } else {
                S.tok_ar[tid] = 0;
                S.tok_o[tid] = -1;
            }
        }
        if (tid == 0) {
            const int64_t nx = (int64_t) gridDim.x + atomicAdd(a.work, 1);
            S.item = (int) (nx < n_items ? nx : n_items);
        }
        __syncthreads();
        const int64_t next = S.item;
        if (e < 0) {  // expert id outside the pool (cannot happen from the index): zeros
            for (int i = tid; i < nrows * ntok; i += kQ8Threads) {
                const int r = i / ntok, k = i - r * ntok;
                ((float *) ((char *) a.dst + S.tok_o[k]))[r0 + r] = 0.f;
            }
            item = next;
            continue;
        }
        const uint8_t *wbase = a.W + (size_t) e * a.nb2 + (size_t) r0 * a.nb1;

        float acc[2][4][4];
#pragma unroll
        for (int mi = 0; mi < 2; ++mi)
#pragma unroll
            for (int ni = 0; ni < 4; ++ni)
#pragma unroll
                for (int v = 0; v < 4; ++v) acc[mi][ni][v] = 0.f;

        q80_issue(a, S, 0, 0, wbase, nrows, ntok);
        for (int ks = 0; ks < nks; ++ks) {
            const int buf = ks & 1;
            if (ks + 1 < nks) {
                q80_issue(a, S, buf ^ 1, ks + 1, wbase, nrows, ntok);
                cp_async_wait1();
            } else {
                cp_async_wait0();
            }
            __syncthreads();  // step ks has landed for every thread
            // repack: row r (threads 2r, 2r+1 take 4 blocks each): 2-byte scale + 32 codes
            {
                const int r = tid >> 1, half = tid & 1;
                const uint8_t *src = S.raw[buf][r] + 136 * half;  // 4 blocks of 34 B
                uint8_t *dst = S.wq[r] + 128 * half;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const uint8_t *blk = src + 34 * b;  // 2-byte aligned
                    S.dw[r][4 * half + b] = h2f(*(const uint16_t *) blk);
                    uint32_t w[8];
                    lds_words8_a2(blk + 2, w);
                    uint4 *d4 = (uint4 *) (dst + 32 * b);
                    d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
                    d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
                }
            }
            __syncthreads();
            // 8 blocks of 32: MMA + scale-and-add
            const uint32_t wq_base = smem_u32(&S.wq[0][0]), aq_base = smem_u32(&S.aq[buf][0][0]);
#pragma unroll 2
            for (int j = 0; j < 8; ++j) {
                uint32_t af[2][4];
#pragma unroll
                for (int mi = 0; mi < 2; ++mi) {
                    const int row = 32 * wm + 16 * mi + (lane & 7) + ((lane >> 3) & 1) * 8;
                    const int col = 32 * j + (lane >> 4) * 16;
                    ldsm_x4(wq_base + row * kQ8Row + col, af[mi][0], af[mi][1], af[mi][2], af[mi][3]);
                }
                uint32_t bf[4][2];
#pragma unroll
                for (int np = 0; np < 2; ++np) {
                    // tokens 32*wn + 16*np + (lane&7) + 8*(lane>>4), bytes 32j + 16*((lane>>3)&1)
                    const int tok = 32 * wn + 16 * np + (lane & 7) + 8 * (lane >> 4);
                    const int col = 32 * j + 16 * ((lane >> 3) & 1);
                    ldsm_x4(aq_base + tok * kQ8Row + col, bf[2 * np][0], bf[2 * np][1], bf[2 * np + 1][0],
                            bf[2 * np + 1][1]);
                }
                float dwr[2][2], dat[4][2];
#pragma unroll
                for (int mi = 0; mi < 2; ++mi) {
                    const int row = 32 * wm + 16 * mi + (lane >> 2);
                    dwr[mi][0] = S.dw[row][j];
                    dwr[mi][1] = S.dw[row + 8][j];
                }
#pragma unroll
                for (int ni = 0; ni < 4; ++ni) {
                    const int tok = 32 * wn + 8 * ni + 2 * (lane & 3);
                    dat[ni][0] = S.da[buf][tok][j];
                    dat[ni][1] = S.da[buf][tok + 1][j];
                }
#pragma unroll
                for (int mi = 0; mi < 2; ++mi) {
#pragma unroll
                    for (int ni = 0; ni < 4; ++ni) {
                        int c[4];
                        mma_s8(c, af[mi], bf[ni][0], bf[ni][1]);
                        // c0: (row g, tok 2q), c1: (g, 2q+1), c2: (g+8, 2q), c3: (g+8, 2q+1)
                        acc[mi][ni][0] += (float) c[0] * __fmul_rn(dwr[mi][0], dat[ni][0]);
                        acc[mi][ni][1] += (float) c[1] * __fmul_rn(dwr[mi][0], dat[ni][1]);
                        acc[mi][ni][2] += (float) c[2] * __fmul_rn(dwr[mi][1], dat[ni][0]);
                        acc[mi][ni][3] += (float) c[3] * __fmul_rn(dwr[mi][1], dat[ni][1]);
                    }
                }
            }
            __syncthreads();  // wq and this step's buffers are free again
        }
        // outputs: dst[row] of each (token, slot) pair
#pragma unroll
        for (int mi = 0; mi < 2; ++mi) {
#pragma unroll
            for (int ni = 0; ni < 4; ++ni) {
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const int row = 32 * wm + 16 * mi + (lane >> 2) + 8 * (v >> 1);
                    const int tok = 32 * wn + 8 * ni + 2 * (lane & 3) + (v & 1);
                    if (row < nrows && tok < ntok)
                        ((float *) ((char *) a.dst + S.tok_o[tok]))[r0 + row] = acc[mi][ni][v];
                }
            }
        }
        item = next;
    }
}

}  // namespace

bool pf_q80_eligible(int type, int64_t K, int64_t M, int64_t P, int64_t n_as, const void *W, size_t nb1, size_t nb2) {
    if (type != QWB_TYPE_Q8_0 || K % kQ8KS || K < kQ8KS || M < 1) return false;
    if (((uintptr_t) W | nb1 | nb2) % 16) return false;  // 16-byte copies of whole block groups
    const int64_t used = std::min<int64_t>(P, n_as);
    return used > 0 && P >= 32 * used;
}

int pf_q80_tile_tokens() { return kQ8TN; }

cudaError_t launch_pf_q80(const Q8PrefillArgs &a, cudaStream_t s) {
    const size_t smem = sizeof(Q8Smem);
    static bool configured = false;
    if (!configured) {
        cudaError_t e = cudaFuncSetAttribute(pf_q80_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
        if (e != cudaSuccess) return e;
        configured = true;
    }
    pf_q80_kernel<<<num_sms(), kQ8Threads, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace qwb
