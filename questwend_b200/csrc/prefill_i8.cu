// prefill_i8.cu - MUL_MAT_ID on Q8_0 and Q6_K experts with many tokens per expert
// (prefill) on the integer tensor cores.
//
// Reference arithmetic (ggml_compute_forward_mul_mat_id, ggml-cpu/ggml-cpu.c:1554-1736):
//   Q8_0 x Q8_0 (ggml-cpu/quants.c:451-480), activations quantized to Q8_0 (CPU variant):
//       for every 32-element block j:  sumf += (float) isum_j * (d_w,j * d_a,j)
//   Q6_K x Q8_K (ggml-cpu/quants.c:851-915): for every superblock of 256,
//       sumf += (d_w * d_a) * (float) sum_s sc_s * isum_s   over its 16 sub-blocks of 16,
//       isum_s = sum (q6 - 32) * q_a, sc_s the sub-block's int8 scale.
// Integer products and sums are exact; mma.sync s8 x s8 -> s32 computes them for a
// 16-row x 8-token fragment: one m16n8k32 per Q8_0 block, one m16n8k16 per Q6_K sub-block
// (whose integer scale is applied in int32, the fp32 scale once per superblock).
//
// Work item = (expert tile of <= TN routed (token, slot) pairs, 128 weight rows); one
// persistent CTA per SM takes items from a counter the index kernel zeroed.  TN = 64 (32 or
// more pairs per expert): 8 warps, each a 32-row x 32-token tile (2 x 4 fragments);
// TN = 8 (8 to 31 pairs per expert, e.g. the output head at 8 tokens): 8 warps of 16 rows
// x 8 tokens, so few tokens do not pay for 64-token MMAs.  Per K step of 256:
//   * cp.async (16 B per thread, double-buffered) brings the 128 weight rows' raw block
//     bytes of the step (Q8_0: 8 blocks of 34 B = 272 B; Q6_K: one 210-byte superblock,
//     widened to 16-byte boundaries) and the tile's 64 activation rows (codes + scales) to
//     shared memory; no spin waits (cp.async groups + block barriers);
//   * the raw blocks are repacked into int8 codes in a bank-padded layout (272-byte row
//     stride) for ldmatrix, with fp32 (and, for Q6_K, int8 sub-block) scales;
//   * the MMAs of the step, each followed by its scale epilogue.
// Q8_0 block scaling without an int -> float conversion instruction: each MMA adds the
// integer dot to the accumulator input 0x4B400000, the bit pattern of 1.5 * 2^23, so the
// int32 result read as a float is exactly 12582912 + isum (|isum| <= 32 * 128 * 127 <
// 2^22 keeps it in [2^23, 2^24), where floats are the consecutive integers).  Then
// t = fma(y, d_a, -12582912 * d_a) = round(isum * d_a): y * d_a is exact inside the fma
// and 12582912 * d_a is exact in fp32 (d_a comes from fp16: 11 significant bits, times
// the 2 bits of 3 * 2^22), and acc = fma(t, d_w, acc).
#include <algorithm>

#include "common.cuh"
#include "dot.cuh"
#include "kernels.cuh"
#include "mmid.cuh"

namespace qwb {

namespace {

constexpr int kI8TM = 128;      // weight rows per item
constexpr int kI8TNBig = 64;    // token pairs per item (index tile size), many tokens per expert
constexpr int kI8TNSmall = 8;   // ... 8 to 31 tokens per expert
constexpr int kI8KS = 256;      // K per step
constexpr int kI8Row = 272;     // padded code row stride in shared memory (256 + 16)
constexpr int kI8Threads = 256;

template <int TYPE>
struct I8Geo {
    static constexpr bool q6 = TYPE == QWB_TYPE_Q6_K;
    static constexpr int raw = q6 ? 240 : 272;  // raw bytes staged per row per step
    static constexpr int ndw = 1;               // Q6_K: fp32 weight scale per row per step
    static constexpr int nda = q6 ? 4 : 8;      // activation scale floats staged per token per step
    static constexpr int nj = q6 ? 1 : 8;       // Q8_0: blocks per row per step (repacked scales)
};

constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23, bit pattern 0x4B400000
constexpr int kMagicBits = 0x4B400000;

// Copy pipeline depth D: K steps whose copies are in flight.  A 64-token step's MMAs take
// about one memory latency, so one step ahead (D = 2) hides it; an 8-token step computes
// little and keeps more steps in flight (3 for Q8_0, 4 for Q6_K: what 227 KB allows).
template <int TYPE, int TN>
struct I8Depth {
    static constexpr int D = TN == kI8TNBig ? 2 : (TYPE == QWB_TYPE_Q8_0 ? 3 : 4);
};

// Pipeline slots of K step ks: copies land in raw / off [ks % D] and aq / da [ks % (D + 1)];
// the repack writes wq / dw / dwp / dap / sc [ks & 1].  In the iteration of step ks the MMAs
// read step ks while the repack writes step ks + 1 and the copies of step ks + D land.
template <int TYPE, int TN>
struct I8Smem {
    static constexpr int D = I8Depth<TYPE, TN>::D;
    uint8_t raw[D][kI8TM][I8Geo<TYPE>::raw];  // raw weight bytes (cp.async)
    uint8_t wq[2][kI8TM][kI8Row];             // repacked int8 codes
    uint8_t aq[D + 1][TN][kI8Row];            // activation codes (cp.async from the planes)
    float dw[2][kI8TM][I8Geo<TYPE>::ndw];     // Q6_K: weight scale of the step
    // Q8_0: weight scales of block j for the rows one lane reads, (g, g+8, g+16, g+24) of its
    // warp's 32 rows; and activation scales of token pair k (tokens 2k, 2k+1) of block j as
    // {d(2k), d(2k+1), -kMagic d(2k), -kMagic d(2k+1)} (stride 33 pairs: no bank conflicts)
    float dwp[2][I8Geo<TYPE>::nj][4][8][4];
    float dap[2][I8Geo<TYPE>::nj][I8Geo<TYPE>::q6 ? 1 : TN / 2 + 1][4];
    int sc[2][I8Geo<TYPE>::q6 ? kI8TM : 1][16];  // Q6_K sub-block scales of the step
    float da[D + 1][TN][I8Geo<TYPE>::nda];       // activation scales (cp.async)
    int off[D][kI8TM];                           // Q6_K: offset of the superblock in its raw row
    long long tok_o[TN];                      // output byte offset of each pair
    int tok_ar[TN];                           // activation plane row of each pair
    int item;
};

static_assert(sizeof(I8Smem<QWB_TYPE_Q8_0, kI8TNBig>) <= 232448 && sizeof(I8Smem<QWB_TYPE_Q6_K, kI8TNBig>) <= 232448 &&
                  sizeof(I8Smem<QWB_TYPE_Q8_0, kI8TNSmall>) <= 232448 &&
                  sizeof(I8Smem<QWB_TYPE_Q6_K, kI8TNSmall>) <= 232448,
              "one CTA per SM: at most 227 KB of shared memory");

__device__ __forceinline__ void cp_async16(void *dst, const void *src, bool valid) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(valid ? 16 : 0)
                 : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// wait until at most N of this thread's most recent copy groups are still pending
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x2(uint32_t addr, uint32_t &r0, uint32_t &r1) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x2.shared.b16 {%0,%1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
}

// one 32-element block (m16n8k32) of A = {a0..a3} and B = {b0, b1}, added to `bias`
__device__ __forceinline__ void mma_k32(int *c, const uint32_t *a, uint32_t b0, uint32_t b1, int bias) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1), "r"(bias));
}
// one 16-element sub-block (m16n8k16) of A = {a0, a1} and B = {b0}
__device__ __forceinline__ void mma_k16(int *c, uint32_t a0, uint32_t a1, uint32_t b0) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}

// Issue the copies of K step `ks` of the current item into its slots.
template <int TYPE, int TN>
__device__ __forceinline__ void i8_issue(const I8PrefillArgs &a, I8Smem<TYPE, TN> &S, int ks, const uint8_t *wbase,
                                         int nrows, int ntok) {
    using G = I8Geo<TYPE>;
    constexpr int D = I8Depth<TYPE, TN>::D;
    const int tid = threadIdx.x;
    const int buf = ks % D, b3 = ks % (D + 1);
    constexpr int pieces = G::raw / 16;
    for (int i = tid; i < kI8TM * pieces; i += kI8Threads) {
        const int r = i / pieces, c = i - r * pieces;
        const bool ok = r < nrows;
        const uint8_t *row = wbase + (size_t) (ok ? r : 0) * a.nb1;
        const uint8_t *src;
        if constexpr (G::q6) {
            // the 210-byte superblock widened to 16-byte boundaries (<= 15 pieces)
            const uintptr_t s0 = (uintptr_t) (row + (size_t) ks * Q6K_BYTES);
            const uintptr_t a0 = s0 & ~(uintptr_t) 15;
            const bool in = ok && (a0 + 16 * c < s0 + Q6K_BYTES);
            if (c == 0) S.off[buf][r] = (int) (s0 - a0);
            src = (const uint8_t *) (in ? a0 + 16 * c : a0);
            cp_async16(&S.raw[buf][r][16 * c], src, in);
        } else {
            src = row + (size_t) ks * 272 + 16 * c;
            cp_async16(&S.raw[buf][r][16 * c], src, ok);
        }
    }
    constexpr int dpieces = G::nda / 4;
    for (int i = tid; i < TN * (16 + dpieces); i += kI8Threads) {
        const int k = i / (16 + dpieces), c = i - k * (16 + dpieces);
        const bool ok = k < ntok;
        const int64_t ar = ok ? S.tok_ar[k] : 0;
        if (c < 16) {
            cp_async16(&S.aq[b3][k][16 * c], a.act.qs + ar * a.K + (int64_t) ks * kI8KS + 16 * c, ok);
        } else if constexpr (G::q6) {
            // one scale per superblock: the 16-byte group of 4 holding it
            cp_async16(&S.da[b3][k][0], a.act.d + ar * a.act_dstride + (ks & ~3), ok);
        } else {
            cp_async16(&S.da[b3][k][4 * (c - 16)], a.act.d + ar * a.act_dstride + (int64_t) ks * 8 + 4 * (c - 16), ok);
        }
    }
    cp_async_commit();
}

// Repack row r's raw bytes of step ks (two threads per row) into int8 codes + scales.
template <int TYPE, int TN>
__device__ __forceinline__ void i8_repack(I8Smem<TYPE, TN> &S, int ks, int tid) {
    constexpr int D = I8Depth<TYPE, TN>::D;
    const int r = tid >> 1, half = tid & 1;
    const int buf = ks & 1, rb = ks % D, b3 = ks % (D + 1);  // repacked / raw / activation slots
    if constexpr (TYPE == QWB_TYPE_Q8_0) {
        const uint8_t *src = S.raw[rb][r] + 136 * half;  // 4 blocks of 34 B
        uint8_t *dst = S.wq[buf][r] + 128 * half;
        // row r = 32 wm + 16 mi + 8 h + g is slot 2 mi + h of lane group g in warp row wm
        const int wm = r >> 5, g = r & 7, slot = ((r >> 3) & 3);
#pragma unroll
        for (int b = 0; b < 4; ++b) {
            const uint8_t *blk = src + 34 * b;  // 2-byte aligned
            S.dwp[buf][4 * half + b][wm][g][slot] = h2f(*(const uint16_t *) blk);
            uint32_t w[8];
            lds_words8_a2(blk + 2, w);
            uint4 *d4 = (uint4 *) (dst + 32 * b);
            d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
            d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
        // activation scales of token pair k, block j (8 threads per pair)
        if (tid < 4 * TN) {
            const int k = tid >> 3, j = tid & 7;
            const float d0 = S.da[b3][2 * k][j], d1 = S.da[b3][2 * k + 1][j];
            *(float4 *) &S.dap[buf][j][k][0] = make_float4(d0, d1, -kMagic * d0, -kMagic * d1);
        }
    } else {
        // Q6_K superblock: ql[128] qh[64] sc[16] d; element 128*hf + 32*i + l has ql nibble
        // (ql[64hf + 32(i&1) + l], high when i >= 2) and qh bits 2i..2i+1 of qh[32hf + l]
        const uint8_t *sb = S.raw[rb][r] + S.off[rb][r];  // 2-byte aligned
        const int hf = half;
        uint32_t qa[8], qb[8], qh[8];
        lds_words8_a2(sb + 64 * hf, qa);
        lds_words8_a2(sb + 64 * hf + 32, qb);
        lds_words8_a2(sb + 128 + 32 * hf, qh);
        uint8_t *dst = S.wq[buf][r] + 128 * hf;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            uint32_t w[8];
#pragma unroll
            for (int m = 0; m < 8; ++m) {
                const uint32_t ql = (i & 1) ? qb[m] : qa[m];
                const uint32_t nib = i < 2 ? (ql & 0x0f0f0f0fu) : ((ql >> 4) & 0x0f0f0f0fu);
                w[m] = __vsub4(nib | (((qh[m] >> (2 * i)) & 0x03030303u) << 4), 0x20202020u);
            }
            uint4 *d4 = (uint4 *) (dst + 32 * i);
            d4[0] = make_uint4(w[0], w[1], w[2], w[3]);
            d4[1] = make_uint4(w[4], w[5], w[6], w[7]);
        }
        const int8_t *scp = (const int8_t *) (sb + 192) + 8 * hf;
#pragma unroll
        for (int j = 0; j < 8; ++j) S.sc[buf][r][8 * hf + j] = scp[j];
        if (hf == 0) S.dw[buf][r][0] = h2f(*(const uint16_t *) (sb + 208));
    }
}

// Warp tiling of the 128-row x TN-token item: TN = 64, 4 x 2 warps of 32 rows x 32 tokens
// (MI = 2 row fragments x NI = 4 token fragments); TN = 8, 8 warps of 16 rows x 8 tokens
// (MI = NI = 1, B fragments from a 2-matrix ldmatrix).
template <int TYPE, int TN>
__global__ void __launch_bounds__(kI8Threads, 1) pf_i8_kernel(const I8PrefillArgs a) {
    using G = I8Geo<TYPE>;
    constexpr int D = I8Depth<TYPE, TN>::D;
    constexpr bool big = TN == kI8TNBig;
    constexpr int MI = big ? 2 : 1, NI = big ? 4 : 1;
    extern __shared__ __align__(128) uint8_t smem_raw[];
    I8Smem<TYPE, TN> &S = *(I8Smem<TYPE, TN> *) smem_raw;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row0 = big ? 32 * (warp & 3) : 16 * warp;  // the warp's first row
    const int tok0 = big ? 32 * (warp >> 2) : 0;          // and first token
    const int n_rb = (int) ceil_div(a.M, kI8TM);
    const int64_t n_items = (int64_t) (*a.n_tiles) * n_rb;
    const int nks = (int) (a.K / kI8KS);

    for (int64_t item = blockIdx.x;;) {
        if (item >= n_items) break;
        const int4 t = a.tiles[item / n_rb];  // (expert, first pair, pair count)
        const int rb = (int) (item % n_rb);
        const int64_t r0 = (int64_t) rb * kI8TM;
        const int nrows = (int) min((int64_t) kI8TM, a.M - r0);
        const int ntok = t.z;
        const int64_t e = (t.x >= 0 && t.x < a.n_as) ? t.x : -1;
        __syncthreads();  // the previous item's buffers are no longer read
        if (tid < TN) {
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
            for (int i = tid; i < nrows * ntok; i += kI8Threads) {
                const int r = i / ntok, k = i - r * ntok;
                ((float *) ((char *) a.dst + S.tok_o[k]))[r0 + r] = 0.f;
            }
            item = next;
            continue;
        }
        const uint8_t *wbase = a.W + (size_t) e * a.nb2 + (size_t) r0 * a.nb1;

        float acc[MI][NI][4];
#pragma unroll
        for (int mi = 0; mi < MI; ++mi)
#pragma unroll
            for (int ni = 0; ni < NI; ++ni)
#pragma unroll
                for (int v = 0; v < 4; ++v) acc[mi][ni][v] = 0.f;

        // prologue: steps 0 .. D-1 in flight (one copy group per step, empty past the last
        // step, so group g is always step g), step 0 repacked
#pragma unroll
        for (int st = 0; st < D; ++st) {
            if (st < nks) i8_issue<TYPE, TN>(a, S, st, wbase, nrows, ntok);
            else cp_async_commit();
        }
        cp_async_wait<D - 1>();  // step 0
        __syncthreads();         // step 0 has landed for every thread
        i8_repack<TYPE, TN>(S, 0, tid);
        for (int ks = 0; ks < nks; ++ks) {
            const int buf = ks & 1, b3 = ks % (D + 1);
            cp_async_wait<D - 2>();  // this thread's copies of step ks + 1
            // One barrier per step: step ks + 1 has landed, step ks is repacked, and the
            // MMAs of step ks - 1 are done, so its slots may be refilled / rewritten.
            __syncthreads();
            if (ks + D < nks) i8_issue<TYPE, TN>(a, S, ks + D, wbase, nrows, ntok);
            else cp_async_commit();
            if (ks + 1 < nks) i8_repack<TYPE, TN>(S, ks + 1, tid);
            const uint32_t wq_base = smem_u32(&S.wq[buf][0][0]), aq_base = smem_u32(&S.aq[b3][0][0]);
            int isum[MI][NI][4];  // Q6_K: integer sum of the superblock (sub-block scales applied)
#pragma unroll
            for (int mi = 0; mi < MI; ++mi)
#pragma unroll
                for (int ni = 0; ni < NI; ++ni)
#pragma unroll
                    for (int v = 0; v < 4; ++v) isum[mi][ni][v] = 0;
#pragma unroll 2
            for (int j = 0; j < 8; ++j) {  // 32 elements per j
                uint32_t af[MI][4];
#pragma unroll
                for (int mi = 0; mi < MI; ++mi) {
                    const int row = row0 + 16 * mi + (lane & 7) + ((lane >> 3) & 1) * 8;
                    const int col = 32 * j + (lane >> 4) * 16;
                    ldsm_x4(wq_base + row * kI8Row + col, af[mi][0], af[mi][1], af[mi][2], af[mi][3]);
                }
                uint32_t bf[NI][2];
                if constexpr (big) {
#pragma unroll
                    for (int np = 0; np < 2; ++np) {
                        const int tok = tok0 + 16 * np + (lane & 7) + 8 * (lane >> 4);
                        const int col = 32 * j + 16 * ((lane >> 3) & 1);
                        ldsm_x4(aq_base + tok * kI8Row + col, bf[2 * np][0], bf[2 * np][1], bf[2 * np + 1][0],
                                bf[2 * np + 1][1]);
                    }
                } else {  // lanes 0-15 address tokens 0-7, k 0-15 / 16-31 (lanes 16-31 repeat them)
                    const int tok = lane & 7, col = 32 * j + 16 * ((lane >> 3) & 1);
                    ldsm_x2(aq_base + tok * kI8Row + col, bf[0][0], bf[0][1]);
                }
                if constexpr (TYPE == QWB_TYPE_Q8_0) {
                    // {row g, g+8} of mi 0, then of mi 1; per ni {d(tok), d(tok+1), -M d(tok), -M d(tok+1)}
                    const float4 dw4 = *(const float4 *) &S.dwp[buf][j][row0 >> 5][lane >> 2][0];
                    float4 da4[NI];
#pragma unroll
                    for (int ni = 0; ni < NI; ++ni)
                        da4[ni] = *(const float4 *) &S.dap[buf][j][tok0 / 2 + 4 * ni + (lane & 3)][0];
#pragma unroll
                    for (int mi = 0; mi < MI; ++mi) {
                        // rows row0 + 16 mi + {g, g + 8}: 16-row half ((row0 >> 4) & 1) + mi of the 32-row group
                        const bool hi = (((row0 >> 4) & 1) + mi) != 0;
                        const float w0 = hi ? dw4.z : dw4.x, w1 = hi ? dw4.w : dw4.y;
#pragma unroll
                        for (int ni = 0; ni < NI; ++ni) {
                            int c[4];
                            mma_k32(c, af[mi], bf[ni][0], bf[ni][1], kMagicBits);
                            // c0: (row g, tok 2q), c1: (g, 2q+1), c2: (g+8, 2q), c3: (g+8, 2q+1)
                            const float4 d = da4[ni];
                            acc[mi][ni][0] = __fmaf_rn(__fmaf_rn(__int_as_float(c[0]), d.x, d.z), w0, acc[mi][ni][0]);
                            acc[mi][ni][1] = __fmaf_rn(__fmaf_rn(__int_as_float(c[1]), d.y, d.w), w0, acc[mi][ni][1]);
                            acc[mi][ni][2] = __fmaf_rn(__fmaf_rn(__int_as_float(c[2]), d.x, d.z), w1, acc[mi][ni][2]);
                            acc[mi][ni][3] = __fmaf_rn(__fmaf_rn(__int_as_float(c[3]), d.y, d.w), w1, acc[mi][ni][3]);
                        }
                    }
                } else {
                    // sub-blocks 2j (A regs 0,1 / B reg 0) and 2j+1 (A regs 2,3 / B reg 1)
                    int scr[MI][2][2];  // [mi][row g / g+8][sub-block]
#pragma unroll
                    for (int mi = 0; mi < MI; ++mi) {
                        const int row = row0 + 16 * mi + (lane >> 2);
                        scr[mi][0][0] = S.sc[buf][row][2 * j];
                        scr[mi][0][1] = S.sc[buf][row][2 * j + 1];
                        scr[mi][1][0] = S.sc[buf][row + 8][2 * j];
                        scr[mi][1][1] = S.sc[buf][row + 8][2 * j + 1];
                    }
#pragma unroll
                    for (int mi = 0; mi < MI; ++mi) {
#pragma unroll
                        for (int ni = 0; ni < NI; ++ni) {
#pragma unroll
                            for (int sb = 0; sb < 2; ++sb) {
                                int c[4];
                                mma_k16(c, af[mi][2 * sb], af[mi][2 * sb + 1], bf[ni][sb]);
                                isum[mi][ni][0] += scr[mi][0][sb] * c[0];
                                isum[mi][ni][1] += scr[mi][0][sb] * c[1];
                                isum[mi][ni][2] += scr[mi][1][sb] * c[2];
                                isum[mi][ni][3] += scr[mi][1][sb] * c[3];
                            }
                        }
                    }
                }
            }
            if constexpr (TYPE == QWB_TYPE_Q6_K) {
                // one fp32 scale per superblock: (d_w * d_a) * isum
#pragma unroll
                for (int mi = 0; mi < MI; ++mi) {
                    const int row = row0 + 16 * mi + (lane >> 2);
                    const float dw0 = S.dw[buf][row][0], dw1 = S.dw[buf][row + 8][0];
#pragma unroll
                    for (int ni = 0; ni < NI; ++ni) {
                        const int tok = tok0 + 8 * ni + 2 * (lane & 3);
                        const float da0 = S.da[b3][tok][ks & 3], da1 = S.da[b3][tok + 1][ks & 3];
                        acc[mi][ni][0] += __fmul_rn(dw0, da0) * (float) isum[mi][ni][0];
                        acc[mi][ni][1] += __fmul_rn(dw0, da1) * (float) isum[mi][ni][1];
                        acc[mi][ni][2] += __fmul_rn(dw1, da0) * (float) isum[mi][ni][2];
                        acc[mi][ni][3] += __fmul_rn(dw1, da1) * (float) isum[mi][ni][3];
                    }
                }
            }
        }
        // outputs: dst[row] of each (token, slot) pair
#pragma unroll
        for (int mi = 0; mi < MI; ++mi) {
#pragma unroll
            for (int ni = 0; ni < NI; ++ni) {
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    const int row = row0 + 16 * mi + (lane >> 2) + 8 * (v >> 1);
                    const int tok = tok0 + 8 * ni + 2 * (lane & 3) + (v & 1);
                    if (row < nrows && tok < ntok)
                        ((float *) ((char *) a.dst + S.tok_o[tok]))[r0 + row] = acc[mi][ni][v];
                }
            }
        }
        item = next;
    }
}

template <int TYPE, int TN>
cudaError_t launch_i8_t(const I8PrefillArgs &a, cudaStream_t s) {
    const size_t smem = sizeof(I8Smem<TYPE, TN>);
    static DeviceSmemLimit limit;
    cudaError_t e = ensure_dyn_smem(pf_i8_kernel<TYPE, TN>, smem, limit);
    if (e != cudaSuccess) return e;
    pf_i8_kernel<TYPE, TN><<<num_sms(), kI8Threads, smem, s>>>(a);
    return cudaGetLastError();
}

}  // namespace

bool pf_i8_eligible(int type, int64_t K, int64_t M, int64_t P, int64_t n_as, const void *W, size_t nb1, size_t nb2) {
    if ((type != QWB_TYPE_Q8_0 && type != QWB_TYPE_Q6_K) || K % kI8KS || K < kI8KS || M < 1) return false;
    // Q8_0: 16-byte copies of whole 8-block groups need aligned rows; Q6_K copies widen
    // each superblock to 16-byte boundaries inside the 16-byte aligned tensor
    if (type == QWB_TYPE_Q8_0 ? ((uintptr_t) W | nb1 | nb2) % 16 : (uintptr_t) W % 16) return false;
    const int64_t used = std::min<int64_t>(P, n_as);
    return used > 0 && P >= kI8TNSmall * used;
}

// Tile size by routed pairs per used expert on average: 128-token tiles on the tcgen05
// kernels (prefill_tc8.cu) for Q6_K from 96 (the sub-block scales ride in the A operand,
// one epilogue pass per superblock) and for Q8_0 from 256 (one accumulator region per
// 32-element block; measured on the config-3 gate/up shape, Zipf routing: 190 against 175
// TOP/s for this file's mma.sync kernel at 512 pairs per expert, 137 against 146 at 128).
// Otherwise >= 32: 64-token tiles here, 8 to 31: 8-token tiles here.
int pf_i8_tile_tokens(int type, int64_t P, int64_t n_as) {
    const int64_t used = std::max<int64_t>(1, std::min<int64_t>(P, n_as));
    if (P >= (type == QWB_TYPE_Q8_0 ? 256 : 96) * used) return kTc8TileTokens;
    return P >= 32 * used ? kI8TNBig : kI8TNSmall;
}

cudaError_t launch_pf_i8(int type, int tile_tokens, const I8PrefillArgs &a, cudaStream_t s) {
    if (tile_tokens == kTc8TileTokens) return launch_pf_tc8(type, a, s);
    if (tile_tokens == kI8TNBig)
        return type == QWB_TYPE_Q6_K ? launch_i8_t<QWB_TYPE_Q6_K, kI8TNBig>(a, s)
                                     : launch_i8_t<QWB_TYPE_Q8_0, kI8TNBig>(a, s);
    if (tile_tokens == kI8TNSmall)
        return type == QWB_TYPE_Q6_K ? launch_i8_t<QWB_TYPE_Q6_K, kI8TNSmall>(a, s)
                                     : launch_i8_t<QWB_TYPE_Q8_0, kI8TNSmall>(a, s);
    return cudaErrorInvalidValue;
}

}  // namespace qwb
