// decode.cu - batch-1 decode MoE layer (T == 1) as three kernels chained with
// programmatic dependent launch (PDL).
//
// Reference: the same build_moe subgraph as moe_ffn.cu (core/runtime.cpp:2743-2816, ffn_norm
// :2979), at the batch-1 decode shape QuestWend runs per token.  Decode is
// HBM-bound: per layer 8 experts x (gate + up + down) are streamed once.  Layout of the work:
//
//   router_decode   CTA = 2 router rows.  Before waiting on the previous kernel it
//                   bulk-copies its router rows into shared memory; then rms_norm(x)*w,
//                   logits, Q8_K of the normed x (side work of the first CTAs), and the
//                   last CTA to finish routes (softmax, top-k, renorm) and resolves the
//                   expert -> slot ids of the three pools.
//   gateup_decode   one CTA per SM (8 warps).  The CTA owns a contiguous range of
//                   (expert, row) pairs; right after the routing is visible it issues
//                   bulk copies of all its gate and up rows (chunked, one mbarrier per
//                   chunk), then lets the down kernel launch.  Lane = (row, superblock):
//                   each lane computes one whole Q4_K superblock dot against the
//                   activation superblock it holds in registers, so scales are decoded
//                   once per superblock; SwiGLU in the epilogue.
//   down_decode     one CTA per SM (8 warps; registers and shared memory are sized so it
//                   can be resident next to gate/up).  Its weights depend only on the
//                   routing, so it copies them while gate/up is still running; then it
//                   waits for act, quantizes
//                   it to Q8_K in shared memory, and each warp produces one output row for
//                   all selected experts (lane = (expert, superblock)), weighted sum and
//                   residual included, no atomics.
//
// Arithmetic is that of dot.cuh (exact integer sub-block sums on the reference's Q8_K
// activation bytes, fp32 combine).  Every mbarrier wait is bounded.
#include <algorithm>

#include <cooperative_groups.h>

#include "common.cuh"
#include "decode.cuh"
#include "decode_dev.cuh"
#include "kernels.cuh"
#include "quant_dev.cuh"

namespace qwb {

// Optional phase timestamps for pipeline analysis (compiled in only with
// -DQWB_DECODE_TRACE; no effect on the default build): thread 0 of each CTA records the
// global timer at numbered points of each kernel.
#ifdef QWB_DECODE_TRACE
__device__ unsigned long long g_decode_trace[3][160][8];
__device__ unsigned int g_decode_smid[3][160];
#define QWB_TRACE(k, p)                                                                   \
    do {                                                                                 \
        if (threadIdx.x == 0 && blockIdx.x < 160) {                                      \
            g_decode_trace[k][blockIdx.x][p] = globaltimer_ns();                         \
            if (p == 0) {                                                                \
                unsigned int sm;                                                         \
                asm volatile("mov.u32 %0, %%smid;" : "=r"(sm));                          \
                g_decode_smid[k][blockIdx.x] = sm;                                       \
            }                                                                            \
        }                                                                                \
    } while (0)
#else
#define QWB_TRACE(k, p) \
    do {                \
    } while (0)
#endif

// ---------------------------------------------------------------- router
// The router is ONE thread-block cluster of kRouterCluster CTAs.  Each CTA owns
// E / kRouterCluster router rows, which it bulk-copies into shared memory before waiting
// on the previous kernel (they do not depend on it).  After the wait: x -> shared memory,
// rms_norm * ffn_norm, the CTA's logits, which it stores straight into CTA 0's shared
// memory (distributed shared memory); one cluster barrier; CTA 0 routes.  The Q8_K of
// the normed x is side work of a few other CTAs.  No global-memory round trip, fence or
// atomic lies between the logits and the routing.
//
// Routing (route_experts, core/runtime.cpp:2693-2734): softmax over the E logits (+ mask),
// top-k of the probabilities ranked by a unique key (probability bits, then lower index
// first: exact ties keep index order), renormalised weights (sum clamped at
// 6.103515625e-5), and the winners' slot ids in the three pools (g2s remap, validated).
struct RouterSmemTail {
    float logit[kMaxRouteE];
    unsigned long long key[kMaxRouteE];
    float ev[kMaxRouteE];
    float red[32];
    double redd[32];
    int sel[32];
};

__device__ void route_in_cta(const RouterDecodeArgs &r, int tok, RouterSmemTail &t) {
    const int tid = threadIdx.x, nth = blockDim.x, warp = tid >> 5, lane = tid & 31, nw = nth >> 5;
    const int E = (int) r.E, k = r.n_used;
    const float *mask = r.mask ? r.mask + (int64_t) tok * E : nullptr;
    // 1. max logit (+ mask)
    float lmax = -INFINITY;
    for (int e = tid; e < E; e += nth) {
        float v = t.logit[e];
        if (mask) v = __fadd_rn(v, mask[e]);
        if (isnan(v)) v = -INFINITY;
        t.logit[e] = v;
        lmax = fmaxf(lmax, v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lmax = fmaxf(lmax, __shfl_xor_sync(0xffffffffu, lmax, o));
    if (lane == 0) t.red[warp] = lmax;
    __syncthreads();
    float mx = t.red[0];
    for (int i = 1; i < nw; ++i) mx = fmaxf(mx, t.red[i]);
    QWB_TRACE(0, 5);
    // 2. exp values, unique ranking keys, partial sums
    float ls = 0.f;
    for (int e = tid; e < E; e += nth) {
        float v = expf(__fsub_rn(t.logit[e], mx));
        if (isnan(v)) v = 0.f;
        t.ev[e] = v;
        // probabilities are e * inv with one common inv: ranking the exp values ranks them
        t.key[e] = ((unsigned long long) __float_as_uint(v) << 32) | (unsigned) (0xffffffffu - (unsigned) e);
        ls += v;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, o);
    if (lane == 0) t.redd[warp] = (double) ls;
    __syncthreads();
    QWB_TRACE(0, 6);
    // 3. rank = number of larger keys; the k winners record themselves
    for (int e = tid; e < E; e += nth) {
        const unsigned long long ke = t.key[e];
        int r0 = 0, r1 = 0, r2 = 0, r3 = 0;
        const ulonglong2 *k2 = (const ulonglong2 *) t.key;
        int j = 0;
        for (; j + 8 <= E; j += 8) {
            const ulonglong2 a = k2[j / 2], b = k2[j / 2 + 1], c = k2[j / 2 + 2], d = k2[j / 2 + 3];
            r0 += (a.x > ke) + (a.y > ke);
            r1 += (b.x > ke) + (b.y > ke);
            r2 += (c.x > ke) + (c.y > ke);
            r3 += (d.x > ke) + (d.y > ke);
        }
        for (; j < E; ++j) r0 += t.key[j] > ke;
        const int rank = (r0 + r1) + (r2 + r3);
        if (rank < k) t.sel[rank] = e;
    }
    __syncthreads();
    QWB_TRACE(0, 7);
    // 4. weights of the winners, renormalised (sum in rank order, clamped), slot ids
    if (warp == 0) {
        float sum = 0.f;
        for (int i = 0; i < nw; ++i) sum += (float) t.redd[i];
        const float inv = sum > 0.f ? __fdiv_rn(1.f, sum) : 0.f;
        const int e = lane < k ? t.sel[lane] : 0;
        const float pj = lane < k ? __fmul_rn(t.ev[e], inv) : 0.f;
        float tot = 0.f;
        for (int j = 0; j < k; ++j) tot = __fadd_rn(tot, __shfl_sync(0xffffffffu, pj, j));
        const float ws = tot < 6.103515625e-5f ? 6.103515625e-5f : tot;
        if (lane < k) {
            r.sel[tok * k + lane] = e;
            r.wts[tok * k + lane] = __fdiv_rn(pj, ws);
#pragma unroll
            for (int role = 0; role < 3; ++role) {
                int64_t sl;
                if (r.own_n > 0) {
                    // expert parallelism: another GPU's expert is skipped here, not an error
                    sl = (e >= r.own_lo && e < r.own_lo + r.own_n) ? e - r.own_lo : -1;
                } else {
                    sl = r.g2s ? (int64_t) r.g2s[role * E + e] : e;
                    if (sl < 0 || sl >= r.n_slots[role]) {
                        report(r.st, QWB_DEVERR_ID_RANGE, (int32_t) sl);
                        sl = -1;
                    }
                }
                r.slots[(role * r.T + tok) * k + lane] = (int32_t) sl;
            }
        }
    }
}

__global__ void __launch_bounds__(kRouterThreads) router_decode_kernel(const RouterDecodeArgs r) {
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bar = (uint64_t *) smem;
    const int64_t H = r.H;
    const int rpc = (int) ceil_div(r.E, kRouterCluster);  // rows per CTA
    RouterSmemTail &tail = *(RouterSmemTail *) (smem + 128);
    float *rows = (float *) (smem + 128 + align_up(sizeof(RouterSmemTail), 128));  // [rpc][H]
    float *xs = rows + (size_t) rpc * H;  // [H] x, normalised in place
    float *gw = xs + H;                   // [H] ffn_norm weight
    __shared__ double dpart[kRouterThreads / 32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rank_in_cluster = (int) cluster.block_rank();
    const int tok = (int) blockIdx.x / kRouterCluster;  // one cluster per token
    const float *x = r.x + (int64_t) tok * H;
    const int e0 = rank_in_cluster * rpc;
    const int ne = max(0, min(rpc, (int) r.E - e0));

    QWB_TRACE(0, 0);
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {  // router rows and the norm weight do not depend on the previous kernel
        const uint32_t rbytes = (uint32_t) (ne * H * 4), gbytes = r.norm_w ? (uint32_t) (H * 4) : 0u;
        mbar_arrive_expect_tx(&bar[0], rbytes + gbytes);
        if (rbytes) bulk_span_issue(rows, r.router_w + (int64_t) e0 * H, rbytes, &bar[0]);
        if (r.norm_w) bulk_span_issue(gw, r.norm_w, gbytes, &bar[0]);
    }
    pdl_wait();  // x is the previous layer's output
    QWB_TRACE(0, 1);

    // x -> shared memory, sum of squares (f32 squares, f64 sum as ggml's rms_norm)
    double acc = 0.0;
    for (int64_t i = 4 * tid; i < H; i += 4 * kRouterThreads) {
        const float4 b = *(const float4 *) (x + i);
        *(float4 *) (xs + i) = b;
        acc += (double) __fmul_rn(b.x, b.x);
        acc += (double) __fmul_rn(b.y, b.y);
        acc += (double) __fmul_rn(b.z, b.z);
        acc += (double) __fmul_rn(b.w, b.w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) dpart[warp] = acc;
    bool ok = mbar_wait(&bar[0], 0);
    ok = __syncthreads_and(ok);
    QWB_TRACE(0, 2);
    if (!ok && tid == 0) {  // copies never landed: record it, drain; these rows route as -inf
        report(r.st, QWB_DEVERR_TIMEOUT, rank_in_cluster);
        mbar_wait(&bar[0], 0);
    }
    if (r.norm_w) {
        double sum = 0.0;
        for (int i = 0; i < kRouterThreads / 32; ++i) sum += dpart[i];
        const float mean = (float) (sum / (double) H);
        const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, r.norm_eps)));
        for (int64_t i = 4 * tid; i < H; i += 4 * kRouterThreads) {
            float4 b = *(const float4 *) (xs + i);
            const float4 g = *(const float4 *) (gw + i);
            b.x = __fmul_rn(__fmul_rn(b.x, scale), g.x);
            b.y = __fmul_rn(__fmul_rn(b.y, scale), g.y);
            b.z = __fmul_rn(__fmul_rn(b.z, scale), g.z);
            b.w = __fmul_rn(__fmul_rn(b.w, scale), g.w);
            *(float4 *) (xs + i) = b;
        }
        __syncthreads();
    }
    QWB_TRACE(0, 3);
    // logits of this CTA's rows (one warp per row, rows strided over warps), stored in CTA 0
    float *logit0 = cluster.map_shared_rank(tail.logit, 0);
    for (int er = warp; er < ne; er += kRouterThreads / 32) {
        const float *wr = rows + (int64_t) er * H;
        float a0 = 0.f, a1 = 0.f;
        for (int h = 4 * lane; h < (int) H; h += 256) {
            const float4 w4 = *(const float4 *) (wr + h);
            const float4 x4 = *(const float4 *) (xs + h);
            a0 = fmaf(w4.x, x4.x, a0);
            a0 = fmaf(w4.y, x4.y, a0);
            a0 = fmaf(w4.z, x4.z, a0);
            a0 = fmaf(w4.w, x4.w, a0);
            if (h + 128 < (int) H) {
                const float4 w5 = *(const float4 *) (wr + h + 128);
                const float4 x5 = *(const float4 *) (xs + h + 128);
                a1 = fmaf(w5.x, x5.x, a1);
                a1 = fmaf(w5.y, x5.y, a1);
                a1 = fmaf(w5.z, x5.z, a1);
                a1 = fmaf(w5.w, x5.w, a1);
            }
        }
        const float a = warp_sum(a0 + a1);
        if (lane == 0) logit0[e0 + er] = ok ? a : -INFINITY;
    }
    cluster.sync();  // every logit is in CTA 0's shared memory
    QWB_TRACE(0, 4);
    // Let the gate/up kernel launch now, while CTA 0 routes: its launch overlaps the
    // routing, and by now the previous layer's down kernel has completed (pdl_wait
    // above), so its CTAs find a free slot on every SM.  Triggering at entry launched it
    // while that down kernel still held every SM, and its CTAs doubled up on some SMs.
    pdl_trigger();
    if (rank_in_cluster != 0) {
        // side work of CTAs 1..: Q8 of the normed x, one 256-chunk per warp (needed by the
        // next kernel, which waits for this grid to complete)
        const int64_t c = (int64_t) (rank_in_cluster - 1) * (kRouterThreads / 32) + warp;
        if (c < H / 256) quantize_chunk_warp(r.kq ? 0 : 1, xs + c * 256, r.xq, tok, c * 256, H);
        if (rank_in_cluster == kRouterCluster - 1 && warp == kRouterThreads / 32 - 1 && r.sh_scale) {
            // the shared expert's gate: sigmoid(gw . ffn_in) (ggml_sigmoid_f32: 1 / (1 + e^-v))
            float v = 1.f;
            if (r.sh_gate_inp) {
                float acc = 0.f;
                for (int64_t h = lane; h < H; h += 32) acc = fmaf(r.sh_gate_inp[h], xs[h], acc);
                acc = warp_sum(acc);
                v = 1.f / (1.f + expf(-acc));
            }
            if (lane == 0) r.sh_scale[tok] = v;
        }
        return;
    }
    route_in_cta(r, tok, tail);
}

// ---------------------------------------------------------------- gate/up
template <int NSB>
__global__ void __launch_bounds__(kDecodeThreads, 2) gateup_decode_kernel(const GateUpDecodeArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bar = (uint64_t *) smem;  // [kChunks]
    uint8_t *buf = smem + 128;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t P = (int64_t) a.n_used * a.F;
    const int64_t p0 = P * blockIdx.x / gridDim.x, p1 = P * (blockIdx.x + 1) / gridDim.x;
    const int n = (int) (p1 - p0);
    const int rb = (int) a.row_bytes;
    const int nch = min(kDecodeChunks, max(1, n));
    auto chunk_lo = [&](int c) { return (int) ((int64_t) n * c / nch); };
    __shared__ int s_sg[32], s_su[32];

    QWB_TRACE(1, 0);
    if (tid == 0) {
        for (int c = 0; c < nch; ++c) mbar_init(&bar[c], 1);
        fence_mbar_init();
    }
    pdl_wait();  // the routing and the quantized x are ready
    QWB_TRACE(1, 1);
    if (tid < a.n_used) {  // validated by the router (-1: invalid)
        const int sg = a.slots[tid], su = a.slots[a.n_used + tid];
        const bool ok = sg >= 0 && sg < a.n_slots_g && su >= 0 && su < a.n_slots_u;
        s_sg[tid] = ok ? sg : -1;
        s_su[tid] = ok ? su : -1;
    }
    __syncthreads();
    if (tid < nch) {  // thread c issues chunk c
        const int c = tid;
        const int c0 = chunk_lo(c), c1 = chunk_lo(c + 1), nc = c1 - c0;
        uint8_t *cb = buf + (size_t) 2 * c0 * rb;
        uint32_t bytes = 0;
        const int F = (int) a.F;
        for (int pass = 0; pass < 2; ++pass) {  // pass 0 counts, pass 1 issues
            if (pass == 1) mbar_arrive_expect_tx(&bar[c], bytes);
            int j = (int) ((p0 + c0) / F), r = (int) ((p0 + c0) % F);
            for (int off = 0; off < nc;) {
                const int len = min(nc - off, F - r);
                const int sg = s_sg[j], su = s_su[j];
                if (sg >= 0) {
                    if (pass == 0) bytes += 2u * (uint32_t) (len * rb);
                    else {
                        bulk_span_issue(cb + off * rb, a.Wg + (size_t) sg * a.g_nb2 + (size_t) r * rb,
                                        (size_t) len * rb, &bar[c]);
                        bulk_span_issue(cb + (size_t) (nc + off) * rb, a.Wu + (size_t) su * a.u_nb2 + (size_t) r * rb,
                                        (size_t) len * rb, &bar[c]);
                    }
                }
                off += len;
                r = 0;
                ++j;
            }
        }
    }
    QWB_TRACE(1, 2);
    pdl_trigger();  // the down kernel may start copying its weights now

    // the activation superblock of this lane (x has one row: T == 1)
    const int s = lane % NSB;
    ActReg<false> act;
    load_act<false>(act, a.xq.qs + (int64_t) s * 256, a.xq.bsum + s * 16, a.xq.d[s]);
    QWB_TRACE(1, 3);

    constexpr int RPW = 32 / (2 * NSB);  // (gate, up) row pairs per warp step
    const int pp_in = lane / (2 * NSB), mat = (lane / NSB) & 1;
    const int F = (int) a.F;
    const int j_first = (int) (p0 / F), r_first = (int) (p0 % F);  // expert/row of the CTA's first pair
    const uint32_t buf_sa = smem_u32(buf);
    bool alive = true;
    for (int c = 0; c < nch; ++c) {
        const int c0 = chunk_lo(c), c1 = chunk_lo(c + 1), nc = c1 - c0;
        const uint32_t cb = buf_sa + (uint32_t) (2 * c0 * rb);
        if (!mbar_wait(&bar[c], 0)) {
            if (lane == 0) report(a.st, QWB_DEVERR_TIMEOUT, c);
            alive = false;
            break;
        }
        if (c == 0) QWB_TRACE(1, 4);
        for (int g = warp; g * RPW < nc; g += kDecodeThreads / 32) {
            const int i = g * RPW + pp_in;  // row pair within the chunk
            int j = j_first, r = r_first + c0 + i;
            while (r >= F) { r -= F; ++j; }
            float v = 0.f;
            if (i < nc && s_sg[j] >= 0)
                v = dot_q4K_sb(buf + (cb - buf_sa) + (uint32_t) ((mat * nc + i) * rb) + (uint32_t) (s * Q4K_BYTES), act);
#pragma unroll
            for (int o = 1; o < NSB; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            const float up = __shfl_down_sync(0xffffffffu, v, NSB);
            if (i < nc && mat == 0 && s == 0) a.act[j * F + r] = swiglu_f(v, up);
        }
    }
    QWB_TRACE(1, 5);
    // a timed-out wait leaves copies possibly in flight: drain them before the CTA exits
    if (!__syncthreads_and(alive) && tid == 0)
        for (int c = 0; c < nch; ++c) mbar_wait(&bar[c], 0);
    QWB_TRACE(1, 6);
}

// ---------------------------------------------------------------- down
// output rows per down CTA: H / #SMs, at most ceil(8192 / 148)
constexpr int kDownMaxRows = 56;

// bytes reserved per expert weight span: the CTA's rows plus the 16-byte widening,
// rounded to 16 mod 128 so consecutive experts start on different shared-memory banks
__host__ __device__ inline size_t down_span_stride(int n, size_t rb) {
    const size_t b = align_up((size_t) n * rb + 32, 16);
    return align_up(b + 112, 128) + 16;
}

// Warp w handles selected expert j = w (and j + 8, ... when more experts than warps);
// lane = (row, superblock): 32 / NSB rows per warp step.  Expert j's rows of this CTA are
// one bulk copy completing on barrier j, issued by thread j.  Each warp quantizes its
// expert's act row into its own shared-memory scratch and keeps its lane's superblock in
// registers; per-(expert, row) partial sums meet in shared memory and the weighted sum
// over experts runs in expert order, so the result does not depend on scheduling.
template <int TYPE, int NSB>
__global__ void __launch_bounds__(kDecodeThreads, 2) down_decode_kernel(const DownDecodeArgs a) {
    constexpr bool KQ6 = TYPE == QWB_TYPE_Q6_K;
    constexpr int SBB = KQ6 ? Q6K_BYTES : Q4K_BYTES;
    constexpr int NW = kDecodeThreads / 32;
    constexpr int RPS = 32 / NSB;  // rows per warp step
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bar = (uint64_t *) smem;  // [n_used] (<= 32)
    __shared__ int s_slot[32];
    __shared__ float s_w[32];
    __shared__ int s_off[32];  // misalignment of each expert's span
    __shared__ float s_res[kDownMaxRows];  // the CTA's residual rows, read before the wait
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nu = a.n_used;
    const int64_t h0 = a.H * blockIdx.x / gridDim.x, h1 = a.H * (blockIdx.x + 1) / gridDim.x;
    const int n = (int) (h1 - h0);
    const size_t rb = a.row_bytes;
    // shared memory: [bars 256][act Q8_K: NW warps x NSB superblocks x 320 B]
    //                [partials: nu x n floats][weight spans, one per expert]
    uint8_t *actq = smem + 256;
    float *part = (float *) (actq + (size_t) NW * NSB * 320);
    uint8_t *wbuf = (uint8_t *) part + align_up((size_t) nu * n * 4, 128);
    const size_t span_stride = down_span_stride(n, rb);

    QWB_TRACE(2, 0);
    // the router grid completed before the gate/up grid passed its wait, so its outputs
    // are visible here while gate/up is still running
    if (tid < nu) {
        const int sl = a.slots[tid];
        s_slot[tid] = (sl >= 0 && sl < a.n_slots) ? sl : -1;
        s_w[tid] = a.wts[tid];
        mbar_init(&bar[tid], 1);
    }
    fence_mbar_init();
    __syncthreads();
    if (tid < nu) {  // thread j copies expert j's rows
        const int j = tid;
        if (s_slot[j] >= 0) {
            const uint8_t *src = a.W + (size_t) s_slot[j] * a.nb2 + (size_t) h0 * rb;
            mbar_arrive_expect_tx(&bar[j], bulk_span_bytes(src, (size_t) n * rb));
            s_off[j] = (int) bulk_span_issue(wbuf + (size_t) j * span_stride, src, (size_t) n * rb, &bar[j]);
        } else {
            s_off[j] = 0;
            mbar_arrive_expect_tx(&bar[j], 0);
        }
    }
    // the residual (this layer's input) was complete before the router ran: load it
    // before waiting on gate/up, off the critical path
    if (a.residual)
        for (int r = tid; r < n; r += kDecodeThreads) s_res[r] = a.residual[h0 + r];
    QWB_TRACE(2, 1);
    pdl_trigger();  // the next layer's router may prefetch its rows
    pdl_wait();     // act (gate/up output) is ready
    QWB_TRACE(2, 2);
    __syncthreads();  // s_off, s_res visible

    const int li = lane / NSB, ls = lane % NSB;
    bool alive = true;
    for (int j = warp; j < nu; j += NW) {
        // this warp's expert: act row -> Q8_K superblocks in its scratch -> lane registers;
        // all NSB superblocks' inputs are loaded before quantizing (one L2 round trip)
        uint8_t *scr = actq + (size_t) warp * NSB * 320;
        float xv[NSB][8];
#pragma unroll
        for (int sb = 0; sb < NSB; ++sb) load8_normed(a.act + (int64_t) j * a.F + sb * 256, 1.f, nullptr, lane, xv[sb]);
        __syncwarp();
#pragma unroll
        for (int sb = 0; sb < NSB; ++sb)
            q8K_block_vals(xv[sb], nullptr, (int8_t *) (scr + sb * 320), (float *) (scr + sb * 320 + 256),
                           (int16_t *) (scr + sb * 320 + 272));
        __syncwarp();
        if (j == 0) QWB_TRACE(2, 3);
        ActReg<KQ6> act;
        {
            const uint8_t *src = scr + (size_t) ls * 320;
            load_act<KQ6>(act, (const int8_t *) src, (const int16_t *) (src + 272), *(const float *) (src + 256));
        }
        const bool valid = s_slot[j] >= 0;
        if (!mbar_wait(&bar[j], 0)) {
            if (lane == 0) report(a.st, QWB_DEVERR_TIMEOUT, j);
            alive = false;
            continue;
        }
        if (j == 0) QWB_TRACE(2, 4);
        const uint8_t *span = wbuf + (size_t) j * span_stride + s_off[j];
        for (int i0 = 0; i0 < n; i0 += RPS) {
            const int i = i0 + li;
            float v = 0.f;
            if (valid && li < RPS && i < n) {
                const uint8_t *sb = span + (size_t) i * rb + (size_t) ls * SBB;
                if constexpr (KQ6) v = dot_q6K_sb(sb, act);
                else v = dot_q4K_sb(sb, act);
            }
            // sum the NSB superblocks of each row (lanes li*NSB .. li*NSB + NSB-1)
            float tot = 0.f;
#pragma unroll
            for (int q = 0; q < NSB; ++q) tot += __shfl_sync(0xffffffffu, v, (li < RPS ? li : 0) * NSB + q);
            if (ls == 0 && li < RPS && i < n) part[(size_t) j * n + i] = tot;
        }
    }
    QWB_TRACE(2, 5);
    const bool all_ok = __syncthreads_and(alive);
    if (all_ok) {
        for (int r = tid; r < n; r += kDecodeThreads) {
            float acc = 0.f;
            for (int j = 0; j < nu; ++j)
                if (s_slot[j] >= 0) acc = fmaf(s_w[j], part[(size_t) j * n + r], acc);
            const int64_t h = h0 + r;
            a.out[h] = a.residual ? acc + s_res[r] : acc;
        }
    } else if (tid < nu) {
        mbar_wait(&bar[tid], 0);  // drain copies still in flight before the CTA exits
    }
    QWB_TRACE(2, 6);
}

// ---------------------------------------------------------------- pair lists
// The decode batch as (token, expert) pairs: every routed pair whose three slots are
// valid (under expert parallelism: the experts this GPU owns), in (token, slot) order,
// then one shared-expert pair per token.  Each CTA of the gate/up and down kernels builds
// the same list from the router's slot ids (a ballot compaction, no extra kernel).
struct PairList {
    int tok[kPairsMax];
    int sg[kPairsMax], su[kPairsMax], sd[kPairsMax];  // slots; -2: the shared expert
    float w[kPairsMax];                                // routing weight / shared-expert factor
};

// all threads of the CTA (blockDim.x >= T * n_used); ends with a CTA barrier
__device__ int build_pairs(const PairsCommon &a, PairList &pl, int *warp_cnt) {
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = (int) (blockDim.x >> 5);
    const int TK = a.T * a.n_used;
    int g = -1, u = -1, d = -1;
    if (tid < TK) {
        g = a.slots[tid];
        u = a.slots[TK + tid];
        d = a.slots[2 * TK + tid];
    }
    const bool valid = tid < TK && g >= 0 && u >= 0 && d >= 0;
    const unsigned bal = __ballot_sync(0xffffffffu, valid);
    if (lane == 0) warp_cnt[warp] = __popc(bal);
    __syncthreads();
    int base = 0, total = 0;
    for (int w = 0; w < nw; ++w) {
        const int c = warp_cnt[w];
        if (w < warp) base += c;
        total += c;
    }
    if (valid) {
        const int c = base + __popc(bal & ((1u << lane) - 1u));
        pl.tok[c] = tid / a.n_used;
        pl.sg[c] = g;
        pl.su[c] = u;
        pl.sd[c] = d;
        pl.w[c] = a.wts[tid];
    }
    if (a.shexp && tid < a.T) {
        const int c = total + tid;
        pl.tok[c] = tid;
        pl.sg[c] = pl.su[c] = pl.sd[c] = -2;
        pl.w[c] = a.sh_scale ? a.sh_scale[tid] : 1.f;
    }
    __syncthreads();
    return total + (a.shexp ? a.T : 0);
}

// Gate/up of every pair: the (pair, row) space is cut into one contiguous range per CTA,
// streamed through two buffers of batch_rows (gate, up) row pairs, bulk copies per
// (pair, row) segment; lane = (row, superblock) as in gateup_decode_kernel, the
// activation superblock reloaded when a lane's row belongs to another token.
template <int NSB>
__global__ void __launch_bounds__(kDecodeThreads, 2) gateup_pairs_kernel(const PairsGateUpArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bar = (uint64_t *) smem;  // [2]
    uint8_t *buf = smem + 128;
    __shared__ PairList pl;
    __shared__ int wcnt[kDecodeThreads / 32];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rb = (int) a.row_bytes, F = (int) a.F;
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    pdl_wait();  // the routing and the quantized x are ready
    const int L = build_pairs(a.pc, pl, wcnt);
    const int64_t P = (int64_t) L * F;
    const int64_t p0 = P * blockIdx.x / gridDim.x, p1 = P * (blockIdx.x + 1) / gridDim.x;
    const int n = (int) (p1 - p0);
    // rows that fit both buffers go out as one batch (fewer, larger bulk copies); more
    // stream through the two buffers batch_rows at a time
    const int RB = n <= 2 * a.batch_rows ? max(n, 1) : a.batch_rows;
    const size_t bstride = (size_t) 2 * RB * rb;
    const int nbat = (n + RB - 1) / RB;
    // batch b: rows [p0 + b RB, ...) into buffer b & 1 (gate rows, then up rows), on bar[b & 1]
    auto issue = [&](int b) {
        const int q0 = b * RB, nq = min(RB, n - q0);
        uint8_t *gb = buf + (size_t) (b & 1) * bstride, *ub = gb + (size_t) RB * rb;
        for (int pass = 0; pass < 2; ++pass) {  // pass 0 counts the bytes, pass 1 issues
            uint32_t bytes = 0;
            const int64_t q = p0 + q0;
            int c = (int) (q / F), r = (int) (q - (int64_t) c * F);
            for (int off = 0; off < nq;) {
                const int len = min(nq - off, F - r);
                const uint8_t *sg = pl.sg[c] == -2 ? a.Wg_sh : a.Wg + (size_t) pl.sg[c] * a.g_nb2;
                const uint8_t *su = pl.su[c] == -2 ? a.Wu_sh : a.Wu + (size_t) pl.su[c] * a.u_nb2;
                if (pass == 0) {
                    bytes += bulk_span_bytes(sg + (size_t) r * rb, (size_t) len * rb) +
                             bulk_span_bytes(su + (size_t) r * rb, (size_t) len * rb);
                } else {
                    bulk_span_issue(gb + (size_t) off * rb, sg + (size_t) r * rb, (size_t) len * rb, &bar[b & 1]);
                    bulk_span_issue(ub + (size_t) off * rb, su + (size_t) r * rb, (size_t) len * rb, &bar[b & 1]);
                }
                off += len;
                r = 0;
                ++c;
            }
            if (pass == 0) mbar_arrive_expect_tx(&bar[b & 1], bytes);
        }
    };
    int issued = 0;
    if (tid == 0) {
        if (nbat > 0) issue(0);
        if (nbat > 1) issue(1);
        issued = min(nbat, 2);
    }
    pdl_trigger();  // the down kernel may start copying its weights now

    const int s = lane % NSB;
    ActReg<false> act;
    int cur_tok = -1;
    constexpr int RPW = 32 / (2 * NSB);  // (gate, up) row pairs per warp step
    const int pp_in = lane / (2 * NSB), mat = (lane / NSB) & 1;
    const int dstride = (int) plane_d_stride(a.K, QK_K), bstride_pl = (int) plane_bsum_stride(a.K);
    int b = 0;
    bool alive = true;
    for (; b < nbat; ++b) {
        const bool ok = mbar_wait(&bar[b & 1], (uint32_t) ((b >> 1) & 1));
        if (!__syncthreads_and(ok)) {
            if (tid == 0) report(a.st, QWB_DEVERR_TIMEOUT, b);
            alive = false;
            break;
        }
        const int q0 = b * RB, nq = min(RB, n - q0);
        const uint8_t *gb = buf + (size_t) (b & 1) * bstride;
        for (int g = warp; g * RPW < nq; g += kDecodeThreads / 32) {
            const int i = g * RPW + pp_in;  // row pair within the batch
            const bool in = i < nq;
            int c = 0, r = 0;
            float v = 0.f;
            if (in) {
                const int64_t q = p0 + q0 + i;
                c = (int) (q / F);
                r = (int) (q - (int64_t) c * F);
                const int t = pl.tok[c];
                if (t != cur_tok) {
                    load_act<false>(act, a.xq.qs + (int64_t) t * a.K + (int64_t) s * 256,
                                    a.xq.bsum + (int64_t) t * bstride_pl + s * 16, a.xq.d[(int64_t) t * dstride + s]);
                    cur_tok = t;
                }
                v = dot_q4K_sb(gb + (size_t) (mat * RB + i) * rb + (size_t) s * Q4K_BYTES, act);
            }
#pragma unroll
            for (int o = 1; o < NSB; o <<= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            const float up = __shfl_down_sync(0xffffffffu, v, NSB);
            if (in && mat == 0 && s == 0) a.act[(int64_t) c * F + r] = swiglu_f(v, up);
        }
        __syncthreads();  // buffer b & 1 is free
        if (tid == 0 && b + 2 < nbat) {
            issue(b + 2);
            issued = b + 3;
        }
    }
    // a timed-out wait leaves copies possibly in flight: drain them before the CTA exits
    if (!alive && tid == 0)
        for (int bb = b; bb < issued; ++bb) mbar_wait(&bar[bb & 1], (uint32_t) ((bb >> 1) & 1));
}

// Down of every pair for the CTA's output rows [h0, h1), weighted sum per token (routed
// pairs in list order, then the shared expert, then the residual: the order of the
// reference graph).  The pairs' weight spans are resident `group` at a time (the first
// group copied before the wait on gate/up); each warp quantizes its pair's act row to
// Q8_K in shared memory as down_decode_kernel does.
template <int TYPE, int NSB>
__global__ void __launch_bounds__(kDecodeThreads, 2) down_pairs_kernel(const PairsDownArgs a) {
    constexpr bool KQ6 = TYPE == QWB_TYPE_Q6_K;
    constexpr int SBB = KQ6 ? Q6K_BYTES : Q4K_BYTES;
    constexpr int NW = kDecodeThreads / 32;
    constexpr int RPS = 32 / NSB;  // rows per warp step
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bar = (uint64_t *) smem;  // [group] (<= 32)
    __shared__ PairList pl;
    __shared__ int wcnt[NW];
    __shared__ int s_off[32];
    __shared__ float s_res[kPairsMaxT * kDownMaxRows];  // residual rows, read before the wait
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.group, T = a.pc.T;
    const int64_t h0 = a.H * blockIdx.x / gridDim.x, h1 = a.H * (blockIdx.x + 1) / gridDim.x;
    const int n = (int) (h1 - h0);
    const size_t rb = a.row_bytes;
    uint8_t *actq = smem + 256;
    float *part = (float *) (actq + (size_t) NW * NSB * 320);  // [pair][n]
    uint8_t *wbuf = (uint8_t *) part + align_up((size_t) kPairsMax * n * 4, 128);
    const size_t span_stride = down_span_stride(n, rb);

    if (tid < G) mbar_init(&bar[tid], 1);
    fence_mbar_init();
    // the router grid completed before the gate/up grid passed its wait: its slot ids,
    // weights and shared-expert factors are visible here while gate/up is still running
    const int L = build_pairs(a.pc, pl, wcnt);
    auto issue_group = [&](int g0) {  // thread j copies pair g0 + j into span j
        const int j = tid;
        if (j < G && g0 + j < L) {
            const int c = g0 + j;
            const uint8_t *src = (pl.sd[c] == -2 ? a.W_sh : a.W + (size_t) pl.sd[c] * a.nb2) + (size_t) h0 * rb;
            mbar_arrive_expect_tx(&bar[j], bulk_span_bytes(src, (size_t) n * rb));
            s_off[j] = (int) bulk_span_issue(wbuf + (size_t) j * span_stride, src, (size_t) n * rb, &bar[j]);
        }
    };
    issue_group(0);
    // the residual (this layer's input) was complete before the router ran
    if (a.residual)
        for (int idx = tid; idx < T * n; idx += kDecodeThreads)
            s_res[idx] = a.residual[(int64_t) (idx / n) * a.H + h0 + idx % n];
    pdl_trigger();  // the next layer's router may prefetch its rows
    pdl_wait();     // act (gate/up output) is ready
    __syncthreads();  // s_off, s_res visible

    const int li = lane / NSB, ls = lane % NSB;
    const int ngroups = (L + G - 1) / G;
    bool alive = true;
    int gi = 0;
    for (; gi < ngroups; ++gi) {
        const int g0 = gi * G, gn = min(G, L - g0);
        bool ok = true;
        for (int jj = warp; jj < gn; jj += NW) {
            const int c = g0 + jj;
            uint8_t *scr = actq + (size_t) warp * NSB * 320;
            float xv[NSB][8];
#pragma unroll
            for (int sb = 0; sb < NSB; ++sb) load8_normed(a.act + (int64_t) c * a.F + sb * 256, 1.f, nullptr, lane, xv[sb]);
            __syncwarp();
#pragma unroll
            for (int sb = 0; sb < NSB; ++sb)
                q8K_block_vals(xv[sb], nullptr, (int8_t *) (scr + sb * 320), (float *) (scr + sb * 320 + 256),
                               (int16_t *) (scr + sb * 320 + 272));
            __syncwarp();
            ActReg<KQ6> act;
            {
                const uint8_t *src = scr + (size_t) ls * 320;
                load_act<KQ6>(act, (const int8_t *) src, (const int16_t *) (src + 272), *(const float *) (src + 256));
            }
            __syncwarp();  // the scratch is rewritten by this warp's next pair
            if (!mbar_wait(&bar[jj], (uint32_t) (gi & 1))) {
                if (lane == 0) report(a.st, QWB_DEVERR_TIMEOUT, c);
                ok = false;
                continue;
            }
            const uint8_t *span = wbuf + (size_t) jj * span_stride + s_off[jj];
            for (int i0 = 0; i0 < n; i0 += RPS) {
                const int i = i0 + li;
                float v = 0.f;
                if (li < RPS && i < n) {
                    const uint8_t *sb = span + (size_t) i * rb + (size_t) ls * SBB;
                    if constexpr (KQ6) v = dot_q6K_sb(sb, act);
                    else v = dot_q4K_sb(sb, act);
                }
                float tot = 0.f;
#pragma unroll
                for (int q = 0; q < NSB; ++q) tot += __shfl_sync(0xffffffffu, v, (li < RPS ? li : 0) * NSB + q);
                if (ls == 0 && li < RPS && i < n) part[(size_t) c * n + i] = tot;
            }
        }
        if (!__syncthreads_and(ok)) {
            alive = false;
            break;
        }
        if (gi + 1 < ngroups) {
            issue_group(g0 + G);  // every warp is done with the spans (barrier above)
            __syncthreads();      // s_off of the new group visible
        }
    }
    if (alive) {
        for (int idx = tid; idx < T * n; idx += kDecodeThreads) {
            const int t = idx / n, i = idx - t * n;
            float acc = 0.f;
            for (int c = 0; c < L; ++c)
                if (pl.tok[c] == t && pl.sd[c] != -2) acc = fmaf(pl.w[c], part[(size_t) c * n + i], acc);
            for (int c = 0; c < L; ++c)
                if (pl.tok[c] == t && pl.sd[c] == -2) acc = __fadd_rn(acc, __fmul_rn(part[(size_t) c * n + i], pl.w[c]));
            const int64_t o = (int64_t) t * a.H + h0 + i;
            a.out[o] = a.residual ? acc + s_res[idx] : acc;
        }
    } else if (tid < G && gi * G + tid < L) {
        mbar_wait(&bar[tid], (uint32_t) (gi & 1));  // drain copies still in flight before the CTA exits
    }
}

// ---------------------------------------------------------------- launches
template <typename Kern, typename Args>
static cudaError_t launch_pdl(Kern kern, dim3 grid, dim3 block, size_t smem, cudaStream_t s, const Args &args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args);
}

template <typename Kern>
static cudaError_t set_smem(Kern kern, size_t smem) {
    // The three decode kernels overlap on every SM under programmatic dependent launch.
    // An SM's L1 / shared-memory split is set for the kernels resident on it and changes
    // only when it drains; with every kernel asking for the largest shared carveout, a CTA
    // fits wherever the shared memory it needs is free (otherwise some CTAs doubled up on
    // other SMs and finished microseconds after the rest).
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                         (int) cudaSharedmemCarveoutMaxShared);
    if (e != cudaSuccess || smem <= 48 * 1024) return e;
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
}

size_t router_decode_smem(const RouterDecodeArgs &r) {
    const int64_t rpc = ceil_div(r.E, kRouterCluster);
    return 128 + align_up(sizeof(RouterSmemTail), 128) + (size_t) (rpc + 2) * r.H * 4;
}

cudaError_t launch_router_decode(const RouterDecodeArgs &r, cudaStream_t s) {
    const size_t smem = router_decode_smem(r);
    static bool configured[kAttrDevices] = {};  // per device: attributes hold for one device
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kAttrDevices) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(router_decode_kernel, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) return e;
        configured[dev] = true;
    }
    cudaError_t e = set_smem(router_decode_kernel, smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kRouterCluster * std::max(1, r.T));
    cfg.blockDim = dim3(kRouterThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = kRouterCluster;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, router_decode_kernel, r);
}

bool gateup_decode_supported(int type, int64_t K, size_t row_bytes, size_t nb1, int64_t F, int n_used) {
    if (type != QWB_TYPE_Q4_K || nb1 != row_bytes) return false;
    if (K != 2048 && K != 4096) return false;
    const int64_t per_cta = ceil_div((int64_t) n_used * F, num_sms());
    return (size_t) per_cta * 2 * row_bytes + 128 <= 200 * 1024;
}

// Shared memory per SM and reserved per CTA (228 KB and 1 KB on B200).
static void sm_smem(size_t &per_sm, size_t &reserved) {
    static int sm = 0, rsv = -1;
    if (!sm) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, dev);
        cudaDeviceGetAttribute(&rsv, cudaDevAttrReservedSharedMemoryPerBlock, dev);
        if (sm <= 0) sm = 233472;
        if (rsv < 0) rsv = 1024;
    }
    per_sm = (size_t) sm;
    reserved = (size_t) rsv;
}

cudaError_t launch_gateup_decode(const GateUpDecodeArgs &a, cudaStream_t s) {
    const int G = num_sms();
    const int64_t per_cta = ceil_div((int64_t) a.n_used * a.F, G);
    size_t smem = 128 + (size_t) per_cta * 2 * a.row_bytes;
    // One gate/up CTA per SM.  At ~95 KB two of them fit one SM, and under programmatic
    // launch (the router still holds 16 SMs when this grid starts) the block scheduler
    // placed two on some SMs while others had none: those SMs streamed twice the bytes and
    // set the layer's time.  Asking for just over half of an SM's shared memory keeps one
    // per SM, while the down kernel launched after it still fits beside it (its weight
    // copies overlap this kernel).  Measured on the 30B-A3B decode stack (48 layers, one
    // B200, A/B on the same box): 975 -> 1103 tok/s.
    size_t per_sm = 0, reserved = 0;
    sm_smem(per_sm, reserved);
    const size_t one_per_sm = per_sm / 2 - reserved + 256;
    if (smem < one_per_sm && a.partner_smem && one_per_sm + a.partner_smem + 2 * reserved <= per_sm)
        smem = one_per_sm;
    if (a.K == 2048) {
        cudaError_t e = set_smem(gateup_decode_kernel<8>, smem);
        if (e != cudaSuccess) return e;
        return launch_pdl(gateup_decode_kernel<8>, dim3(G), dim3(kDecodeThreads), smem, s, a);
    }
    cudaError_t e = set_smem(gateup_decode_kernel<16>, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(gateup_decode_kernel<16>, dim3(G), dim3(kDecodeThreads), smem, s, a);
}

static size_t down_decode_smem(int64_t H, int n_used, int nsb, size_t rb) {
    const int64_t n = ceil_div(H, num_sms());
    return 256 + (size_t) (kDecodeThreads / 32) * nsb * 320 + align_up((size_t) n_used * n * 4, 128) +
           (size_t) n_used * down_span_stride((int) n, rb);
}

size_t down_decode_smem_bytes(int64_t H, int n_used, size_t row_bytes) {
    return down_decode_smem(H, n_used, 3, row_bytes);
}

bool down_decode_supported(int type, int64_t F, int64_t H, size_t row_bytes, size_t nb1, int n_used) {
    if ((type != QWB_TYPE_Q4_K && type != QWB_TYPE_Q6_K) || nb1 != row_bytes) return false;
    if (ceil_div(H, num_sms()) > kDownMaxRows) return false;
    const int nsb = (int) (F / 256);
    if (nsb != 3 || n_used * nsb > 32) return false;
    return down_decode_smem(H, n_used, nsb, row_bytes) <= 220 * 1024;
}

cudaError_t launch_down_decode(int type, const DownDecodeArgs &a, cudaStream_t s) {
    const int G = num_sms();
    const size_t smem = down_decode_smem(a.H, a.n_used, 3, a.row_bytes);
    if (type == QWB_TYPE_Q6_K) {
        cudaError_t e = set_smem(down_decode_kernel<QWB_TYPE_Q6_K, 3>, smem);
        if (e != cudaSuccess) return e;
        return launch_pdl(down_decode_kernel<QWB_TYPE_Q6_K, 3>, dim3(G), dim3(kDecodeThreads), smem, s, a);
    }
    cudaError_t e = set_smem(down_decode_kernel<QWB_TYPE_Q4_K, 3>, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(down_decode_kernel<QWB_TYPE_Q4_K, 3>, dim3(G), dim3(kDecodeThreads), smem, s, a);
}

// ---------------------------------------------------------------- pair path launches
constexpr size_t kPairsGateUpSmem = 96 * 1024;  // dynamic shared memory of the two kernels:
constexpr size_t kPairsDownSmem = 116 * 1024;   // both fit one SM together (overlap under PDL)

static size_t pairs_down_fixed(int64_t H, int nsb) {
    const int64_t n = ceil_div(H, num_sms());
    return 256 + (size_t) (kDecodeThreads / 32) * nsb * 320 + align_up((size_t) kPairsMax * n * 4, 128);
}

bool pairs_supported(int type_gu, int type_d, int64_t H, int64_t F, int64_t E, int n_used, int T, size_t rb_gu,
                     size_t nb1_g, size_t nb1_u, size_t rb_d, size_t nb1_d) {
    if (type_gu != QWB_TYPE_Q4_K || (type_d != QWB_TYPE_Q4_K && type_d != QWB_TYPE_Q6_K)) return false;
    if (nb1_g != rb_gu || nb1_u != rb_gu || nb1_d != rb_d || rb_gu % 16) return false;
    if (H != 2048 && H != 4096) return false;
    if (F % 256) return false;
    const int nsb = (int) (F / 256);
    if (nsb != 2 && nsb != 3 && nsb != 4 && nsb != 6) return false;
    if (T < 1 || T > kPairsMaxT || n_used < 1 || n_used > kPairsMaxUsed) return false;
    if (E > kMaxRouteE || E < kRouterCluster || E % kRouterCluster) return false;
    if (4 * rb_gu + 128 > kPairsGateUpSmem) return false;
    const int64_t n = ceil_div(H, num_sms());
    return pairs_down_fixed(H, nsb) + down_span_stride((int) n, rb_d) <= kPairsDownSmem;
}

cudaError_t launch_gateup_pairs(PairsGateUpArgs a, cudaStream_t s) {
    a.batch_rows = (int) ((kPairsGateUpSmem - 128) / (4 * a.row_bytes));
    const size_t smem = 128 + (size_t) 4 * a.batch_rows * a.row_bytes;
    const int G = num_sms();
    if (a.K == 2048) {
        cudaError_t e = set_smem(gateup_pairs_kernel<8>, smem);
        if (e != cudaSuccess) return e;
        return launch_pdl(gateup_pairs_kernel<8>, dim3(G), dim3(kDecodeThreads), smem, s, a);
    }
    cudaError_t e = set_smem(gateup_pairs_kernel<16>, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(gateup_pairs_kernel<16>, dim3(G), dim3(kDecodeThreads), smem, s, a);
}

template <int TYPE, int NSB>
static cudaError_t launch_down_pairs_t(const PairsDownArgs &a, size_t smem, cudaStream_t s) {
    cudaError_t e = set_smem(down_pairs_kernel<TYPE, NSB>, smem);
    if (e != cudaSuccess) return e;
    return launch_pdl(down_pairs_kernel<TYPE, NSB>, dim3(num_sms()), dim3(kDecodeThreads), smem, s, a);
}

cudaError_t launch_down_pairs(int type, PairsDownArgs a, cudaStream_t s) {
    const int nsb = (int) (a.F / 256);
    const int64_t n = ceil_div(a.H, num_sms());
    const size_t fixed = pairs_down_fixed(a.H, nsb), span = down_span_stride((int) n, a.row_bytes);
    if (fixed + span > kPairsDownSmem) return cudaErrorInvalidValue;
    a.group = (int) std::min<size_t>(16, (kPairsDownSmem - fixed) / span);
    const size_t smem = fixed + (size_t) a.group * span;
    const bool q6 = type == QWB_TYPE_Q6_K;
    switch (nsb) {
        case 2: return q6 ? launch_down_pairs_t<QWB_TYPE_Q6_K, 2>(a, smem, s) : launch_down_pairs_t<QWB_TYPE_Q4_K, 2>(a, smem, s);
        case 3: return q6 ? launch_down_pairs_t<QWB_TYPE_Q6_K, 3>(a, smem, s) : launch_down_pairs_t<QWB_TYPE_Q4_K, 3>(a, smem, s);
        case 4: return q6 ? launch_down_pairs_t<QWB_TYPE_Q6_K, 4>(a, smem, s) : launch_down_pairs_t<QWB_TYPE_Q4_K, 4>(a, smem, s);
        case 6: return q6 ? launch_down_pairs_t<QWB_TYPE_Q6_K, 6>(a, smem, s) : launch_down_pairs_t<QWB_TYPE_Q4_K, 6>(a, smem, s);
        default: return cudaErrorInvalidValue;
    }
}

cudaError_t run_pairs_layer(const PairsLayer &p, cudaStream_t s) {
    const bool sh = p.sh_down != nullptr;
    RouterDecodeArgs r{};
    r.x = p.x; r.router_w = p.router_w; r.mask = p.mask; r.norm_w = p.norm_w; r.norm_eps = p.norm_eps;
    r.H = p.H; r.E = p.E; r.n_used = p.n_used; r.T = p.T;
    r.g2s = p.g2s;
    r.n_slots[0] = p.gate->ne[2]; r.n_slots[1] = p.up->ne[2]; r.n_slots[2] = p.down->ne[2];
    r.own_lo = p.own_lo; r.own_n = p.own_n;
    r.sel = p.sel; r.wts = p.wts; r.slots = p.slots;
    r.xq = p.xq; r.kq = 1;
    r.sh_gate_inp = sh ? p.sh_gate_inp : nullptr;
    r.sh_scale = sh ? p.sh_scale : nullptr;
    r.st = p.st;
    cudaError_t e = launch_router_decode(r, s);
    if (e != cudaSuccess) return e;
    profile_mark(s, QWB_KERNEL_ROUTER);
    PairsCommon pc{};
    pc.T = p.T; pc.n_used = p.n_used; pc.slots = p.slots; pc.wts = p.wts;
    pc.shexp = sh ? 1 : 0;
    pc.sh_scale = sh ? p.sh_scale : nullptr;
    PairsGateUpArgs g{};
    g.pc = pc;
    g.Wg = (const uint8_t *) p.gate->data; g.Wu = (const uint8_t *) p.up->data;
    g.g_nb2 = p.gate->nb[2]; g.u_nb2 = p.up->nb[2]; g.row_bytes = row_bytes(p.gate->type, p.H);
    g.Wg_sh = sh ? (const uint8_t *) p.sh_gate->data : nullptr;
    g.Wu_sh = sh ? (const uint8_t *) p.sh_up->data : nullptr;
    g.F = p.F; g.K = p.H; g.n_slots_g = p.gate->ne[2]; g.n_slots_u = p.up->ne[2];
    g.xq = p.xq; g.act = p.act; g.st = p.st;
    e = launch_gateup_pairs(g, s);
    if (e != cudaSuccess) return e;
    profile_mark(s, QWB_KERNEL_GATE_UP);
    PairsDownArgs d{};
    d.pc = pc;
    d.W = (const uint8_t *) p.down->data; d.nb2 = p.down->nb[2]; d.row_bytes = row_bytes(p.down->type, p.F);
    d.W_sh = sh ? (const uint8_t *) p.sh_down->data : nullptr;
    d.F = p.F; d.H = p.H; d.n_slots = p.down->ne[2];
    d.act = p.act; d.out = p.out; d.residual = p.residual; d.st = p.st;
    e = launch_down_pairs(p.down->type, d, s);
    if (e != cudaSuccess) return e;
    profile_mark(s, QWB_KERNEL_DOWN);
    return cudaSuccess;
}

}  // namespace qwb

#ifdef QWB_DECODE_TRACE
extern "C" QWB_API int qwb_debug_decode_smid(void *host, size_t bytes) {
    return cudaMemcpyFromSymbol(host, qwb::g_decode_smid, bytes) == cudaSuccess ? 0 : 1;
}
extern "C" QWB_API int qwb_debug_decode_trace(void *host, size_t bytes) {
    return cudaMemcpyFromSymbol(host, qwb::g_decode_trace, bytes) == cudaSuccess ? 0 : 1;
}
#endif
