// mmid_one.cu - MUL_MAT_ID for a single token (T == 1) on Q4_K / Q6_K experts: the decode
// GEMV of a ggml graph's MUL_MAT_ID node (ggml_compute_forward_mul_mat_id,
// ggml-cpu/ggml-cpu.c:1554-1736, at n_tokens = 1), in ONE kernel launch.
//
// The (selected expert, row) pairs, n_used x M of them, are cut into one contiguous range
// per CTA (one CTA per SM).  Each CTA reads the expert ids and bulk-copies its rows in
// kOneChunks consecutive chunks, each on its own mbarrier (one copy per expert segment of
// a chunk), so the dots on a landed chunk overlap the flight of the later ones.  While the
// first chunk is in flight it quantizes the activation rows its segments use to Q8_K in
// shared memory (the CPU backend's from_float, bit for bit: quant_dev.cuh; each warp's
// first 256 values are loaded before the copies start, so that read does not queue behind
// them); no expert index and no separate quantizer kernel.  Lane = (row, superblock): one
// whole superblock dot per lane against the activation superblock it holds in registers
// (decode_dev.cuh), the NSB lanes of a row summed in superblock order; a chunk's warp
// steps are dealt round-robin continuing from the previous chunk, so no warp idles while
// another takes two steps.  Rows of an id outside [0, n_as) come out as zeros and the id
// is recorded (QWB_DEVERR_ID_RANGE), as the expert-index path does.
#include <algorithm>

#include "common.cuh"
#include "decode_dev.cuh"
#include "kernels.cuh"
#include "mmid.cuh"
#include "quant_dev.cuh"

namespace qwb {

namespace {

// 16 warps for Q4_K (the dots are latency-bound: more warps per scheduler), 12 for Q6_K,
// whose dot needs more registers (a 16-warp CTA caps them at 128)
template <int TYPE>
constexpr int one_threads() { return TYPE == QWB_TYPE_Q6_K ? 384 : 512; }
constexpr int kOneMaxUsed = 32;
constexpr int kOneChunks = 4;   // mbarrier chunks of a CTA's rows
constexpr int kOneActRows = 4;  // activation rows quantized per CTA (segments of one CTA)
// shared-memory Q8_K row: per superblock 256 + 16 bytes of qs, a 4-byte d, 16 + 2 bsums
constexpr int kOneQsStride = QK_K + 16, kOneBsStride = 18;
constexpr int kOneActSbBytes = kOneQsStride + 4 + 2 * kOneBsStride;
constexpr size_t kOneMaxSmem = 220 * 1024;

// Optional phase timestamps (compiled in only with -DQWB_DECODE_TRACE; no effect on the
// default build): thread 0 of each CTA records the global timer at numbered points.
#ifdef QWB_DECODE_TRACE
__device__ unsigned long long g_one_trace[160][12];
#define ONE_TRACE(p)                                                                           \
    do {                                                                                       \
        if (threadIdx.x == 0 && blockIdx.x < 160) g_one_trace[blockIdx.x][p] = globaltimer_ns(); \
    } while (0)
#else
#define ONE_TRACE(p) \
    do {             \
    } while (0)
#endif

struct OneArgs {
    const uint8_t *W;
    size_t nb2, rb;          // expert stride, row bytes (rows contiguous)
    int64_t M, K, n_as;
    const int32_t *ids;      // ids[j * ids_s0], j < n_used
    int64_t ids_s0;
    int n_used, n_b;
    const float *x;          // activation row a at x + a * x_s1 (f32, n_b rows)
    int64_t x_s1;
    int act_rows;            // Q8_K rows a CTA holds (1, or its segments' rows)
    float *dst;              // element (r, j) at dst[j * dst_s1 + r]
    int64_t dst_s1;
    qwb_status_block *st;
};

template <int TYPE, int NSB>
__global__ void __launch_bounds__(one_threads<TYPE>(), 1) mmid_one_kernel(const OneArgs a) {
    constexpr bool KQ6 = TYPE == QWB_TYPE_Q6_K;
    constexpr int NW = one_threads<TYPE>() / 32;
    constexpr int SBB = KQ6 ? Q6K_BYTES : Q4K_BYTES;
    constexpr int RPS = 32 / NSB;  // rows per warp step
    // one Q8_K row: qs, d and bsum planes, each superblock's qs padded to 272 bytes and its
    // 16 bsums to 36 so that the NSB lanes loading their superblocks hit distinct banks (at
    // 256 / 32 bytes eight lanes of a quarter-warp share banks); rows 16-byte aligned
    constexpr int kActBytes = (NSB * kOneActSbBytes + 15) / 16 * 16;
    constexpr int kD = NSB * kOneQsStride, kBs = kD + NSB * 4;  // d and bsum planes
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bar = (uint64_t *) smem;                       // [kOneChunks]
    uint8_t *actp = smem + 128;                              // [act_rows] Q8_K rows
    uint8_t *buf = actp + align_up((size_t) a.act_rows * kActBytes, 128);  // weight rows
    __shared__ int s_slot[kOneMaxUsed];
    // s_base[c][k]: row i (CTA-local) of segment k, copied with chunk c, starts at
    // buf + s_base[c][k] + i * rb
    __shared__ int s_base[kOneChunks][kOneMaxUsed + 1];
    __shared__ int s_act[kOneMaxUsed + 1];  // activation slot of segment k
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t M = a.M, P = (int64_t) a.n_used * M;
    const int64_t p0 = P * blockIdx.x / gridDim.x, p1 = P * (blockIdx.x + 1) / gridDim.x;
    const int n = (int) (p1 - p0);
    const int j_first = (int) (p0 / M);
    const int rlo_first = (int) (p0 - (int64_t) j_first * M);
    const int nseg = n > 0 ? (int) ((p1 - 1) / M) - j_first + 1 : 0;
    const int nch = min(kOneChunks, max(1, n));
    auto chunk_lo = [&](int c) { return n * c / nch; };
    const int rb = (int) a.rb;
    const int Mi = (int) M;  // rlo_first + i < M + n fits an int

    // activation rows of the CTA's segments: with n_b == 1 every segment uses row 0, else
    // segment k (expert j) uses row j % n_b (act_rows covers the segments); one 256-value
    // block per warp task, the first task's values read now (they do not need the ids)
    const int n_act = a.n_b == 1 ? 1 : min(nseg, a.act_rows);
    auto task_x = [&](int task) {
        const int slot = task / NSB, sb = task - slot * NSB;
        const int arow = a.n_b == 1 ? 0 : (j_first + slot) % a.n_b;
        return a.x + (int64_t) arow * a.x_s1 + sb * QK_K;
    };
    float xv[8];
    if (warp < n_act * NSB) load8_normed(task_x(warp), 1.f, nullptr, lane, xv);

    ONE_TRACE(0);
    if (tid < a.n_used) {
        const int id = a.ids[(int64_t) tid * a.ids_s0];
        const bool ok = id >= 0 && id < a.n_as;
        s_slot[tid] = ok ? id : -1;
        if (!ok && blockIdx.x == 0) report(a.st, QWB_DEVERR_ID_RANGE, id);
    }
    if (tid == 0) {
        for (int c = 0; c < nch; ++c) mbar_init(&bar[c], 1);
        fence_mbar_init();
    }
    __syncthreads();
    ONE_TRACE(1);
    if (tid < nch) {  // thread c issues chunk c: one bulk copy per expert segment of the chunk
        const int c = tid;
        const int c0 = chunk_lo(c), c1 = chunk_lo(c + 1);
        // chunk c's region (16-byte aligned): starts past chunks < c, each at most its rows
        // plus < 32 bytes of widening per segment it touches (<= nseg) and 16 of alignment
        const size_t base = align_up((size_t) c0 * rb + (size_t) 32 * c * (nseg + 1), 16);
        const int q0 = rlo_first + c0;  // < M + n: fits an int
        const int k0 = q0 / Mi, r0 = q0 - k0 * Mi;
        uint32_t bytes = 0;
        for (int pass = 0; pass < 2; ++pass) {  // pass 0 counts, pass 1 issues
            if (pass == 1) mbar_arrive_expect_tx(&bar[c], bytes);
            size_t pp = base;
            int k = k0, r = r0;
            for (int i = c0; i < c1; r = 0, ++k) {
                const int len = min(c1 - i, Mi - r);
                const int slot = s_slot[j_first + k];
                if (slot >= 0) {
                    const uint8_t *src = a.W + (size_t) slot * a.nb2 + (size_t) r * a.rb;
                    const size_t bytes_k = (size_t) len * a.rb;
                    const uint32_t span = bulk_span_bytes(src, bytes_k);
                    if (pass == 0) {
                        bytes += span;
                    } else {
                        const uint32_t off = bulk_span_issue(buf + pp, src, bytes_k, &bar[c]);
                        s_base[c][k] = (int) (pp + off) - i * rb;
                    }
                    pp += span;  // a multiple of 16
                }
                i += len;
            }
        }
    }
    ONE_TRACE(2);
    if (tid <= kOneMaxUsed) s_act[tid] = a.n_b == 1 ? 0 : tid;
    for (int task = warp; task < n_act * NSB; task += NW) {
        const int slot = task / NSB, sb = task - slot * NSB;
        if (task != warp) load8_normed(task_x(task), 1.f, nullptr, lane, xv);
        uint8_t *row = actp + (size_t) slot * kActBytes;
        q8K_block_vals(xv, nullptr, (int8_t *) row + sb * kOneQsStride, (float *) (row + kD) + sb,
                       (int16_t *) (row + kBs) + sb * kOneBsStride);
    }
    __syncthreads();  // s_base, s_act and the quantized rows visible
    ONE_TRACE(3);

    const int li = lane / NSB, ls = lane % NSB;
    ActReg<KQ6> act;
    int cur = -1;  // activation row held in `act`
    bool alive = true;
    int dealt = 0;  // warp steps of the chunks before this one
    for (int c = 0; c < nch; ++c) {
        const int c0 = chunk_lo(c), c1 = chunk_lo(c + 1);
        const int steps = (c1 - c0 + RPS - 1) / RPS;
        if (!mbar_wait(&bar[c], 0)) {
            if (lane == 0) report(a.st, QWB_DEVERR_TIMEOUT, (int) blockIdx.x);
            alive = false;
            break;
        }
        ONE_TRACE(4 + c);
        for (int g = ((warp - dealt) % NW + NW) % NW; g < steps; g += NW) {
            const int i = c0 + g * RPS + li;
            const bool in = li < RPS && i < c1;
            const int q = rlo_first + (in ? i : c0);
            const int k = q / Mi, r = q - k * Mi;
            const int j = j_first + k;
            float v = 0.f;
            if (in && s_slot[j] >= 0) {
                const int slot = s_act[k];
                if (slot != cur) {
                    const uint8_t *row = actp + (size_t) slot * kActBytes;
                    load_act<KQ6>(act, (const int8_t *) row + ls * kOneQsStride,
                                  (const int16_t *) (row + kBs) + ls * kOneBsStride, ((const float *) (row + kD))[ls]);
                    cur = slot;
                }
                const uint8_t *sb = buf + s_base[c][k] + i * rb + ls * SBB;
                if constexpr (KQ6) v = dot_q6K_sb(sb, act);
                else v = dot_q4K_sb(sb, act);
            }
            float tot = 0.f;
#pragma unroll
            for (int t = 0; t < NSB; ++t) tot += __shfl_sync(0xffffffffu, v, (li < RPS ? li : 0) * NSB + t);
            if (in && ls == 0) a.dst[(int64_t) j * a.dst_s1 + r] = tot;
        }
        dealt += steps;
    }
    ONE_TRACE(8);
    // a timed-out wait leaves copies possibly in flight: drain them before the CTA exits
    if (!__syncthreads_and(alive) && tid == 0)
        for (int c = 0; c < nch; ++c) mbar_wait(&bar[c], 0);
    ONE_TRACE(9);
}

// Q8_K activation rows a CTA quantizes: one, or one per segment of its range
int one_act_rows(int64_t P, int64_t M, int n_b) {
    return n_b == 1 ? 1 : (int) (ceil_div(ceil_div(P, num_sms()), M) + 1);
}

size_t one_smem(int64_t P, int64_t K, int64_t M, int n_used, int n_b, size_t rb) {
    const int64_t rows = ceil_div(P, num_sms());
    const size_t row = align_up((size_t) (K / QK_K * kOneActSbBytes), 16);  // as kActBytes in the kernel
    const size_t act = align_up((size_t) one_act_rows(P, M, n_b) * row, 128);
    // Q8_K rows + weight rows + 32 bytes per chunk and segment of the CTA's range (each
    // copied piece widened to 16-byte boundaries) + the Q6_K dot's over-read past the last row
    const int64_t segs = std::min<int64_t>(n_used, ceil_div(rows, M) + 1);
    return 128 + act + (size_t) rows * rb + (size_t) 32 * kOneChunks * (segs + 1) + 64;
}

template <int TYPE, int NSB>
cudaError_t launch_one_t(const OneArgs &a, size_t smem, cudaStream_t s) {
    static DeviceSmemLimit limit;
    auto kern = mmid_one_kernel<TYPE, NSB>;
    cudaError_t e = ensure_dyn_smem(kern, smem, limit);
    if (e != cudaSuccess) return e;
    // a plain launch: the ids come from the kernels before it in the stream
    kern<<<num_sms(), one_threads<TYPE>(), smem, s>>>(a);
    return cudaGetLastError();
}

using OneLaunch = cudaError_t (*)(const OneArgs &, size_t, cudaStream_t);

OneLaunch pick_one(int type, int64_t K) {
    const bool q6 = type == QWB_TYPE_Q6_K;
    if (type != QWB_TYPE_Q4_K && type != QWB_TYPE_Q6_K) return nullptr;
    switch (K / QK_K) {
        case 3: return q6 ? launch_one_t<QWB_TYPE_Q6_K, 3> : launch_one_t<QWB_TYPE_Q4_K, 3>;
        case 6: return q6 ? launch_one_t<QWB_TYPE_Q6_K, 6> : launch_one_t<QWB_TYPE_Q4_K, 6>;
        case 8: return q6 ? launch_one_t<QWB_TYPE_Q6_K, 8> : launch_one_t<QWB_TYPE_Q4_K, 8>;
        case 16: return q6 ? launch_one_t<QWB_TYPE_Q6_K, 16> : launch_one_t<QWB_TYPE_Q4_K, 16>;
        default: return nullptr;
    }
}

}  // namespace

bool mmid_one_supported(int type, int64_t K, int64_t M, int n_used, int n_b, size_t nb1) {
    if (K % QK_K || !pick_one(type, K)) return false;
    const size_t rb = row_bytes(type, K);
    if (nb1 != rb || (type == QWB_TYPE_Q4_K && rb % 16)) return false;
    if (n_used < 1 || n_used > kOneMaxUsed || n_b < 1 || n_used % n_b) return false;
    const int64_t P = (int64_t) n_used * M;
    // with one activation row per slot, a CTA quantizes the rows of all its segments
    if (one_act_rows(P, M, n_b) > kOneActRows) return false;
    return one_smem(P, K, M, n_used, n_b, rb) <= kOneMaxSmem;
}

cudaError_t launch_mmid_one(int type, const uint8_t *W, size_t nb2, int64_t M, int64_t K, int64_t n_as,
                            const int32_t *ids, int64_t ids_s0, int n_used, int n_b, const float *x, int64_t x_s1,
                            float *dst, int64_t dst_s1, qwb_status_block *st, cudaStream_t s) {
    const OneLaunch lf = pick_one(type, K);
    if (!lf) return cudaErrorInvalidValue;
    OneArgs a{};
    a.W = W;
    a.nb2 = nb2;
    a.rb = row_bytes(type, K);
    a.M = M;
    a.K = K;
    a.n_as = n_as;
    a.ids = ids;
    a.ids_s0 = ids_s0;
    a.n_used = n_used;
    a.n_b = n_b;
    a.x = x;
    a.x_s1 = x_s1;
    a.act_rows = one_act_rows((int64_t) n_used * M, M, n_b);
    a.dst = dst;
    a.dst_s1 = dst_s1;
    a.st = st;
    return lf(a, one_smem((int64_t) n_used * M, K, M, n_used, n_b, a.rb), s);
}

}  // namespace qwb

#ifdef QWB_DECODE_TRACE
extern "C" QWB_API int qwb_debug_one_trace(void *host, size_t bytes) {
    return cudaMemcpyFromSymbol(host, qwb::g_one_trace, bytes) == cudaSuccess ? 0 : 1;
}
#endif
