// mmid_one.cu - MUL_MAT_ID for a single token (T == 1) on Q4_K / Q6_K experts: the decode
// GEMV of a ggml graph's MUL_MAT_ID node (ggml_compute_forward_mul_mat_id,
// ggml-cpu/ggml-cpu.c:1554-1736, at n_tokens = 1), in ONE kernel launch.
//
// The (selected expert, row) pairs, n_used x M of them, are cut into one contiguous range
// per CTA (one CTA per SM).  Each CTA reads the expert ids, bulk-copies its rows (one copy
// per expert segment, all on one mbarrier), and while they are in flight quantizes the
// activation rows its segments use to Q8_K in shared memory (the CPU backend's
// from_float, bit for bit: quant_dev.cuh); no expert index and no separate quantizer
// kernel.  Lane = (row, superblock): one whole superblock dot per lane against the
// activation superblock it holds in registers (decode_dev.cuh), the NSB lanes of a row
// summed in superblock order.  Rows of an id outside [0, n_as) come out as zeros and the
// id is recorded (QWB_DEVERR_ID_RANGE), as the expert-index path does.
#include <algorithm>

#include "common.cuh"
#include "decode_dev.cuh"
#include "kernels.cuh"
#include "mmid.cuh"
#include "quant_dev.cuh"

namespace qwb {

namespace {

constexpr int kOneThreads = 256;
constexpr int kOneNW = kOneThreads / 32;
constexpr int kOneMaxUsed = 32;
constexpr int kOneActRows = 4;  // activation rows quantized per CTA (segments of one CTA)
constexpr size_t kOneMaxSmem = 220 * 1024;

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
__global__ void __launch_bounds__(kOneThreads, 1) mmid_one_kernel(const OneArgs a) {
    constexpr bool KQ6 = TYPE == QWB_TYPE_Q6_K;
    constexpr int SBB = KQ6 ? Q6K_BYTES : Q4K_BYTES;
    constexpr int RPS = 32 / NSB;  // rows per warp step
    constexpr int K = NSB * QK_K;
    // one Q8_K row: qs, d, bsum planes; rows 16-byte aligned (16-byte loads of qs)
    constexpr int kActBytes = (K + NSB * 36 + 15) / 16 * 16;
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bar = (uint64_t *) smem;
    uint8_t *actp = smem + 128;                              // [kOneActRows] Q8_K rows
    uint8_t *buf = actp + align_up((size_t) a.act_rows * kActBytes, 128);  // weight rows
    __shared__ int s_slot[kOneMaxUsed];
    __shared__ int s_base[kOneMaxUsed + 1];  // byte offset in buf of the first row of segment k (-1: none)
    __shared__ int s_act[kOneMaxUsed + 1];   // activation slot of segment k
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t M = a.M, P = (int64_t) a.n_used * M;
    const int64_t p0 = P * blockIdx.x / gridDim.x, p1 = P * (blockIdx.x + 1) / gridDim.x;
    const int n = (int) (p1 - p0);
    const int j_first = (int) (p0 / M);
    const int rlo_first = (int) (p0 - (int64_t) j_first * M);
    const int nseg = n > 0 ? (int) ((p1 - 1) / M) - j_first + 1 : 0;

    if (tid < a.n_used) {
        const int id = a.ids[(int64_t) tid * a.ids_s0];
        const bool ok = id >= 0 && id < a.n_as;
        s_slot[tid] = ok ? id : -1;
        if (!ok && blockIdx.x == 0) report(a.st, QWB_DEVERR_ID_RANGE, id);
    }
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) {  // one bulk copy per expert segment of the CTA's range
        uint32_t bytes = 0;
        for (int pass = 0; pass < 2; ++pass) {  // pass 0 counts, pass 1 issues
            if (pass == 1) mbar_arrive_expect_tx(&bar[0], bytes);
            size_t pos = 0;
            for (int k = 0; k < nseg; ++k) {
                const int j = j_first + k;
                const int64_t lo = k == 0 ? rlo_first : 0;
                const int64_t hi = std::min<int64_t>(M, p1 - (int64_t) j * M);
                const int slot = s_slot[j];
                if (slot < 0 || hi <= lo) {
                    if (pass == 1) s_base[k] = -1;
                    continue;
                }
                const uint8_t *src = a.W + (size_t) slot * a.nb2 + (size_t) lo * a.rb;
                const size_t len = (size_t) (hi - lo) * a.rb;
                const uint32_t span = bulk_span_bytes(src, len);
                if (pass == 0) {
                    bytes += span;
                } else {
                    const uint32_t off = bulk_span_issue(buf + pos, src, len, &bar[0]);
                    s_base[k] = (int) (pos + off);
                }
                pos += align_up((size_t) span, 16);
            }
        }
    }
    // activation rows of the CTA's segments -> Q8_K in shared memory (one 256-block per
    // warp task) while the weight copies are in flight; with n_b == 1 every segment uses
    // row 0, else segment k (expert j) uses row j % n_b (act_rows covers the segments)
    const int n_act = a.n_b == 1 ? 1 : min(nseg, a.act_rows);
    if (tid <= kOneMaxUsed) s_act[tid] = a.n_b == 1 ? 0 : tid;
    for (int task = warp; task < n_act * NSB; task += kOneNW) {
        const int slot = task / NSB, sb = task - slot * NSB;
        const int arow = a.n_b == 1 ? 0 : (j_first + slot) % a.n_b;
        uint8_t *row = actp + (size_t) slot * kActBytes;
        q8K_block_warp(a.x + (int64_t) arow * a.x_s1 + sb * QK_K, nullptr, (int8_t *) row + sb * QK_K,
                       (float *) (row + K) + sb, (int16_t *) (row + K + NSB * 4) + sb * 16);
    }
    __syncthreads();  // s_base, s_act and the quantized rows visible

    const int li = lane / NSB, ls = lane % NSB;
    const bool landed = mbar_wait(&bar[0], 0);
    if (!landed && lane == 0) report(a.st, QWB_DEVERR_TIMEOUT, (int) blockIdx.x);
    ActReg<KQ6> act;
    int cur = -1;  // activation row held in `act`
    for (int i0 = warp * RPS; i0 < n; i0 += kOneNW * RPS) {
        const int i = i0 + li;
        const bool in = li < RPS && i < n;
        const int64_t p = p0 + (in ? i : 0);
        const int j = (int) (p / M), r = (int) (p - (int64_t) j * M);
        const int k = j - j_first;
        float v = 0.f;
        if (in && landed && s_base[k] >= 0) {
            const int slot = s_act[k];
            if (slot != cur) {
                const uint8_t *row = actp + (size_t) slot * kActBytes;
                load_act<KQ6>(act, (const int8_t *) row + ls * QK_K, (const int16_t *) (row + K + NSB * 4) + ls * 16,
                              ((const float *) (row + K))[ls]);
                cur = slot;
            }
            const int rlo = k == 0 ? rlo_first : 0;
            const uint8_t *sb = buf + s_base[k] + (size_t) (r - rlo) * a.rb + (size_t) ls * SBB;
            if constexpr (KQ6) v = dot_q6K_sb(sb, act);
            else v = dot_q4K_sb(sb, act);
        }
        float tot = 0.f;
#pragma unroll
        for (int q = 0; q < NSB; ++q) tot += __shfl_sync(0xffffffffu, v, (li < RPS ? li : 0) * NSB + q);
        if (in && ls == 0) a.dst[(int64_t) j * a.dst_s1 + r] = tot;
    }
    // a timed-out wait leaves copies possibly in flight: drain them before the CTA exits
    if (!__syncthreads_and(landed) && tid == 0) mbar_wait(&bar[0], 0);
}

// Q8_K activation rows a CTA quantizes: one, or one per segment of its range
int one_act_rows(int64_t P, int64_t M, int n_b) {
    return n_b == 1 ? 1 : (int) (ceil_div(ceil_div(P, num_sms()), M) + 1);
}

size_t one_smem(int64_t P, int64_t K, int64_t M, int n_used, int n_b, size_t rb) {
    const int64_t rows = ceil_div(P, num_sms());
    const size_t row = align_up((size_t) (K + K / QK_K * 36), 16);  // as kActBytes in the kernel
    const size_t act = align_up((size_t) one_act_rows(P, M, n_b) * row, 128);
    // Q8_K rows + weight rows + each segment widened to 16-byte boundaries (< 32 bytes) +
    // the Q6_K dot's over-read past the last row
    return 128 + act + (size_t) rows * rb + 32 * (size_t) (n_used + 1) + 64;
}

template <int TYPE, int NSB>
cudaError_t launch_one_t(const OneArgs &a, size_t smem, cudaStream_t s) {
    static DeviceSmemLimit limit;
    auto kern = mmid_one_kernel<TYPE, NSB>;
    cudaError_t e = ensure_dyn_smem(kern, smem, limit);
    if (e != cudaSuccess) return e;
    // a plain launch: the ids come from the kernels before it in the stream
    kern<<<num_sms(), kOneThreads, smem, s>>>(a);
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
