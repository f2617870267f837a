// ep.cu - expert-parallel MoE layer: per-GPU routing/quantisation of its own tokens, and
// the SwiGLU expert FFN restricted to the experts a GPU owns (the collectives between the
// two are the caller's NCCL all-gather and reduce-scatter).
//
// The arithmetic per (token, slot) is build_moe's (core/runtime.cpp:2743-2816) with the
// reference CPU backend's numerics: activations quantized to the weights' vec_dot type
// (bit-exact, per row), integer sub-block dots, f32 combine.  Splitting the expert sum
// over GPUs changes only the f32 summation order of the weighted expert outputs.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"
#include "mmid.cuh"
#include "route.cuh"

namespace qwb {

// packed ggml blocks -> q8 planes (the layout the expert kernels read)
__global__ void unpack_q8K_kernel(const uint8_t *__restrict__ packed, int64_t n_rows, int64_t K, Q8Planes pl) {
    const int64_t nb = K / QK_K;
    const int64_t b = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // one block per warp
    const int lane = threadIdx.x & 31;
    if (b >= n_rows * nb) return;
    const int64_t r = b / nb, c = b - r * nb;
    // d (f32), qs[256], bsums[16]; blocks are 292 bytes, so only 4-byte alignment holds
    const uint8_t *src = packed + b * Q8K_BYTES;
    const uint32_t *q = (const uint32_t *) (src + 4 + 8 * lane);
    *(uint2 *) (pl.qs + r * K + c * QK_K + 8 * lane) = make_uint2(q[0], q[1]);
    if (lane == 0) pl.d[r * plane_d_stride(K, QK_K) + c] = *(const float *) src;
    if (lane < 16) pl.bsum[r * plane_bsum_stride(K) + c * 16 + lane] = *(const int16_t *) (src + 4 + QK_K + 2 * lane);
}
__global__ void unpack_q80_kernel(const uint8_t *__restrict__ packed, int64_t n_rows, int64_t K, Q8Planes pl) {
    const int64_t nb = K / QK8_0;
    const int64_t b = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;  // one block per thread
    if (b >= n_rows * nb) return;
    const int64_t r = b / nb, c = b - r * nb;
    const uint8_t *src = packed + b * Q80_BYTES;  // d (fp16), qs[32]
    pl.d[r * plane_d_stride(K, QK8_0) + c] = h2f(*(const uint16_t *) src);
    int8_t *dst = pl.qs + r * K + c * QK8_0;
    for (int i = 0; i < QK8_0; ++i) dst[i] = (int8_t) src[2 + i];
}

// q8 planes -> packed ggml blocks (the exchange format)
__global__ void pack_q8K_kernel(Q8Planes pl, int64_t n_rows, int64_t K, uint8_t *__restrict__ packed) {
    const int64_t nb = K / QK_K;
    const int64_t b = (int64_t) blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // one block per warp
    const int lane = threadIdx.x & 31;
    if (b >= n_rows * nb) return;
    const int64_t r = b / nb, c = b - r * nb;
    uint8_t *dst = packed + b * Q8K_BYTES;  // 4-byte aligned only (292-byte blocks)
    const uint2 q = *(const uint2 *) (pl.qs + r * K + c * QK_K + 8 * lane);
    uint32_t *d32 = (uint32_t *) (dst + 4 + 8 * lane);
    d32[0] = q.x;
    d32[1] = q.y;
    if (lane == 0) *(float *) dst = pl.d[r * plane_d_stride(K, QK_K) + c];
    if (lane < 16) *(int16_t *) (dst + 4 + QK_K + 2 * lane) = pl.bsum[r * plane_bsum_stride(K) + c * 16 + lane];
}
__global__ void pack_q80_kernel(Q8Planes pl, int64_t n_rows, int64_t K, uint8_t *__restrict__ packed) {
    const int64_t nb = K / QK8_0;
    const int64_t b = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (b >= n_rows * nb) return;
    const int64_t r = b / nb, c = b - r * nb;
    uint8_t *dst = packed + b * Q80_BYTES;
    *(uint16_t *) dst = f2h_rn(pl.d[r * plane_d_stride(K, QK8_0) + c]);  // exact: d came from an fp16
    const int8_t *src = pl.qs + r * K + c * QK8_0;
    for (int i = 0; i < QK8_0; ++i) dst[2 + i] = (uint8_t) src[i];
}

// local expert id of every (token, slot): id - lo when this GPU owns it, -1 otherwise;
// ids outside [0, E) are reported and also skipped
__global__ void local_ids_kernel(const int32_t *__restrict__ sel, int64_t P, int64_t lo, int64_t n_local, int64_t E,
                                 int32_t *__restrict__ lid, qwb_status_block *st) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= P) return;
    const int32_t e = sel[i];
    if (e < 0 || e >= E) report(st, QWB_DEVERR_ID_RANGE, e);
    lid[i] = (e >= lo && e < lo + n_local) ? (int32_t) (e - lo) : -1;
}

// out[t] = sum over local slots j of w[t][j] * ex[t][j]  (slot order, f32)
__global__ void weighted_sum_local_kernel(const float *__restrict__ ex, const float *__restrict__ w,
                                          const int32_t *__restrict__ lid, float *__restrict__ out, int64_t H,
                                          int n_used, int64_t T) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= H * T) return;
    const int64_t t = i / H, h = i - t * H;
    float acc = 0.f;
    for (int j = 0; j < n_used; ++j)
        if (lid[t * n_used + j] >= 0) acc = fmaf(w[t * n_used + j], ex[(t * n_used + j) * H + h], acc);
    out[i] = acc;
}

}  // namespace qwb

using namespace qwb;

namespace {

bool ok_weight_type(int t) { return t == QWB_TYPE_Q4_K || t == QWB_TYPE_Q6_K || t == QWB_TYPE_Q8_0; }

// ------------------------------------------------------------------ prepare
// few tokens: the fused router kernel (H % 1024 == 0)
bool fused_router(const qwb_moe_ep_prepare_desc *d) { return d->T <= kMaxRouterT && d->H % 1024 == 0; }

struct PrepPlan {
    size_t off_logits, off_xn, off_planes, total;
};
qwb_status plan_prep(const qwb_moe_ep_prepare_desc *d, PrepPlan &p) {
    if (!d) return QWB_ERR_INVALID_ARG;
    if (d->H <= 0 || d->E <= 0 || d->n_used <= 0 || d->T < 0) return QWB_ERR_INVALID_ARG;
    if (d->E > kMaxExperts || d->n_used > kMaxUsed || d->n_used > d->E) return QWB_ERR_LIMIT;
    if (d->act_type != QWB_TYPE_Q8_K && d->act_type != QWB_TYPE_Q8_0) return QWB_ERR_UNSUPPORTED_TYPE;
    if (d->H % QK_K) return QWB_ERR_SHAPE;
    size_t o = kCtrlBytes;
    p.off_logits = o;
    o += align_up((size_t) (d->T * d->E) * 4, 256);
    p.off_xn = o;
    if (d->norm_w) o += align_up((size_t) (d->T * d->H) * 4, 256);
    p.off_planes = o;
    if (fused_router(d)) o += planes_bytes(d->T, d->H, d->act_type == QWB_TYPE_Q8_K);
    p.total = o;
    return QWB_OK;
}

// ------------------------------------------------------------------ experts
struct ExpPlan {
    bool kq_gu, kq_d;
    int NT;
    bool stream;  // expert GEMVs on the streaming kernel (index: one tile per expert)
    int64_t P, n_local;
    size_t off_xq, off_lid, off_index, off_act, off_actq, off_ex, total;
};
qwb_status plan_exp(const qwb_moe_ep_experts_desc *d, ExpPlan &p) {
    if (!d) return QWB_ERR_INVALID_ARG;
    if (d->H <= 0 || d->F <= 0 || d->E <= 0 || d->n_used <= 0 || d->T < 0) return QWB_ERR_INVALID_ARG;
    if (d->n_used > kMaxUsed || d->n_used > d->E || d->E > kMaxExperts) return QWB_ERR_LIMIT;
    const int tg = d->gate.type, td = d->down.type;
    if (!ok_weight_type(tg) || !ok_weight_type(td) || d->up.type != tg) return QWB_ERR_UNSUPPORTED_TYPE;
    if (d->H % 1024 || d->F % 256) return QWB_ERR_SHAPE;
    p.n_local = d->gate.ne[2];
    if (p.n_local <= 0 || d->expert_lo < 0 || d->expert_lo + p.n_local > d->E) return QWB_ERR_SHAPE;
    if (d->gate.ne[0] != d->H || d->gate.ne[1] != d->F || d->up.ne[0] != d->H || d->up.ne[1] != d->F ||
        d->up.ne[2] != p.n_local || d->down.ne[0] != d->F || d->down.ne[1] != d->H || d->down.ne[2] != p.n_local)
        return QWB_ERR_SHAPE;
    p.kq_gu = tg != QWB_TYPE_Q8_0;
    p.kq_d = td != QWB_TYPE_Q8_0;
    p.P = d->n_used * d->T;
    p.stream = stream_fits_ffn(tg, d->H, d->gate.nb[1], d->up.nb[1], td, d->F, d->down.nb[1]);
    p.NT = p.stream ? (int) std::max<int64_t>(1, p.P) : pick_nt(std::max<int64_t>(1, p.P * p.n_local / d->E), p.n_local);
    size_t o = kCtrlBytes;
    p.off_xq = o; o += planes_bytes(d->T, d->H, p.kq_gu);
    p.off_lid = o; o += align_up((size_t) p.P * 4, 256);
    p.off_index = o; o += mmid_index_bytes(std::max<int64_t>(p.P, 1), p.n_local, p.NT);
    p.off_act = o; o += align_up((size_t) p.P * d->F * 4, 256);
    p.off_actq = o; o += planes_bytes(p.P, d->F, p.kq_d);
    p.off_ex = o; o += align_up((size_t) p.P * d->H * 4, 256);
    p.total = o;
    return QWB_OK;
}

}  // namespace

extern "C" QWB_API size_t qwb_moe_ep_prepare_workspace_size(const qwb_moe_ep_prepare_desc *desc) {
    PrepPlan p;
    return plan_prep(desc, p) == QWB_OK ? p.total : 0;
}

extern "C" QWB_API qwb_status qwb_moe_ep_prepare(const qwb_moe_ep_prepare_desc *d, void *ws, size_t ws_bytes,
                                                 qwb_status_block *st, qwb_stream_t stream) {
    PrepPlan p;
    qwb_status rc = plan_prep(d, p);
    if (rc != QWB_OK) return rc;
    if (d->T == 0) return QWB_OK;
    if (!d->x || !d->router_w || !d->xq || !d->selected || !d->weights) return QWB_ERR_INVALID_ARG;
    if (!ws || ws_bytes < p.total) return QWB_ERR_WORKSPACE;
    if ((uintptr_t) ws % 256) return QWB_ERR_ALIGNMENT;
    if (((uintptr_t) d->x | (uintptr_t) d->router_w | (uintptr_t) d->norm_w) % 16) return QWB_ERR_ALIGNMENT;
    cudaStream_t s = (cudaStream_t) stream;
    char *w = (char *) ws;
    const bool kq = d->act_type == QWB_TYPE_Q8_K;
    if (fused_router(d)) {
        // few tokens: one fused launch (norm, router GEMV, top-k, Q8 planes), then pack
        Q8Planes pl = planes_at(w + p.off_planes, d->T, d->H, kq);
        RouterArgs r{};
        r.x = d->x; r.router_w = d->router_w; r.mask = d->mask;
        r.H = d->H; r.E = d->E; r.T = d->T; r.n_used = d->n_used;
        r.logits = (float *) (w + p.off_logits);
        r.counter = (unsigned *) w;
        r.selected = d->selected; r.weights = d->weights;
        r.xq = pl; r.kq = kq;
        r.norm_w = d->norm_w; r.norm_eps = d->norm_eps;
        cudaError_t e = launch_router_fused(r, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
        if (kq) {
            const int64_t blocks = d->T * (d->H / QK_K);
            pack_q8K_kernel<<<(unsigned) ceil_div(blocks, 8), 256, 0, s>>>(pl, d->T, d->H, (uint8_t *) d->xq);
        } else {
            const int64_t blocks = d->T * (d->H / QK8_0);
            pack_q80_kernel<<<(unsigned) ceil_div(blocks, 256), 256, 0, s>>>(pl, d->T, d->H, (uint8_t *) d->xq);
        }
        return cudaGetLastError() == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
    }
    const float *xin = d->x;
    cudaError_t e = cudaSuccess;
    if (d->norm_w) {
        float *xn = (float *) (w + p.off_xn);
        e = launch_rmsnorm(d->x, d->norm_w, d->norm_eps, d->T, d->H, xn, s);
        xin = xn;
    }
    float *logits = (float *) (w + p.off_logits);
    if (e == cudaSuccess) e = launch_logits_gemm(xin, d->router_w, logits, d->T, d->E, d->H, s);
    if (e == cudaSuccess) e = launch_route(logits, d->mask, d->E, d->T, d->n_used, 1, 0.0f, d->selected, d->weights, s);
    Q8Planes none{};
    if (e == cudaSuccess)
        e = launch_quantize_rows(d->act_type == QWB_TYPE_Q8_K ? 0 : 1, xin, d->H, d->T, d->H, (uint8_t *) d->xq, none,
                                 nullptr, s);
    return e == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
}

extern "C" QWB_API size_t qwb_moe_ep_experts_workspace_size(const qwb_moe_ep_experts_desc *desc) {
    ExpPlan p;
    return plan_exp(desc, p) == QWB_OK ? p.total : 0;
}

extern "C" QWB_API qwb_status qwb_moe_ep_experts(const qwb_moe_ep_experts_desc *d, void *ws, size_t ws_bytes,
                                                 qwb_status_block *st, qwb_stream_t stream) {
    ExpPlan p;
    qwb_status rc = plan_exp(d, p);
    if (rc != QWB_OK) return rc;
    if (d->T == 0) return QWB_OK;
    if (!d->xq || !d->selected || !d->weights || !d->out || !d->gate.data || !d->up.data || !d->down.data)
        return QWB_ERR_INVALID_ARG;
    if (!ws || ws_bytes < p.total) return QWB_ERR_WORKSPACE;
    if ((uintptr_t) ws % 256) return QWB_ERR_ALIGNMENT;
    if (((uintptr_t) d->xq % (p.kq_gu ? 4 : 2)) || ((uintptr_t) d->out % 16)) return QWB_ERR_ALIGNMENT;
    for (const qwb_tensor *t : {&d->gate, &d->up, &d->down}) {
        if (t->nb[0] != row_bytes(t->type, block_elems(t->type))) return QWB_ERR_LAYOUT;
        if (t->nb[1] < row_bytes(t->type, t->ne[0]) || t->nb[2] < t->nb[1] * (size_t) t->ne[1]) return QWB_ERR_LAYOUT;
        const uintptr_t al = (uintptr_t) t->data | t->nb[1] | t->nb[2];
        if (t->type == QWB_TYPE_Q4_K ? al % 16 : al % 2) return QWB_ERR_ALIGNMENT;
    }
    cudaStream_t s = (cudaStream_t) stream;
    char *w = (char *) ws;
    const int64_t H = d->H, F = d->F, T = d->T, K = d->n_used, P = p.P, NL = p.n_local;
    Q8Planes xq = planes_at(w + p.off_xq, T, H, p.kq_gu);
    int32_t *lid = (int32_t *) (w + p.off_lid);
    MmidIndex ix = mmid_index_at(w + p.off_index, std::max<int64_t>(P, 1), NL, p.NT);
    float *act = (float *) (w + p.off_act);
    float *ex = (float *) (w + p.off_ex);
    cudaError_t e;
    profile_mark(s, 0);
    if (p.kq_gu) {
        const int64_t blocks = T * (H / QK_K);
        unpack_q8K_kernel<<<(unsigned) ceil_div(blocks, 8), 256, 0, s>>>((const uint8_t *) d->xq, T, H, xq);
    } else {
        const int64_t blocks = T * (H / QK8_0);
        unpack_q80_kernel<<<(unsigned) ceil_div(blocks, 256), 256, 0, s>>>((const uint8_t *) d->xq, T, H, xq);
    }
    e = cudaGetLastError();
    if (e != cudaSuccess) return QWB_ERR_CUDA;
    local_ids_kernel<<<(unsigned) ceil_div(P, 256), 256, 0, s>>>(d->selected, P, d->expert_lo, NL, d->E, lid, st);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = launch_index(lid, 1, K, (int) K, (int) T, (int) NL, p.NT, ix, nullptr, 0, 0, 0, st, s, 1);
    if (e != cudaSuccess) return QWB_ERR_CUDA;
    profile_mark(s, QWB_KERNEL_ROUTER);
    {
        GemvArgs a{};
        a.W = (const uint8_t *) d->gate.data; a.nb1 = d->gate.nb[1]; a.nb2 = d->gate.nb[2];
        a.W2 = (const uint8_t *) d->up.data; a.nb1_2 = d->up.nb[1]; a.nb2_2 = d->up.nb[2];
        a.row_bytes = row_bytes(d->gate.type, H);
        a.M = F; a.K = H;
        a.act = xq;
        a.tiles = ix.tiles; a.n_tiles = ix.n_tiles; a.pairs = ix.pairs;
        a.n_used = (int) K; a.n_b = 1;
        a.dst = act; a.dnb1 = (size_t) F * 4; a.dnb2 = (size_t) K * F * 4;
        a.n_ids = NL; a.n_slots = NL;
        a.st = st;
        e = launch_expert_gemv(d->gate.type, true, a, p.stream, p.NT, ix.max_tiles, P, NL, ix.work, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
        profile_mark(s, QWB_KERNEL_GATE_UP);
    }
    Q8Planes aq = planes_at(w + p.off_actq, P, F, p.kq_d);
    e = launch_quantize_rows(p.kq_d ? 0 : 1, act, F, P, F, nullptr, aq, nullptr, s);
    if (e != cudaSuccess) return QWB_ERR_CUDA;
    {
        GemvArgs a{};
        a.W = (const uint8_t *) d->down.data; a.nb1 = d->down.nb[1]; a.nb2 = d->down.nb[2];
        a.row_bytes = row_bytes(d->down.type, F);
        a.M = H; a.K = F;
        a.act = aq;
        a.tiles = ix.tiles; a.n_tiles = ix.n_tiles; a.pairs = ix.pairs;
        a.n_used = (int) K; a.n_b = (int) K;
        a.dst = ex; a.dnb1 = (size_t) H * 4; a.dnb2 = (size_t) K * H * 4;
        a.n_ids = NL; a.n_slots = NL;
        a.st = st;
        e = launch_expert_gemv(d->down.type, false, a, p.stream, p.NT, ix.max_tiles, P, NL, ix.work + 1, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
        profile_mark(s, QWB_KERNEL_DOWN);
    }
    weighted_sum_local_kernel<<<(unsigned) ceil_div(H * T, 256), 256, 0, s>>>(ex, d->weights, lid, d->out, H, (int) K, T);
    e = cudaGetLastError();
    profile_mark(s, QWB_KERNEL_OTHER);
    return e == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
}
