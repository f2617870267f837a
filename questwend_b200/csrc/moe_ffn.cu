// moe_ffn.cu - the fused MoE FFN layer (QuestWend's build_moe subgraph) on B200.
//
// Reference: core/runtime.cpp:2743-2816 (build_moe), :2769-2778 (in-graph slot remap),
// :2693-2734 (route_experts).  The chain router mul_mat -> softmax/top-k/renorm ->
// get_rows(g2s) -> 3x mul_mat_id -> swiglu -> weighted reduce runs as
//   decode (T == 1), 3 kernels:
//     router_fused   logits GEMV + x -> Q8 + top-k (last CTA) + GEMV tile list
//     gemv<GLU>      gate and up rows of each selected expert slot, SwiGLU epilogue
//     down_decode    act -> Q8 in the prologue (overlapping the weight copies), down
//                    rows of all selected slots per output row, weighted sum + residual
//   batched (T > 1): router (+ quantize x), index build, gemv<GLU>, act -> Q8,
//                    gemv (down, n_b = n_used), weighted sum + residual.
// Numerics are the reference CPU backend's: Q8_K (or Q8_0-cpu) activations bit-exact,
// integer sub-block dots exact, fp32 combine (see dot.cuh).
#include <algorithm>

#include "common.cuh"
#include "decode.cuh"
#include "dot.cuh"
#include "kernels.cuh"
#include "mmid.cuh"
#include "moe.cuh"
#include "quant_dev.cuh"
#include "route.cuh"

namespace qwb {

struct DownArgs {
    const uint8_t *W;
    size_t nb1, nb2, row_bytes;
    int64_t n_slots, E;
    const int32_t *remap;      // g2s down table [E] or null
    const int32_t *selected;   // [n_used] logical expert ids
    const float *weights;      // [n_used]
    int n_used;
    const float *act;          // [n_used][F] f32
    int64_t F, H;
    float *out;
    const float *residual;
    const float *sh, *sh_scale;  // shared expert output [H] and its factor, or null
    int kq;
    int R, n_rb, wspan, act_stride, act_d_off, act_b_off, smem_act;
    qwb_status_block *st;
};

template <int TYPE>
__global__ void __launch_bounds__(128) moe_down_decode_kernel(const DownArgs d) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bar = (uint64_t *) smem;
    __shared__ int64_t s_slot[kMaxUsed];
    __shared__ float s_w[kMaxUsed];
    uint8_t *act = smem + 128;
    uint8_t *wbuf = act + d.smem_act;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int64_t per = ceil_div((int64_t) d.n_rb, (int64_t) gridDim.x);
    const int64_t i0 = (int64_t) blockIdx.x * per, i1 = min((int64_t) d.n_rb, i0 + per);
    if (i0 >= i1) return;

    if (tid < d.n_used) {
        const int e = d.selected[tid];
        int64_t sl = -1;
        if (e >= 0 && e < d.E) sl = d.remap ? (int64_t) d.remap[e] : e;
        if (sl < 0 || sl >= d.n_slots) {
            if (blockIdx.x == 0) report(d.st, QWB_DEVERR_ID_RANGE, e);
            sl = -1;
        }
        s_slot[tid] = sl;
        s_w[tid] = d.weights[tid];
    }
    if (tid == 0) {
        mbar_init(&bar[0], 1);
        fence_mbar_init();
    }
    __syncthreads();

    auto issue = [&](int64_t it) {
        const int64_t r0 = it * d.R;
        const int nr = (int) min((int64_t) d.R, d.H - r0);
        const size_t span = (size_t) (nr - 1) * d.nb1 + d.row_bytes;
        uint32_t bytes = 0;
        for (int j = 0; j < d.n_used; ++j)
            if (s_slot[j] >= 0) bytes += bulk_span_bytes(d.W + (size_t) s_slot[j] * d.nb2 + (size_t) r0 * d.nb1, span);
        mbar_arrive_expect_tx(&bar[0], bytes);
        for (int j = 0; j < d.n_used; ++j)
            if (s_slot[j] >= 0)
                bulk_span_issue(wbuf + j * d.wspan, d.W + (size_t) s_slot[j] * d.nb2 + (size_t) r0 * d.nb1, span,
                                &bar[0]);
    };
    if (tid == 0) issue(i0);

    // prologue (overlaps the first copy): quantize the n_used act rows into shared memory
    {
        const int64_t nck = d.F / 256;
        for (int64_t c = warp; c < d.n_used * nck; c += 4) {
            const int j = (int) (c / nck);
            const int64_t cc = c - j * nck;
            uint8_t *tok = act + j * d.act_stride;
            const float *x = d.act + (int64_t) j * d.F + cc * 256;
            if (d.kq)
                q8K_block_warp(x, nullptr, (int8_t *) tok + cc * 256, (float *) (tok + d.act_d_off) + cc,
                               (int16_t *) (tok + d.act_b_off) + cc * 16);
            else
                q80_8blocks_warp(x, QWB_Q8_0_CPU, nullptr, (int8_t *) tok + cc * 256,
                                 (float *) (tok + d.act_d_off) + cc * 8);
        }
    }
    __syncthreads();

    const int units = (int) (d.F / 32);
    for (int64_t it = i0; it < i1; ++it) {
        const uint32_t ph = (uint32_t) ((it - i0) & 1);
        bool ok = mbar_wait(&bar[0], ph);
        ok = __syncthreads_and(ok);
        if (!ok) {
            if (tid == 0) {
                report(d.st, QWB_DEVERR_TIMEOUT, (int32_t) it);
                mbar_wait(&bar[0], ph);
            }
            return;
        }
        const int64_t r0 = it * d.R;
        const int nr = (int) min((int64_t) d.R, d.H - r0);
        for (int r = warp; r < nr; r += 4) {
            float acc = 0.f;
            for (int j = 0; j < d.n_used; ++j) {
                if (s_slot[j] < 0) continue;
                const uint8_t *row = wbuf + j * d.wspan +
                                     ((uintptr_t) (d.W + (size_t) s_slot[j] * d.nb2 + (size_t) r0 * d.nb1) & 15) +
                                     (size_t) r * d.nb1;
                ActSmem A{act + j * d.act_stride, d.act_stride, d.act_d_off, d.act_b_off};
                float pj = 0.f;
                for (int u = lane; u < units; u += 32) unit_dot<TYPE, 1>(row, u, A, 1, &pj);
                acc = fmaf(s_w[j], pj, acc);
            }
            acc = warp_sum(acc);
            if (lane == 0) {
                const int64_t h = r0 + r;
                if (d.sh) acc = __fadd_rn(acc, d.sh_scale ? __fmul_rn(d.sh[h], d.sh_scale[0]) : d.sh[h]);
                d.out[h] = d.residual ? acc + d.residual[h] : acc;
            }
        }
        __syncthreads();
        if (tid == 0 && it + 1 < i1) {
            fence_proxy_async_smem();
            issue(it + 1);
        }
    }
}

template <int TYPE>
static cudaError_t launch_down_t(DownArgs d, cudaStream_t s) {
    auto kern = moe_down_decode_kernel<TYPE>;
    const size_t smem = 128 + (size_t) d.smem_act + (size_t) d.n_used * d.wspan;
    static DeviceSmemLimit limit;
    cudaError_t e = ensure_dyn_smem(kern, smem, limit);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 128, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int grid = std::max(1, std::min(d.n_rb, per_sm * num_sms()));
    kern<<<grid, 128, smem, s>>>(d);
    return cudaGetLastError();
}

static cudaError_t launch_down(int type, DownArgs d, cudaStream_t s) {
    const bool kq = type != QWB_TYPE_Q8_0;
    const int dstride = (int) plane_d_stride(d.F, kq ? QK_K : QK8_0);
    const int bstride = kq ? (int) plane_bsum_stride(d.F) : 0;
    d.kq = kq;
    d.act_d_off = (int) d.F;
    d.act_b_off = (int) (d.F + dstride * 4);
    d.act_stride = (int) align_up((size_t) (d.F + dstride * 4 + bstride * 2), 16);
    d.smem_act = (int) align_up((size_t) d.n_used * d.act_stride, 128);
    // rows per item: keep the n_used weight spans within ~96 KB
    int R = 32;
    while (R > 1 && (size_t) d.n_used * align_up((size_t) R * d.nb1 + 32, 16) + d.smem_act > 96 * 1024) R >>= 1;
    d.R = R;
    d.wspan = (int) align_up((size_t) R * d.nb1 + 32, 16);
    d.n_rb = (int) ceil_div(d.H, R);
    switch (type) {
        case QWB_TYPE_Q4_K: return launch_down_t<QWB_TYPE_Q4_K>(d, s);
        case QWB_TYPE_Q6_K: return launch_down_t<QWB_TYPE_Q6_K>(d, s);
        default: return launch_down_t<QWB_TYPE_Q8_0>(d, s);
    }
}

// ------------------------------------------------------------ shared expert
qwb_status shexp_check(const qwb_tensor &g, const qwb_tensor &u, const qwb_tensor &d, const float *gate_inp, int tg,
                       int td, int64_t H, Shexp &sh) {
    sh = Shexp{&g, &u, &d, gate_inp, 0};
    if (!d.data) return QWB_OK;
    if (!g.data || !u.data) return QWB_ERR_INVALID_ARG;
    if (g.type != tg || u.type != tg || d.type != td) return QWB_ERR_UNSUPPORTED_TYPE;
    const int64_t F = g.ne[1];
    if (F <= 0 || F % 256 || g.ne[0] != H || u.ne[0] != H || u.ne[1] != F || d.ne[0] != F || d.ne[1] != H)
        return QWB_ERR_SHAPE;
    for (const qwb_tensor *t : {&g, &u, &d}) {
        if (t->ne[2] != 1 || t->ne[3] != 1) return QWB_ERR_SHAPE;
        if (t->nb[0] != row_bytes(t->type, block_elems(t->type)) || t->nb[1] != row_bytes(t->type, t->ne[0]))
            return QWB_ERR_LAYOUT;
        if ((uintptr_t) t->data % 16) return QWB_ERR_ALIGNMENT;
    }
    if ((uintptr_t) gate_inp % 16) return QWB_ERR_ALIGNMENT;
    sh.F = F;
    return QWB_OK;
}

namespace {
struct ShexpPlan {
    bool stream;
    int NT;
    size_t off_ids, off_index, off_act, off_actq, off_out, total;
};
ShexpPlan shexp_plan(const Shexp &sh, int64_t H, int64_t T) {
    ShexpPlan q{};
    const int tg = sh.gate->type, td = sh.down->type;
    q.stream = stream_fits_ffn(tg, H, sh.gate->nb[1], sh.up->nb[1], td, sh.F, sh.down->nb[1]);
    q.NT = q.stream ? (int) std::max<int64_t>(1, T) : pick_nt(std::max<int64_t>(1, T), 1);
    size_t o = 0;
    q.off_ids = o; o += align_up((size_t) T * 4, 256);
    q.off_index = o; o += mmid_index_bytes(std::max<int64_t>(T, 1), 1, q.NT);
    q.off_act = o; o += align_up((size_t) T * sh.F * 4, 256);
    q.off_actq = o; o += planes_bytes(T, sh.F, td != QWB_TYPE_Q8_0);
    q.off_out = o; o += align_up((size_t) T * H * 4, 256);
    q.total = o;
    return q;
}
}  // namespace

size_t shexp_bytes(const Shexp &sh, int64_t H, int64_t T) { return sh.F ? shexp_plan(sh, H, T).total : 0; }
float *shexp_out_at(const Shexp &sh, int64_t H, int64_t T, void *ws) {
    return (float *) ((char *) ws + shexp_plan(sh, H, T).off_out);
}

cudaError_t shexp_run(const Shexp &sh, const Q8Planes &xq, const float *x, const float *norm_w, float eps, int64_t H,
                      int64_t T, void *ws, float *sh_out, float *sh_scale, qwb_status_block *st, cudaStream_t s) {
    const ShexpPlan q = shexp_plan(sh, H, T);
    char *w = (char *) ws;
    const int tg = sh.gate->type, td = sh.down->type;
    // every token selects the one shared expert
    int32_t *ids = (int32_t *) (w + q.off_ids);
    cudaError_t e = cudaMemsetAsync(ids, 0, (size_t) T * 4, s);
    MmidIndex ix = mmid_index_at(w + q.off_index, std::max<int64_t>(T, 1), 1, q.NT);
    if (e == cudaSuccess) e = launch_index(ids, 1, 1, 1, (int) T, 1, q.NT, ix, nullptr, 0, 0, 0, st, s);
    if (e != cudaSuccess) return e;
    float *act = (float *) (w + q.off_act);
    {
        GemvArgs a{};
        a.W = (const uint8_t *) sh.gate->data; a.nb1 = sh.gate->nb[1]; a.nb2 = sh.gate->nb[1] * (size_t) sh.F;
        a.W2 = (const uint8_t *) sh.up->data; a.nb1_2 = sh.up->nb[1]; a.nb2_2 = sh.up->nb[1] * (size_t) sh.F;
        a.row_bytes = row_bytes(tg, H);
        a.M = sh.F; a.K = H;
        a.act = xq;
        a.tiles = ix.tiles; a.n_tiles = ix.n_tiles; a.pairs = ix.pairs;
        a.n_used = 1; a.n_b = 1;
        a.dst = act; a.dnb1 = (size_t) sh.F * 4; a.dnb2 = (size_t) sh.F * 4;
        a.n_ids = 1; a.n_slots = 1;
        a.st = st;
        e = launch_expert_gemv(tg, true, a, q.stream, q.NT, ix.max_tiles, T, 1, ix.work, s);
        if (e != cudaSuccess) return e;
    }
    const bool kq_d = td != QWB_TYPE_Q8_0;
    Q8Planes aq = planes_at(w + q.off_actq, T, sh.F, kq_d);
    e = launch_quantize_rows(kq_d ? 0 : 1, act, sh.F, T, sh.F, nullptr, aq, nullptr, s);
    if (e != cudaSuccess) return e;
    {
        GemvArgs a{};
        a.W = (const uint8_t *) sh.down->data; a.nb1 = sh.down->nb[1]; a.nb2 = sh.down->nb[1] * (size_t) H;
        a.row_bytes = row_bytes(td, sh.F);
        a.M = H; a.K = sh.F;
        a.act = aq;
        a.tiles = ix.tiles; a.n_tiles = ix.n_tiles; a.pairs = ix.pairs;
        a.n_used = 1; a.n_b = 1;
        a.dst = sh_out; a.dnb1 = (size_t) H * 4; a.dnb2 = (size_t) H * 4;
        a.n_ids = 1; a.n_slots = 1;
        a.st = st;
        e = launch_expert_gemv(td, false, a, q.stream, q.NT, ix.max_tiles, T, 1, ix.work + 1, s);
        if (e != cudaSuccess) return e;
    }
    if (sh.gate_inp) e = launch_shexp_gate(x, norm_w, eps, sh.gate_inp, T, H, sh_scale, s);
    return e;
}

// ------------------------------------------------------------ workspace plan
struct FfnPlan {
    bool kq_gu, kq_d;
    int NT;
    bool stream;  // batched expert GEMVs on the streaming kernel (index: one tile per expert)
    bool pairs;   // decode batches / shared expert on the pair kernels (decode.cu)
    Shexp sh;
    int64_t P;
    size_t off_logits, off_sel, off_w, off_slots, off_xq, off_index, off_act, off_xn, off_actq, off_experts;
    size_t off_shs, off_sh, total;
};

static qwb_status plan_ffn(const qwb_moe_ffn_desc *d, FfnPlan &p) {
    if (!d) return QWB_ERR_INVALID_ARG;
    if (d->H <= 0 || d->F <= 0 || d->E <= 0 || d->n_used <= 0 || d->T < 0) return QWB_ERR_INVALID_ARG;
    const int tg = d->gate.type, tu = d->up.type, td = d->down.type;
    auto ok_t = [](int t) { return t == QWB_TYPE_Q4_K || t == QWB_TYPE_Q6_K || t == QWB_TYPE_Q8_0; };
    if (!ok_t(tg) || !ok_t(td) || tu != tg) return QWB_ERR_UNSUPPORTED_TYPE;
    if (d->n_used > kMaxUsed || d->E > kMaxExperts || d->n_used > d->E) return QWB_ERR_LIMIT;
    if (d->H % 1024 || d->F % 256) return QWB_ERR_SHAPE;
    const int64_t n_mat = d->gate.ne[2];
    if (d->gate.ne[0] != d->H || d->gate.ne[1] != d->F || d->up.ne[0] != d->H || d->up.ne[1] != d->F ||
        d->up.ne[2] != n_mat || d->down.ne[0] != d->F || d->down.ne[1] != d->H || d->down.ne[2] != n_mat)
        return QWB_ERR_SHAPE;
    if (!d->g2s && n_mat != d->E) return QWB_ERR_SHAPE;
    qwb_status rc = shexp_check(d->shexp_gate, d->shexp_up, d->shexp_down, d->shexp_gate_inp, tg, td, d->H, p.sh);
    if (rc != QWB_OK) return rc;
    p.kq_gu = tg != QWB_TYPE_Q8_0;
    p.kq_d = td != QWB_TYPE_Q8_0;
    p.P = d->n_used * d->T;
    // the pair kernels: batch-1 decode with a shared expert of the routed experts' size
    // (without one it keeps the kernels tuned for it) and decode batches of up to 16
    // (token, expert) pairs; they read an expert's rows once per pair, so larger batches
    // take the streaming kernels, which read each selected expert once for all its
    // tokens.  The act output is in pair order there, so not when act is requested.
    p.pairs = !d->act && ((d->T == 1 && p.sh.F) || (d->T > 1 && d->T * d->n_used <= kPairsDirect)) &&
              (!p.sh.F || p.sh.F == d->F) &&
              pairs_supported(tg, td, d->H, d->F, d->E, (int) d->n_used, (int) d->T, row_bytes(tg, d->H),
                              d->gate.nb[1], d->up.nb[1], row_bytes(td, d->F), d->down.nb[1]);
    // batched (T > 1): the streaming kernel when it fits, with one index tile per expert
    p.stream = d->T > 1 && stream_fits_ffn(tg, d->H, d->gate.nb[1], d->up.nb[1], td, d->F, d->down.nb[1]);
    p.NT = p.stream ? (int) std::max<int64_t>(1, p.P) : pick_nt(p.P, d->E);
    size_t o = kCtrlBytes;
    p.off_logits = o; o += align_up((size_t) (d->T * d->E) * 4, 256);
    p.off_sel = o; o += align_up((size_t) p.P * 4, 256);
    p.off_w = o; o += align_up((size_t) p.P * 4, 256);
    p.off_slots = o; o += align_up((size_t) 3 * p.P * 4, 256);
    p.off_xq = o; o += planes_bytes(d->T, d->H, p.kq_gu);
    p.off_index = o; o += mmid_index_bytes(std::max<int64_t>(p.P, 1), d->E, p.NT);
    p.off_act = o; o += align_up((size_t) (p.P + (p.pairs && p.sh.F ? d->T : 0)) * d->F * 4, 256);
    p.off_shs = o; o += align_up((size_t) d->T * 4, 256);
    p.off_sh = o;
    if (p.sh.F && !p.pairs) o += shexp_bytes(p.sh, d->H, d->T);
    p.off_xn = o;
    if (d->norm_w && d->T > kMaxRouterT) o += align_up((size_t) d->T * d->H * 4, 256);
    p.off_actq = o;
    p.off_experts = o;
    if (d->T > 1) {
        o += planes_bytes(p.P, d->F, p.kq_d);
        p.off_experts = o;
        o += align_up((size_t) p.P * d->H * 4, 256);
    }
    p.total = o;
    return QWB_OK;
}

}  // namespace qwb

using namespace qwb;

extern "C" QWB_API size_t qwb_moe_ffn_workspace_size(const qwb_moe_ffn_desc *desc) {
    FfnPlan p;
    if (plan_ffn(desc, p) != QWB_OK) return 0;
    return p.total;
}

extern "C" QWB_API qwb_status qwb_moe_ffn(const qwb_moe_ffn_desc *d, void *ws, size_t ws_bytes,
                                          qwb_status_block *st, qwb_stream_t stream) {
    FfnPlan p;
    qwb_status rc = plan_ffn(d, p);
    if (rc != QWB_OK) return rc;
    if (d->T == 0) return QWB_OK;
    if (!d->x || !d->router_w || !d->out || !d->gate.data || !d->up.data || !d->down.data) return QWB_ERR_INVALID_ARG;
    if (!ws || ws_bytes < p.total) return QWB_ERR_WORKSPACE;
    if ((uintptr_t) ws % 256) return QWB_ERR_ALIGNMENT;
    if (((uintptr_t) d->x | (uintptr_t) d->router_w | (uintptr_t) d->out | (uintptr_t) d->act |
         (uintptr_t) d->norm_w) % 16)
        return QWB_ERR_ALIGNMENT;
    for (const qwb_tensor *t : {&d->gate, &d->up, &d->down}) {
        if (t->nb[0] != row_bytes(t->type, block_elems(t->type))) return QWB_ERR_LAYOUT;
        if (t->nb[1] < row_bytes(t->type, t->ne[0]) || t->nb[2] < t->nb[1] * (size_t) t->ne[1]) return QWB_ERR_LAYOUT;
        const uintptr_t al = (uintptr_t) t->data | t->nb[1] | t->nb[2];
        if (t->type == QWB_TYPE_Q4_K ? al % 16 : al % 2) return QWB_ERR_ALIGNMENT;
    }
    cudaStream_t s = (cudaStream_t) stream;
    char *w = (char *) ws;
    const int64_t H = d->H, F = d->F, E = d->E, T = d->T, K = d->n_used;
    const int64_t n_mat = d->gate.ne[2];
    int32_t *sel = d->selected ? d->selected : (int32_t *) (w + p.off_sel);
    float *wts = d->weights ? d->weights : (float *) (w + p.off_w);
    float *logits = (float *) (w + p.off_logits);
    Q8Planes xq = planes_at(w + p.off_xq, T, H, p.kq_gu);
    MmidIndex ix = mmid_index_at(w + p.off_index, std::max<int64_t>(p.P, 1), E, p.NT);
    float *act = d->act ? d->act : (float *) (w + p.off_act);
    const int32_t *g2s_g = d->g2s, *g2s_u = d->g2s ? d->g2s + E : nullptr, *g2s_d = d->g2s ? d->g2s + 2 * E : nullptr;
    cudaError_t e;

    const bool decode = T == 1;
    profile_mark(s, 0);
    if (p.pairs) {
        PairsLayer L{};
        L.x = d->x; L.router_w = d->router_w; L.mask = d->mask; L.norm_w = d->norm_w; L.norm_eps = d->norm_eps;
        L.H = H; L.F = F; L.E = E; L.n_used = (int) K; L.T = (int) T;
        L.g2s = d->g2s;
        L.gate = &d->gate; L.up = &d->up; L.down = &d->down;
        if (p.sh.F) { L.sh_gate = &d->shexp_gate; L.sh_up = &d->shexp_up; L.sh_down = &d->shexp_down; }
        L.sh_gate_inp = d->shexp_gate_inp;
        L.residual = d->residual; L.out = d->out;
        L.sel = sel; L.wts = wts; L.slots = (int32_t *) (w + p.off_slots);
        L.sh_scale = (float *) (w + p.off_shs); L.act = act; L.xq = xq;
        L.st = st;
        return run_pairs_layer(L, s) == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
    }
    if (decode && !p.sh.F && E <= kMaxRouteE && E >= kRouterCluster && (E % kRouterCluster) == 0 && K <= 32 &&
        gateup_decode_supported(d->gate.type, H, row_bytes(d->gate.type, H), d->gate.nb[1], F, (int) K) &&
        d->up.nb[1] == d->gate.nb[1] &&
        down_decode_supported(d->down.type, F, H, row_bytes(d->down.type, F), d->down.nb[1], (int) K)) {
        // batch-1 decode: three PDL-chained kernels (decode.cu)
        int32_t *slots = (int32_t *) (w + p.off_slots);
        RouterDecodeArgs r{};
        r.x = d->x; r.router_w = d->router_w; r.mask = d->mask; r.norm_w = d->norm_w; r.norm_eps = d->norm_eps;
        r.H = H; r.E = E; r.n_used = (int) K; r.T = 1;
        r.g2s = d->g2s;
        r.n_slots[0] = d->gate.ne[2]; r.n_slots[1] = d->up.ne[2]; r.n_slots[2] = d->down.ne[2];
        r.sel = sel; r.wts = wts; r.slots = slots;
        r.xq = xq; r.kq = 1;
        r.st = st;
        e = launch_router_decode(r, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
        profile_mark(s, QWB_KERNEL_ROUTER);
        GateUpDecodeArgs g{};
        g.Wg = (const uint8_t *) d->gate.data; g.Wu = (const uint8_t *) d->up.data;
        g.g_nb2 = d->gate.nb[2]; g.u_nb2 = d->up.nb[2]; g.row_bytes = row_bytes(d->gate.type, H);
        g.F = F; g.K = H; g.n_slots_g = d->gate.ne[2]; g.n_slots_u = d->up.ne[2];
        g.n_used = (int) K; g.slots = slots; g.xq = xq; g.act = act; g.st = st;
        g.partner_smem = down_decode_smem_bytes(H, (int) K, row_bytes(d->down.type, F));
        e = launch_gateup_decode(g, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
        profile_mark(s, QWB_KERNEL_GATE_UP);
        DownDecodeArgs dn{};
        dn.W = (const uint8_t *) d->down.data; dn.nb2 = d->down.nb[2]; dn.row_bytes = row_bytes(d->down.type, F);
        dn.F = F; dn.H = H; dn.n_slots = d->down.ne[2]; dn.n_used = (int) K;
        dn.slots = slots + 2 * K; dn.wts = wts; dn.act = act; dn.out = d->out; dn.residual = d->residual; dn.st = st;
        e = launch_down_decode(d->down.type, dn, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
        profile_mark(s, QWB_KERNEL_DOWN);
        return QWB_OK;
    }
    if (T <= kMaxRouterT) {
        RouterArgs r{};
        r.x = d->x; r.router_w = d->router_w; r.mask = d->mask;
        r.H = H; r.E = E; r.T = T; r.n_used = K;
        r.logits = logits;
        r.counter = (unsigned *) w;
        r.selected = sel; r.weights = wts;
        r.xq = xq; r.kq = p.kq_gu;
        r.norm_w = d->norm_w; r.norm_eps = d->norm_eps;
        if (decode) { r.tiles = ix.tiles; r.pairs = ix.pairs; r.n_tiles = ix.n_tiles; }
        e = launch_router_fused(r, s);
    } else {
        const float *xin = d->x;
        if (d->norm_w) {
            float *xn = (float *) (w + p.off_xn);
            e = launch_rmsnorm(d->x, d->norm_w, d->norm_eps, T, H, xn, s);
            if (e != cudaSuccess) return QWB_ERR_CUDA;
            xin = xn;
        }
        e = launch_logits_gemm(xin, d->router_w, logits, T, E, H, s);
        if (e == cudaSuccess) e = launch_route(logits, d->mask, E, T, K, 1, 0.0f, sel, wts, s);
        if (e == cudaSuccess) e = launch_quantize_rows(p.kq_gu ? 0 : 1, xin, H, T, H, nullptr, xq, nullptr, s);
    }
    if (e != cudaSuccess) return QWB_ERR_CUDA;
    profile_mark(s, QWB_KERNEL_ROUTER);
    // the shared expert (its own GEMVs; the routed experts' reduction adds it)
    float *sh_out = nullptr, *sh_scale = nullptr;
    if (p.sh.F) {
        sh_out = shexp_out_at(p.sh, H, T, w + p.off_sh);
        sh_scale = d->shexp_gate_inp ? (float *) (w + p.off_shs) : nullptr;
        e = shexp_run(p.sh, xq, d->x, d->norm_w, d->norm_eps, H, T, w + p.off_sh, sh_out, sh_scale, st, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
    }
    if (!decode) {
        e = launch_index(sel, 1, K, (int) K, (int) T, (int) E, p.NT, ix, nullptr, 0, 0, 0, st, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
    }
    // gate + up + SwiGLU -> act [T][n_used][F]
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
        a.remap = g2s_g; a.remap2 = g2s_u; a.n_ids = E; a.n_slots = n_mat;
        a.st = st;
        const int NT = decode ? 1 : p.NT;
        e = launch_expert_gemv(d->gate.type, true, a, !decode && p.stream, NT, decode ? (int) K : ix.max_tiles, p.P,
                               E, ix.work, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
        profile_mark(s, QWB_KERNEL_GATE_UP);
    }
    if (decode) {
        DownArgs dn{};
        dn.W = (const uint8_t *) d->down.data; dn.nb1 = d->down.nb[1]; dn.nb2 = d->down.nb[2];
        dn.row_bytes = row_bytes(d->down.type, F);
        dn.n_slots = n_mat; dn.E = E;
        dn.remap = g2s_d; dn.selected = sel; dn.weights = wts; dn.n_used = (int) K;
        dn.act = act; dn.F = F; dn.H = H;
        dn.out = d->out; dn.residual = d->residual;
        dn.sh = sh_out; dn.sh_scale = sh_scale;
        dn.st = st;
        e = launch_down(d->down.type, dn, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
        profile_mark(s, QWB_KERNEL_DOWN);
        return QWB_OK;
    }
    // batched: act -> Q8, down GEMV per (slot, token), weighted sum
    Q8Planes aq = planes_at(w + p.off_actq, p.P, F, p.kq_d);
    e = launch_quantize_rows(p.kq_d ? 0 : 1, act, F, p.P, F, nullptr, aq, nullptr, s);
    if (e != cudaSuccess) return QWB_ERR_CUDA;
    float *experts = (float *) (w + p.off_experts);
    {
        GemvArgs a{};
        a.W = (const uint8_t *) d->down.data; a.nb1 = d->down.nb[1]; a.nb2 = d->down.nb[2];
        a.row_bytes = row_bytes(d->down.type, F);
        a.M = H; a.K = F;
        a.act = aq;
        a.tiles = ix.tiles; a.n_tiles = ix.n_tiles; a.pairs = ix.pairs;
        a.n_used = (int) K; a.n_b = (int) K;
        a.dst = experts; a.dnb1 = (size_t) H * 4; a.dnb2 = (size_t) K * H * 4;
        a.remap = g2s_d; a.n_ids = E; a.n_slots = n_mat;
        a.st = st;
        e = launch_expert_gemv(d->down.type, false, a, p.stream, p.NT, ix.max_tiles, p.P, E, ix.work + 1, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
        profile_mark(s, QWB_KERNEL_DOWN);
    }
    e = launch_weighted_sum(experts, wts, d->residual, d->out, H, K, T, s, sh_out, sh_scale);
    if (e != cudaSuccess) return QWB_ERR_CUDA;
    profile_mark(s, QWB_KERNEL_OTHER);
    return QWB_OK;
}
