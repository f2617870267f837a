// ep.cu - the expert-parallel MoE layer: one GPU's share of build_moe
// (core/runtime.cpp:2743-2816) when the experts of every layer are split over N GPUs.
//
// Every GPU holds the hidden states of all T tokens (identical copies) and routes all of
// them (the router is replicated); it then runs the SwiGLU expert FFN of the experts it
// owns over the (token, slot) pairs routed to them and writes the weighted sum of those
// experts' outputs per token (zero for a token with none of its experts here), plus the
// residual on the one GPU the caller passes it to.  The caller sums the N partial
// outputs with one all-reduce, which leaves every GPU with the layer's output for all
// tokens: the next layer's input, again identical everywhere.  One collective per layer.
//
// The arithmetic per (token, slot) is the reference CPU backend's, as in qwb_moe_ffn:
// activations quantized to the weights' vec_dot type (bit-exact, per row), integer
// sub-block dots, f32 combine.  Splitting the expert sum over GPUs changes only the f32
// summation order of the weighted expert outputs.
#include <algorithm>

#include "common.cuh"
#include "decode.cuh"
#include "kernels.cuh"
#include "mmid.cuh"
#include "moe.cuh"
#include "route.cuh"

namespace qwb {

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
//          (+ sh[t] * sh_scale[t], the shared expert) (+ residual[t])
__global__ void weighted_sum_local_kernel(const float *__restrict__ ex, const float *__restrict__ w,
                                          const int32_t *__restrict__ lid, const float *__restrict__ sh,
                                          const float *__restrict__ sh_scale, const float *__restrict__ residual,
                                          float *__restrict__ out, int64_t H, int n_used, int64_t T) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= H * T) return;
    const int64_t t = i / H, h = i - t * H;
    float acc = 0.f;
    for (int j = 0; j < n_used; ++j)
        if (lid[t * n_used + j] >= 0) acc = fmaf(w[t * n_used + j], ex[(t * n_used + j) * H + h], acc);
    if (sh) acc = __fadd_rn(acc, sh_scale ? __fmul_rn(sh[i], sh_scale[t]) : sh[i]);
    out[i] = residual ? acc + residual[i] : acc;
}

}  // namespace qwb

using namespace qwb;

namespace {

bool ok_weight_type(int t) { return t == QWB_TYPE_Q4_K || t == QWB_TYPE_Q6_K || t == QWB_TYPE_Q8_0; }

struct EpPlan {
    bool kq_gu, kq_d;
    int NT;
    bool stream;  // expert GEMVs on the streaming kernel (index: one tile per expert)
    bool pairs;   // decode batches of <= 8 tokens on the pair kernels (decode.cu)
    Shexp sh;
    int64_t P, n_local;
    size_t off_logits, off_sel, off_w, off_xn, off_xq, off_lid, off_index, off_act, off_actq, off_ex;
    size_t off_slots, off_shs, off_sh, total;
};
qwb_status plan_ep(const qwb_moe_ep_layer_desc *d, EpPlan &p) {
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
    qwb_status rc = shexp_check(d->shexp_gate, d->shexp_up, d->shexp_down, d->shexp_gate_inp, tg, td, d->H, p.sh);
    if (rc != QWB_OK) return rc;
    p.kq_gu = tg != QWB_TYPE_Q8_0;
    p.kq_d = td != QWB_TYPE_Q8_0;
    p.P = d->n_used * d->T;
    // the pair kernels when few pairs are expected here (they read an expert's rows once
    // per pair; the streaming kernels read each selected expert once for all its tokens)
    p.pairs = d->T * d->n_used * p.n_local <= (int64_t) kPairsDirect * d->E && (!p.sh.F || p.sh.F == d->F) &&
              pairs_supported(tg, td, d->H, d->F, d->E, (int) d->n_used, (int) d->T, row_bytes(tg, d->H),
                              d->gate.nb[1], d->up.nb[1], row_bytes(td, d->F), d->down.nb[1]);
    p.stream = stream_fits_ffn(tg, d->H, d->gate.nb[1], d->up.nb[1], td, d->F, d->down.nb[1]);
    p.NT = p.stream ? (int) std::max<int64_t>(1, p.P) : pick_nt(std::max<int64_t>(1, p.P * p.n_local / d->E), p.n_local);
    size_t o = kCtrlBytes;
    p.off_logits = o; o += align_up((size_t) (d->T * d->E) * 4, 256);
    p.off_sel = o; o += align_up((size_t) p.P * 4, 256);
    p.off_w = o; o += align_up((size_t) p.P * 4, 256);
    p.off_xn = o;
    if (d->norm_w && d->T > kMaxRouterT) o += align_up((size_t) (d->T * d->H) * 4, 256);
    p.off_xq = o; o += planes_bytes(d->T, d->H, p.kq_gu);
    p.off_lid = o; o += align_up((size_t) p.P * 4, 256);
    p.off_index = o; o += mmid_index_bytes(std::max<int64_t>(p.P, 1), p.n_local, p.NT);
    p.off_act = o; o += align_up((size_t) (p.P + d->T) * d->F * 4, 256);
    p.off_actq = o; o += planes_bytes(p.P, d->F, p.kq_d);
    p.off_ex = o; o += align_up((size_t) p.P * d->H * 4, 256);
    p.off_slots = o; o += align_up((size_t) 3 * p.P * 4, 256);
    p.off_shs = o; o += align_up((size_t) d->T * 4, 256);
    p.off_sh = o; o += shexp_bytes(p.sh, d->H, d->T);
    p.total = o;
    return QWB_OK;
}

}  // namespace

extern "C" QWB_API size_t qwb_moe_ep_layer_workspace_size(const qwb_moe_ep_layer_desc *desc) {
    EpPlan p;
    return plan_ep(desc, p) == QWB_OK ? p.total : 0;
}

extern "C" QWB_API qwb_status qwb_moe_ep_layer(const qwb_moe_ep_layer_desc *d, void *ws, size_t ws_bytes,
                                               qwb_status_block *st, qwb_stream_t stream) {
    EpPlan p;
    qwb_status rc = plan_ep(d, p);
    if (rc != QWB_OK) return rc;
    if (d->T == 0) return QWB_OK;
    if (!d->x || !d->router_w || !d->out || !d->gate.data || !d->up.data || !d->down.data) return QWB_ERR_INVALID_ARG;
    if (!ws || ws_bytes < p.total) return QWB_ERR_WORKSPACE;
    if ((uintptr_t) ws % 256) return QWB_ERR_ALIGNMENT;
    if (((uintptr_t) d->x | (uintptr_t) d->router_w | (uintptr_t) d->norm_w | (uintptr_t) d->out |
         (uintptr_t) d->residual) % 16)
        return QWB_ERR_ALIGNMENT;
    for (const qwb_tensor *t : {&d->gate, &d->up, &d->down}) {
        if (t->nb[0] != row_bytes(t->type, block_elems(t->type))) return QWB_ERR_LAYOUT;
        if (t->nb[1] < row_bytes(t->type, t->ne[0]) || t->nb[2] < t->nb[1] * (size_t) t->ne[1]) return QWB_ERR_LAYOUT;
        const uintptr_t al = (uintptr_t) t->data | t->nb[1] | t->nb[2];
        if (t->type == QWB_TYPE_Q4_K ? al % 16 : al % 2) return QWB_ERR_ALIGNMENT;
    }
    cudaStream_t s = (cudaStream_t) stream;
    char *w = (char *) ws;
    const int64_t H = d->H, F = d->F, E = d->E, T = d->T, K = d->n_used, P = p.P, NL = p.n_local;
    int32_t *sel = d->selected ? d->selected : (int32_t *) (w + p.off_sel);
    float *wts = d->weights ? d->weights : (float *) (w + p.off_w);
    Q8Planes xq = planes_at(w + p.off_xq, T, H, p.kq_gu);
    int32_t *lid = (int32_t *) (w + p.off_lid);
    MmidIndex ix = mmid_index_at(w + p.off_index, std::max<int64_t>(P, 1), NL, p.NT);
    float *act = (float *) (w + p.off_act);
    float *ex = (float *) (w + p.off_ex);
    cudaError_t e;
    profile_mark(s, 0);
    if (p.pairs) {
        // decode batches: router clusters, gate/up and down over the pairs routed to this
        // GPU's experts (and the shared expert), PDL-chained
        PairsLayer L{};
        L.x = d->x; L.router_w = d->router_w; L.mask = d->mask; L.norm_w = d->norm_w; L.norm_eps = d->norm_eps;
        L.H = H; L.F = F; L.E = E; L.n_used = (int) K; L.T = (int) T;
        L.own_lo = d->expert_lo; L.own_n = NL;
        L.gate = &d->gate; L.up = &d->up; L.down = &d->down;
        if (p.sh.F) { L.sh_gate = &d->shexp_gate; L.sh_up = &d->shexp_up; L.sh_down = &d->shexp_down; }
        L.sh_gate_inp = d->shexp_gate_inp;
        L.residual = d->residual; L.out = d->out;
        L.sel = sel; L.wts = wts; L.slots = (int32_t *) (w + p.off_slots);
        L.sh_scale = (float *) (w + p.off_shs); L.act = act; L.xq = xq;
        L.st = st;
        return run_pairs_layer(L, s) == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
    }
    // routing of all T tokens (the same on every GPU) and their quantized rows
    if (T <= kMaxRouterT) {
        RouterArgs r{};
        r.x = d->x; r.router_w = d->router_w; r.mask = d->mask;
        r.H = H; r.E = E; r.T = T; r.n_used = K;
        r.logits = (float *) (w + p.off_logits);
        r.counter = (unsigned *) w;
        r.selected = sel; r.weights = wts;
        r.xq = xq; r.kq = p.kq_gu;
        r.norm_w = d->norm_w; r.norm_eps = d->norm_eps;
        e = launch_router_fused(r, s);
    } else {
        const float *xin = d->x;
        e = cudaSuccess;
        if (d->norm_w) {
            float *xn = (float *) (w + p.off_xn);
            e = launch_rmsnorm(d->x, d->norm_w, d->norm_eps, T, H, xn, s);
            xin = xn;
        }
        float *logits = (float *) (w + p.off_logits);
        if (e == cudaSuccess) e = launch_logits_gemm(xin, d->router_w, logits, T, E, H, s);
        if (e == cudaSuccess) e = launch_route(logits, d->mask, E, T, K, 1, 0.0f, sel, wts, s);
        if (e == cudaSuccess) e = launch_quantize_rows(p.kq_gu ? 0 : 1, xin, H, T, H, nullptr, xq, nullptr, s);
    }
    if (e != cudaSuccess) return QWB_ERR_CUDA;
    float *sh_out = nullptr, *sh_scale = nullptr;
    if (p.sh.F) {
        sh_out = shexp_out_at(p.sh, H, T, w + p.off_sh);
        sh_scale = d->shexp_gate_inp ? (float *) (w + p.off_shs) : nullptr;
        e = shexp_run(p.sh, xq, d->x, d->norm_w, d->norm_eps, H, T, w + p.off_sh, sh_out, sh_scale, st, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
    }
    // the pairs routed to this GPU's experts
    local_ids_kernel<<<(unsigned) ceil_div(P, 256), 256, 0, s>>>(sel, P, d->expert_lo, NL, E, lid, st);
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
    weighted_sum_local_kernel<<<(unsigned) ceil_div(H * T, 256), 256, 0, s>>>(ex, wts, lid, sh_out, sh_scale,
                                                                             d->residual, d->out, H, (int) K, T);
    e = cudaGetLastError();
    profile_mark(s, QWB_KERNEL_OTHER);
    return e == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
}
