// ggml-qwb.cpp - a ggml backend (interface version 3) for B200 that runs QuestWend's MoE
// hot path through libqwb.so.
//
// Two modes, chosen once when the registry is created:
//
//  * Delegating (the drop-in).  When the stock ggml-cuda backend library can be loaded
//    ($QWB_GGML_CUDA, else libggml-cuda.so beside this library), every QWB device wraps
//    one of its devices.  Tensors live in ggml-cuda's own buffer type (so the expert
//    cache's pool tensors and set_tensor_async work unchanged), the backend accepts
//    every op, and graph_compute runs
//      - each build_moe subgraph (core/runtime.cpp:2743-2816: router mul_mat, soft_max,
//        argsort top-k, weight normalisation, 3x MUL_MAT_ID, swiglu, weighted sum; the
//        resident branch and the in-graph slot-remap branch) as ONE qwb_moe_ffn call,
//      - other quantized MUL_MAT_ID and GET_ROWS nodes on libqwb.so kernels,
//      - every remaining node on the wrapped ggml-cuda backend, in runs of consecutive
//        nodes (sub-graphs), on its stream.
//    libqwb.so kernels run on this backend's own stream; CUDA events order the two
//    streams at every hand-over, and each graph_compute ends with the work joined back
//    into ggml-cuda's stream, so synchronize, events and async copies are ggml-cuda's.
//    QuestWend takes the first GPU device that initialises (runtime.cpp:996-1010) and
//    runs whole graphs with ggml_backend_graph_compute (runtime.cpp:6177-6178):
//    installed as libggml-cuda-<name>.so beside the stock libggml-cuda.so, this library
//    is the "cuda" backend ggml_backend_load_all() picks (highest ggml_backend_score).
//
//  * Standalone, when no ggml-cuda library is found: own cudaMalloc'd buffers; it
//    computes MUL_MAT_ID / quantized MUL_MAT / GET_ROWS and reports every other op
//    unsupported, so ggml's scheduler places those on another backend.
//
// The vtables are the ones of ggml-backend-impl.h (buffer type / buffer :17-85, backend
// :122-164, device :177-225, registry :231-247).  Loading is ggml's dynamic-backend path
// (ggml_backend_load -> ggml_backend_init / ggml_backend_score, ggml-backend-reg.cpp).
//
// graph_compute never allocates: scratch is reserved when the backend is created
// (params "workspace_mb=N", default 256), or grown by graph_optimize (which ggml's
// scheduler calls before computing) and by ggml_backend_qwb_reserve (get_proc_address);
// a graph needing more fails with GGML_STATUS_ALLOC_FAILED.  Expert or row ids out of
// range never fault the device: the affected outputs are zeroed and synchronize reports
// them from the status block (the reference CPU backend aborts on such ids instead).
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "ggml-backend-impl.h"
#include "ggml-impl.h"
#include "ggml.h"
#include "qwb.h"
#include "qwb_ggml_backend.h"

#define QWB_SHIM_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr size_t kAlign = 256;
constexpr size_t kDefaultWorkspaceMb = 256;

bool cuda_ok(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    std::fprintf(stderr, "ggml-qwb: %s: %s\n", what, cudaGetErrorString(e));
    return false;
}

qwb_tensor view_of(const ggml_tensor *t) {
    qwb_tensor q{};
    q.data = t->data;
    q.type = (int32_t) t->type;
    for (int i = 0; i < 4; ++i) {
        q.ne[i] = t->ne[i];
        q.nb[i] = t->nb[i];
    }
    return q;
}

bool weight_type(ggml_type t) { return t == GGML_TYPE_Q4_K || t == GGML_TYPE_Q6_K || t == GGML_TYPE_Q8_0; }
bool view_op(ggml_op op) {
    return op == GGML_OP_NONE || op == GGML_OP_RESHAPE || op == GGML_OP_VIEW || op == GGML_OP_PERMUTE ||
           op == GGML_OP_TRANSPOSE;
}

// ops libqwb.so computes one node at a time (mul_mat: quantized weights)
bool supported_mmid(const ggml_tensor *op) {
    const ggml_tensor *a = op->src[0], *b = op->src[1], *ids = op->src[2];
    if (!weight_type(a->type) || b->type != GGML_TYPE_F32 || ids->type != GGML_TYPE_I32 || op->type != GGML_TYPE_F32)
        return false;
    // b rows and dst rows contiguous, weight rows packed blocks
    if (b->nb[0] != sizeof(float) || op->nb[0] != sizeof(float)) return false;
    if (a->nb[0] != ggml_type_size(a->type)) return false;
    qwb_tensor qa = view_of(a), qb = view_of(b), qi = view_of(ids);
    return qwb_mul_mat_id_workspace_size(&qa, &qb, &qi) > 0;
}
bool supported_mul_mat(const ggml_tensor *op) {
    const ggml_tensor *a = op->src[0], *b = op->src[1];
    if (!weight_type(a->type) || b->type != GGML_TYPE_F32 || op->type != GGML_TYPE_F32) return false;
    if (b->nb[0] != sizeof(float) || op->nb[0] != sizeof(float) || a->nb[0] != ggml_type_size(a->type)) return false;
    qwb_tensor qa = view_of(a), qb = view_of(b);
    return qwb_mul_mat_workspace_size(&qa, &qb) > 0;
}
bool supported_get_rows(const ggml_tensor *op, bool any_type) {
    const ggml_tensor *s = op->src[0], *i = op->src[1];
    const bool rows = weight_type(s->type) ||
                      (any_type && (s->type == GGML_TYPE_F16 || s->type == GGML_TYPE_F32 || s->type == GGML_TYPE_I32));
    const ggml_type out = s->type == GGML_TYPE_I32 ? GGML_TYPE_I32 : GGML_TYPE_F32;
    return rows && i->type == GGML_TYPE_I32 && op->type == out && op->nb[0] == ggml_type_size(out) &&
           s->nb[0] == ggml_type_size(s->type) && i->ne[3] == 1;
}
bool supported_standalone(const ggml_tensor *op) {
    if (view_op(op->op)) return true;
    switch (op->op) {
        case GGML_OP_MUL_MAT_ID: return supported_mmid(op);
        case GGML_OP_MUL_MAT: return supported_mul_mat(op);
        case GGML_OP_GET_ROWS: return supported_get_rows(op, true);
        default: return false;
    }
}

// Workspace and status block shared by both modes' backends.
struct Scratch {
    int device = 0;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    qwb_status_block *status = nullptr;

    bool init(int dev, size_t mb) {
        device = dev;
        if (!cuda_ok(cudaMalloc((void **) &status, sizeof(qwb_status_block)), "cudaMalloc(status)")) return false;
        if (!cuda_ok(cudaMemset(status, 0, sizeof(qwb_status_block)), "cudaMemset(status)")) return false;
        return mb == 0 || grow(mb << 20);
    }
    // outside graph_compute only (backend creation, graph_optimize, the reserve proc)
    bool grow(size_t need) {
        if (need <= ws_bytes) return true;
        cudaSetDevice(device);
        if (ws) {
            cudaDeviceSynchronize();
            cudaFree(ws);
        }
        ws = nullptr;
        ws_bytes = 0;
        if (!cuda_ok(cudaMalloc(&ws, need), "cudaMalloc(workspace)")) return false;
        // the fused layer keeps a control block at the start of its workspace, zero
        // between calls (its kernels leave it zeroed)
        if (!cuda_ok(cudaMemset(ws, 0, need), "cudaMemset(workspace)")) return false;
        ws_bytes = need;
        return true;
    }
    void release() {
        cudaSetDevice(device);
        if (ws) cudaFree(ws);
        if (status) cudaFree(status);
        ws = nullptr;
        status = nullptr;
    }
    // a graph needing more than was reserved fails instead of allocating mid-compute
    bool fits(size_t need, const ggml_tensor *t) const {
        if (need <= ws_bytes) return true;
        std::fprintf(stderr,
                     "ggml-qwb: %s (%s) needs %zu workspace bytes, %zu are reserved: raise workspace_mb or "
                     "reserve with the graph first\n",
                     ggml_op_name(t->op), t->name, need, ws_bytes);
        return false;
    }
    void report(cudaStream_t s) {
        qwb_status_block h{};
        if (qwb_status_block_read(status, &h, 1, (qwb_stream_t) s) != QWB_OK) {
            std::fprintf(stderr, "ggml-qwb: status read failed: %s\n", cudaGetErrorString(cudaGetLastError()));
            return;
        }
        if (h.flags)
            std::fprintf(stderr, "ggml-qwb: %u out-of-range %s (first: %d); affected outputs were zeroed\n", h.count,
                         (h.flags & QWB_DEVERR_ID_RANGE) ? "expert ids" : "row ids", h.bad_value);
    }
};

// One node computed by libqwb.so on stream s.
qwb_status run_node(const ggml_tensor *t, Scratch &sc, cudaStream_t s, bool *ws_short) {
    *ws_short = false;
    switch (t->op) {
        case GGML_OP_MUL_MAT_ID: {
            qwb_tensor a = view_of(t->src[0]), b = view_of(t->src[1]), ids = view_of(t->src[2]), d = view_of(t);
            if (!sc.fits(qwb_mul_mat_id_workspace_size(&a, &b, &ids), t)) {
                *ws_short = true;
                return QWB_ERR_WORKSPACE;
            }
            return qwb_mul_mat_id(&a, &b, &ids, &d, sc.ws, sc.ws_bytes, sc.status, (qwb_stream_t) s);
        }
        case GGML_OP_MUL_MAT: {
            qwb_tensor a = view_of(t->src[0]), b = view_of(t->src[1]), d = view_of(t);
            if (!sc.fits(qwb_mul_mat_workspace_size(&a, &b), t)) {
                *ws_short = true;
                return QWB_ERR_WORKSPACE;
            }
            return qwb_mul_mat(&a, &b, &d, sc.ws, sc.ws_bytes, sc.status, (qwb_stream_t) s);
        }
        case GGML_OP_GET_ROWS: {
            qwb_tensor src = view_of(t->src[0]), i = view_of(t->src[1]), d = view_of(t);
            return qwb_get_rows(&src, &i, &d, sc.status, (qwb_stream_t) s);
        }
        default:
            return QWB_ERR_UNSUPPORTED_TYPE;
    }
}

size_t node_workspace(const ggml_tensor *t) {
    if (t->op == GGML_OP_MUL_MAT_ID && supported_mmid(t)) {
        qwb_tensor a = view_of(t->src[0]), b = view_of(t->src[1]), ids = view_of(t->src[2]);
        return qwb_mul_mat_id_workspace_size(&a, &b, &ids);
    }
    if (t->op == GGML_OP_MUL_MAT && supported_mul_mat(t)) {
        qwb_tensor a = view_of(t->src[0]), b = view_of(t->src[1]);
        return qwb_mul_mat_workspace_size(&a, &b);
    }
    return 0;
}

// ==================================================================== build_moe fusion
//
// Recognises the nodes build_moe emits for one layer (core/runtime.cpp:2743-2816, with
// route_experts :2693-2734 for softmax gating, expert_weights_norm, no scale, no bias,
// no mask) and describes them as one qwb_moe_ffn call.  Anything else - sigmoid gating,
// a probability bias, a weight scale, an intermediate that is read outside the layer or
// marked as a graph output - leaves the nodes to the per-node path.

struct Uses {
    std::unordered_map<const ggml_tensor *, std::vector<ggml_tensor *>> consumers;
    std::unordered_map<const ggml_tensor *, int> index;
    void build(ggml_cgraph *g) {
        consumers.clear();
        index.clear();
        for (int i = 0; i < g->n_nodes; ++i) {
            ggml_tensor *n = g->nodes[i];
            index[n] = i;
            for (int s = 0; s < GGML_MAX_SRC; ++s)
                if (n->src[s]) consumers[n->src[s]].push_back(n);
        }
    }
    const std::vector<ggml_tensor *> &of(const ggml_tensor *t) const {
        static const std::vector<ggml_tensor *> none;
        auto it = consumers.find(t);
        return it == consumers.end() ? none : it->second;
    }
    ggml_tensor *only(const ggml_tensor *t) const {
        const auto &c = of(t);
        return c.size() == 1 ? c[0] : nullptr;
    }
};

struct MoeRegion {
    ggml_tensor *x = nullptr, *router_w = nullptr, *wg = nullptr, *wu = nullptr, *wd = nullptr;
    ggml_tensor *out = nullptr;       // moe_out, or the residual add when that is absorbed
    ggml_tensor *sel = nullptr;       // [n_used, T] i32 view of the argsort
    ggml_tensor *weights = nullptr;   // [1, n_used, T] normalised routing weights
    ggml_tensor *norm_w = nullptr;    // ffn_norm weight when rms_norm * ffn_norm is absorbed (x: its input)
    ggml_tensor *residual = nullptr;  // the residual add's other operand when the add is absorbed
    ggml_tensor *sh_g = nullptr, *sh_u = nullptr, *sh_d = nullptr;  // shared expert when absorbed
    ggml_tensor *sh_gate_inp = nullptr;                               // its sigmoid gate weight, or none
    float norm_eps = 0.f;
    const int32_t *g2s = nullptr;     // gate, up, down tables, consecutive (slot-remap branch)
    int64_t H = 0, F = 0, E = 0, n_used = 0, T = 0;
    std::vector<ggml_tensor *> nodes;
    int first = 0;        // node index where the fused call runs (the layer's first node)
    bool direct = false;  // the layer's nodes are consecutive: results written in place
    bool sel_out = false, weights_out = false;  // read after the layer: materialise
};

bool is_op(const ggml_tensor *t, ggml_op op) { return t && t->op == op; }
bool f32_contig(const ggml_tensor *t) { return t && t->type == GGML_TYPE_F32 && ggml_is_contiguous(t); }

bool match_moe(const Uses &u, ggml_tensor *D, MoeRegion &r) {
    r = MoeRegion();
    std::vector<ggml_tensor *> &N = r.nodes;
    if (!is_op(D, GGML_OP_MUL_MAT_ID)) return false;
    ggml_tensor *act = D->src[1];
    if (!is_op(act, GGML_OP_GLU) || ggml_get_op_params_i32(act, 0) != GGML_GLU_OP_SWIGLU ||
        ggml_get_op_params_i32(act, 1) != 0 || !act->src[1])
        return false;
    ggml_tensor *G = act->src[0], *U = act->src[1];
    if (!is_op(G, GGML_OP_MUL_MAT_ID) || !is_op(U, GGML_OP_MUL_MAT_ID) || G->src[1] != U->src[1]) return false;
    r.wg = G->src[0];
    r.wu = U->src[0];
    r.wd = D->src[0];
    if (!weight_type(r.wg->type) || r.wu->type != r.wg->type || !weight_type(r.wd->type)) return false;
    if (u.of(G).size() != 1 || u.of(U).size() != 1 || u.of(act).size() != 1) return false;
    N.insert(N.end(), {G, U, act, D});

    // selection: the argsort's top-k view, either used directly (resident experts) or
    // through one I32 [1, E] expert -> slot table per role (the expert-cache branch)
    ggml_tensor *sel = nullptr;
    if (G->src[2] == U->src[2] && U->src[2] == D->src[2]) {
        sel = G->src[2];
    } else {
        ggml_tensor *tab[3];
        ggml_tensor *ids[3] = {G->src[2], U->src[2], D->src[2]};
        for (int k = 0; k < 3; ++k) {
            ggml_tensor *rs = ids[k];
            if (!is_op(rs, GGML_OP_RESHAPE) || !is_op(rs->src[0], GGML_OP_GET_ROWS)) return false;
            ggml_tensor *gr = rs->src[0];
            if (gr->src[0]->type != GGML_TYPE_I32 || gr->src[0]->ne[0] != 1 || gr->src[0]->nb[1] != 4) return false;
            if (sel && gr->src[1] != sel) return false;
            sel = gr->src[1];
            tab[k] = gr->src[0];
            if (u.of(gr).size() != 1 || u.of(rs).size() != 1) return false;
            N.insert(N.end(), {gr, rs});
            if (view_op(tab[k]->op)) N.push_back(tab[k]);
        }
        const int64_t E = tab[0]->ne[1];
        if ((char *) tab[1]->data != (char *) tab[0]->data + E * 4 ||
            (char *) tab[2]->data != (char *) tab[0]->data + 2 * E * 4)
            return false;
        r.g2s = (const int32_t *) tab[0]->data;
    }
    if (!is_op(sel, GGML_OP_VIEW) || !is_op(sel->src[0], GGML_OP_ARGSORT)) return false;
    ggml_tensor *A = sel->src[0];
    if (ggml_get_op_params_i32(A, 0) != GGML_SORT_ORDER_DESC || sel->view_offs != 0 || sel->nb[1] != A->nb[1])
        return false;
    r.sel = sel;
    r.n_used = sel->ne[0];
    N.insert(N.end(), {sel, A});
    ggml_tensor *probs = A->src[0];
    if (!is_op(probs, GGML_OP_SOFT_MAX) || probs->src[1] || probs->src[2]) return false;
    float sm_scale = 0.f, max_bias = 1.f;
    memcpy(&sm_scale, (const float *) probs->op_params + 0, sizeof(float));
    memcpy(&max_bias, (const float *) probs->op_params + 1, sizeof(float));
    if (sm_scale != 1.0f || max_bias != 0.0f) return false;
    ggml_tensor *logits = probs->src[0];
    if (!is_op(logits, GGML_OP_MUL_MAT) || u.of(logits).size() != 1) return false;
    r.router_w = logits->src[0];
    r.x = logits->src[1];
    if (!f32_contig(r.router_w) || !f32_contig(r.x) || r.x->ne[2] != 1 || r.x->ne[3] != 1) return false;
    r.H = r.x->ne[0];
    r.T = r.x->ne[1];
    r.E = r.router_w->ne[1];
    if (r.router_w->ne[0] != r.H || A->ne[0] != r.E || A->ne[1] != r.T) return false;
    N.insert(N.end(), {probs, logits});
    // the experts' input is x itself or a [H, 1, T] reshape of it
    ggml_tensor *x3 = G->src[1];
    if (x3 != r.x) {
        if (!is_op(x3, GGML_OP_RESHAPE) || x3->src[0] != r.x) return false;
        N.push_back(x3);
    }
    if (r.wg->ne[0] != r.H || r.wd->ne[1] != r.H || r.wd->ne[0] != r.wg->ne[1]) return false;
    r.F = r.wg->ne[1];

    // weights: reshape(div(reshape(get_rows(reshape(probs), sel)), clamp(sum_rows(...))))
    ggml_tensor *P3 = nullptr, *GR = nullptr;
    for (ggml_tensor *c : u.of(probs)) {
        if (c == A) continue;
        if (!is_op(c, GGML_OP_RESHAPE) || P3) return false;
        P3 = c;
    }
    if (!P3 || !(GR = u.only(P3)) || !is_op(GR, GGML_OP_GET_ROWS) || GR->src[1] != sel) return false;
    ggml_tensor *W2 = u.only(GR);
    if (!is_op(W2, GGML_OP_RESHAPE)) return false;
    ggml_tensor *SR = nullptr, *DV = nullptr;
    for (ggml_tensor *c : u.of(W2)) {
        if (is_op(c, GGML_OP_SUM_ROWS)) SR = c;
        else if (is_op(c, GGML_OP_DIV)) DV = c;
        else return false;
    }
    if (!SR || !DV || u.of(W2).size() != 2) return false;
    ggml_tensor *CL = u.only(SR);
    if (!is_op(CL, GGML_OP_CLAMP) || DV->src[0] != W2 || DV->src[1] != CL || u.only(CL) != DV) return false;
    float cmin = 0.f, cmax = 0.f;
    memcpy(&cmin, (const float *) CL->op_params + 0, sizeof(float));
    memcpy(&cmax, (const float *) CL->op_params + 1, sizeof(float));
    if (cmin != 6.103515625e-5f || !std::isinf(cmax)) return false;
    ggml_tensor *Wn = u.only(DV);
    if (!Wn) {
        // DV may have other readers besides the reshape: not this layer's shape
        return false;
    }
    if (!is_op(Wn, GGML_OP_RESHAPE)) return false;
    r.weights = Wn;
    N.insert(N.end(), {P3, GR, W2, SR, CL, DV, Wn});

    // weighted sum of the experts
    if (r.T == 1) {
        // moe_out = mul_mat(cont(transpose(reshape_2d(experts))), reshape_2d(weights))
        ggml_tensor *R1 = u.only(D), *TR = R1 ? u.only(R1) : nullptr, *CT = TR ? u.only(TR) : nullptr;
        ggml_tensor *MM = CT ? u.only(CT) : nullptr;
        if (!is_op(R1, GGML_OP_RESHAPE) || !is_op(TR, GGML_OP_TRANSPOSE) || !is_op(CT, GGML_OP_CONT) ||
            !is_op(MM, GGML_OP_MUL_MAT) || MM->src[0] != CT)
            return false;
        ggml_tensor *WR = MM->src[1];
        if (!is_op(WR, GGML_OP_RESHAPE) || WR->src[0] != Wn) return false;
        N.insert(N.end(), {R1, TR, CT, WR, MM});
        r.out = MM;
    } else {
        // experts * weights, then the sum of the n_used [H, T] views
        ggml_tensor *MU = u.only(D);
        if (!is_op(MU, GGML_OP_MUL) || MU->src[0] != D || MU->src[1] != Wn) return false;
        N.push_back(MU);
        std::vector<ggml_tensor *> views;
        for (ggml_tensor *c : u.of(MU)) {
            if (!is_op(c, GGML_OP_VIEW)) return false;
            views.push_back(c);
        }
        if ((int64_t) views.size() != r.n_used) return false;
        N.insert(N.end(), views.begin(), views.end());
        if (r.n_used == 1) {
            ggml_tensor *CT = u.only(views[0]);
            if (!is_op(CT, GGML_OP_CONT)) return false;
            N.push_back(CT);
            r.out = CT;
        } else {
            // the chain add(add(v0, v1), v2) ... : every view feeds one add of the chain
            std::unordered_set<ggml_tensor *> vs(views.begin(), views.end());
            ggml_tensor *cur = nullptr;
            for (ggml_tensor *v : views) {
                ggml_tensor *a = u.only(v);
                if (!is_op(a, GGML_OP_ADD)) return false;
                if (vs.count(a->src[0]) && vs.count(a->src[1])) cur = a;
            }
            if (!cur) return false;
            N.push_back(cur);
            for (int64_t k = 2; k < r.n_used; ++k) {
                ggml_tensor *nx = u.only(cur);
                if (!is_op(nx, GGML_OP_ADD) || nx->src[0] != cur || !vs.count(nx->src[1])) return false;
                N.push_back(nx);
                cur = nx;
            }
            r.out = cur;
        }
        // the sum must not have used the views in any other way
        for (ggml_tensor *v : views)
            for (ggml_tensor *c : u.of(v))
                if (!is_op(c, GGML_OP_ADD) && !is_op(c, GGML_OP_CONT)) return false;
    }
    if (!f32_contig(r.out) || r.out->ne[0] != r.H || r.out->ne[1] != r.T) return false;

    // the shared expert (runtime.cpp:2825-2833): moe_out + down_sh(silu(gate_sh x) * up_sh x),
    // the down output optionally times sigmoid(gate_inp_sh x), x the experts' input
    if (ggml_tensor *sa = u.only(r.out)) {
        ggml_tensor *sh = is_op(sa, GGML_OP_ADD) ? (sa->src[0] == r.out ? sa->src[1] : sa->src[0]) : nullptr;
        std::vector<ggml_tensor *> SN;
        ggml_tensor *gw = nullptr;
        if (sh && sh != r.out && is_op(sh, GGML_OP_MUL) && is_op(sh->src[1], GGML_OP_UNARY) &&
            ggml_get_unary_op(sh->src[1]) == GGML_UNARY_OP_SIGMOID) {
            ggml_tensor *sg = sh->src[1], *gi = sg->src[0];
            if (is_op(gi, GGML_OP_MUL_MAT) && gi->src[1] == r.x && f32_contig(gi->src[0]) &&
                ggml_nelements(gi->src[0]) == r.H && u.only(gi) == sg && u.only(sg) == sh) {
                gw = gi->src[0];
                SN.insert(SN.end(), {gi, sg, sh});
                sh = sh->src[0];
            } else {
                sh = nullptr;
            }
        }
        ggml_tensor *md = sh && is_op(sh, GGML_OP_MUL_MAT) ? sh : nullptr;
        ggml_tensor *mu = md ? md->src[1] : nullptr;
        ggml_tensor *sl = is_op(mu, GGML_OP_MUL) ? mu->src[0] : nullptr;
        ggml_tensor *mg = is_op(sl, GGML_OP_UNARY) && ggml_get_unary_op(sl) == GGML_UNARY_OP_SILU ? sl->src[0] : nullptr;
        ggml_tensor *mup = mu ? mu->src[1] : nullptr;
        if (is_op(mg, GGML_OP_MUL_MAT) && is_op(mup, GGML_OP_MUL_MAT) && mg->src[1] == r.x && mup->src[1] == r.x &&
            mg->src[0]->type == r.wg->type && mup->src[0]->type == r.wg->type && md->src[0]->type == r.wd->type &&
            ggml_n_dims(mg->src[0]) == 2 && ggml_n_dims(mup->src[0]) == 2 && ggml_n_dims(md->src[0]) == 2 &&
            u.only(mg) == sl && u.only(sl) == mu && u.only(mup) == mu && u.only(mu) == md &&
            (SN.empty() ? u.only(md) == sa : u.only(md) == SN.back()) && f32_contig(sa) &&
            ggml_are_same_shape(sa, r.out) && !(r.out->flags & GGML_TENSOR_FLAG_OUTPUT)) {
            r.sh_g = mg->src[0];
            r.sh_u = mup->src[0];
            r.sh_d = md->src[0];
            r.sh_gate_inp = gw;
            N.insert(N.end(), {mg, mup, sl, mu, md});
            N.insert(N.end(), SN.begin(), SN.end());
            N.push_back(sa);
            r.out = sa;
        }
    }

    ggml_tensor *head = logits;  // the layer's first node: it reads only inputs from outside
    // ffn_in = rms_norm(cur) * ffn_norm (runtime.cpp:2979) when nothing else reads it (a
    // shared expert does), and l_out = moe_out + cur (:2993): one qwb_moe_ffn call then
    // covers the whole block, its router normalising on the fly
    {
        ggml_tensor *xm = r.x, *rn = xm->src[0], *nw = xm->src[1];
        bool only_region = is_op(xm, GGML_OP_MUL) && is_op(rn, GGML_OP_RMS_NORM) && u.only(rn) == xm &&
                           !(xm->flags & GGML_TENSOR_FLAG_OUTPUT) && !(rn->flags & GGML_TENSOR_FLAG_OUTPUT) &&
                           f32_contig(nw) && nw->ne[0] == r.H && ggml_nelements(nw) == r.H &&
                           f32_contig(rn->src[0]) && ggml_are_same_shape(rn->src[0], xm);
        if (only_region) {
            std::unordered_set<const ggml_tensor *> in0(N.begin(), N.end());
            for (ggml_tensor *c : u.of(xm)) only_region &= in0.count(c) != 0;
        }
        if (only_region) {
            memcpy(&r.norm_eps, rn->op_params, sizeof(float));
            r.norm_w = nw;
            r.x = rn->src[0];
            head = rn;
            N.insert(N.end(), {rn, xm});
        }
    }
    if (ggml_tensor *add = u.only(r.out)) {
        ggml_tensor *other = add->src[0] == r.out ? add->src[1] : add->src[0];
        if (is_op(add, GGML_OP_ADD) && (add->src[0] == r.out || add->src[1] == r.out) && other != r.out &&
            f32_contig(other) && ggml_are_same_shape(other, r.out) && f32_contig(add) &&
            !(r.out->flags & GGML_TENSOR_FLAG_OUTPUT) && (!r.norm_w || other == r.x)) {
            N.push_back(add);
            r.residual = other;
            r.out = add;
        }
    }

    // every intermediate is read only inside the layer; the selection and the weights may
    // also be read after it (the expert cache records the selection)
    std::unordered_set<const ggml_tensor *> in(N.begin(), N.end());
    for (ggml_tensor *n : N) {
        const bool is_out = n == r.out;
        bool external = (n->flags & GGML_TENSOR_FLAG_OUTPUT) != 0;
        for (ggml_tensor *c : u.of(n))
            if (!in.count(c)) external = true;
        if (!external || is_out) continue;
        if (n == r.sel) r.sel_out = true;
        else if (n == r.weights) r.weights_out = true;
        else return false;
    }
    r.first = 1 << 30;
    for (ggml_tensor *n : N) {
        auto it = u.index.find(n);
        if (it == u.index.end()) return false;
        r.first = std::min(r.first, it->second);
    }
    if (u.index.at(head) != r.first) return false;
    // consecutive nodes: nothing runs between the fused call and the nodes that would have
    // produced its results, so it writes them in place (see d_compute)
    int last = 0;
    for (ggml_tensor *n : N) last = std::max(last, u.index.at(n));
    r.direct = last - r.first + 1 == (int) N.size();
    qwb_moe_ffn_desc d{};
    d.gate = view_of(r.wg);
    d.up = view_of(r.wu);
    d.down = view_of(r.wd);
    d.H = r.H; d.F = r.F; d.E = r.E; d.n_used = r.n_used; d.T = r.T;
    if (r.sh_d) {
        d.shexp_gate = view_of(r.sh_g);
        d.shexp_up = view_of(r.sh_u);
        d.shexp_down = view_of(r.sh_d);
    }
    return qwb_moe_ffn_workspace_size(&d) > 0;
}

// ============================================================== standalone mode

struct DevCtx {
    int device = 0;
    std::string name, description, pci_id;
    ggml_backend_buffer_type buft{};
    ggml_backend_device dev{};
};

struct BufCtx {
    void *ptr = nullptr;
    int device = 0;
};

struct BackendCtx {
    DevCtx *dev = nullptr;
    cudaStream_t stream = nullptr;
    Scratch sc;
};

std::vector<DevCtx *> &devices() {
    static std::vector<DevCtx *> d;
    return d;
}

void buf_free(ggml_backend_buffer_t b) {
    auto *c = (BufCtx *) b->context;
    cudaSetDevice(c->device);
    cuda_ok(cudaFree(c->ptr), "cudaFree");
    delete c;
}

void *buf_base(ggml_backend_buffer_t b) { return ((BufCtx *) b->context)->ptr; }

// Host copies are ordered after all work queued on the device: the backend's stream is a
// blocking stream, so the legacy default stream used here waits for it.
void buf_memset(ggml_backend_buffer_t b, ggml_tensor *t, uint8_t v, size_t off, size_t n) {
    cudaSetDevice(((BufCtx *) b->context)->device);
    cuda_ok(cudaMemset((char *) t->data + off, v, n), "cudaMemset");
}

void buf_set(ggml_backend_buffer_t b, ggml_tensor *t, const void *src, size_t off, size_t n) {
    cudaSetDevice(((BufCtx *) b->context)->device);
    cuda_ok(cudaMemcpy((char *) t->data + off, src, n, cudaMemcpyHostToDevice), "set_tensor");
}

void buf_get(ggml_backend_buffer_t b, const ggml_tensor *t, void *dst, size_t off, size_t n) {
    cudaSetDevice(((BufCtx *) b->context)->device);
    cuda_ok(cudaMemcpy(dst, (const char *) t->data + off, n, cudaMemcpyDeviceToHost), "get_tensor");
}

const char *buft_name(ggml_backend_buffer_type_t bt);

bool is_qwb_buffer(ggml_backend_buffer_t b) { return b && b->buft && b->buft->iface.get_name == buft_name; }

bool buf_cpy(ggml_backend_buffer_t b, const ggml_tensor *src, ggml_tensor *dst) {
    ggml_backend_buffer_t sb = src->view_src ? src->view_src->buffer : src->buffer;
    if (!is_qwb_buffer(sb)) return false;
    cudaSetDevice(((BufCtx *) b->context)->device);
    return cuda_ok(cudaMemcpy(dst->data, src->data, ggml_nbytes(src), cudaMemcpyDefault), "cpy_tensor");
}

void buf_clear(ggml_backend_buffer_t b, uint8_t v) {
    cudaSetDevice(((BufCtx *) b->context)->device);
    cuda_ok(cudaMemset(((BufCtx *) b->context)->ptr, v, b->size), "clear");
}

ggml_backend_buffer_i buffer_iface() {
    ggml_backend_buffer_i i{};
    i.free_buffer = buf_free;
    i.get_base = buf_base;
    i.memset_tensor = buf_memset;
    i.set_tensor = buf_set;
    i.get_tensor = buf_get;
    i.cpy_tensor = buf_cpy;
    i.clear = buf_clear;
    return i;
}

const char *buft_name(ggml_backend_buffer_type_t bt) { return ((DevCtx *) bt->context)->name.c_str(); }

ggml_backend_buffer_t buft_alloc(ggml_backend_buffer_type_t bt, size_t size) {
    auto *d = (DevCtx *) bt->context;
    cudaSetDevice(d->device);
    void *p = nullptr;
    // ggml asks for 0-byte buffers for graphs without tensors; hand out one aligned unit
    if (!cuda_ok(cudaMalloc(&p, size ? size : kAlign), "cudaMalloc")) return nullptr;
    auto *c = new BufCtx{p, d->device};
    return ggml_backend_buffer_init(bt, buffer_iface(), c, size);
}

size_t buft_alignment(ggml_backend_buffer_type_t) { return kAlign; }
bool buft_is_host(ggml_backend_buffer_type_t) { return false; }

ggml_guid *backend_guid() {
    static ggml_guid g = {0x51, 0x57, 0x42, 0x32, 0x30, 0x30, 0x6d, 0x6f,
                          0x65, 0x2d, 0x73, 0x6d, 0x31, 0x30, 0x30, 0x61};
    return &g;
}

const char *be_name(ggml_backend_t be) { return ((BackendCtx *) be->context)->dev->name.c_str(); }

void be_free(ggml_backend_t be) {
    auto *c = (BackendCtx *) be->context;
    cudaSetDevice(c->dev->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    c->sc.release();
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    delete be;
}

void be_set_async(ggml_backend_t be, ggml_tensor *t, const void *src, size_t off, size_t n) {
    auto *c = (BackendCtx *) be->context;
    cuda_ok(cudaMemcpyAsync((char *) t->data + off, src, n, cudaMemcpyHostToDevice, c->stream), "set_tensor_async");
}

void be_get_async(ggml_backend_t be, const ggml_tensor *t, void *dst, size_t off, size_t n) {
    auto *c = (BackendCtx *) be->context;
    cuda_ok(cudaMemcpyAsync(dst, (const char *) t->data + off, n, cudaMemcpyDeviceToHost, c->stream),
            "get_tensor_async");
}

// Waits for the stream, then reports (and clears) device-side id errors recorded by the
// kernels since the last synchronize.
void be_sync(ggml_backend_t be) {
    auto *c = (BackendCtx *) be->context;
    cudaSetDevice(c->dev->device);
    c->sc.report(c->stream);
}

ggml_status be_compute(ggml_backend_t be, ggml_cgraph *g) {
    auto *c = (BackendCtx *) be->context;
    cudaSetDevice(c->dev->device);
    for (int n = 0; n < ggml_graph_n_nodes(g); ++n) {
        ggml_tensor *t = ggml_graph_node(g, n);
        if (ggml_is_empty(t) || view_op(t->op)) continue;
        if (t->op != GGML_OP_MUL_MAT_ID && t->op != GGML_OP_MUL_MAT && t->op != GGML_OP_GET_ROWS) {
            std::fprintf(stderr, "ggml-qwb: op %s (%s) is not supported\n", ggml_op_name(t->op), t->name);
            return GGML_STATUS_FAILED;
        }
        bool short_ws = false;
        const qwb_status rc = run_node(t, c->sc, c->stream, &short_ws);
        if (short_ws) return GGML_STATUS_ALLOC_FAILED;
        if (rc != QWB_OK) {
            std::fprintf(stderr, "ggml-qwb: %s (%s): %s\n", ggml_op_name(t->op), t->name, qwb_status_string(rc));
            return GGML_STATUS_FAILED;
        }
    }
    return GGML_STATUS_SUCCESS;
}

// The scheduler hands every split to graph_optimize before computing it: size the
// workspace here, outside graph_compute.
void be_optimize(ggml_backend_t be, ggml_cgraph *g, ggml_backend_graph_optimize_params *) {
    auto *c = (BackendCtx *) be->context;
    size_t need = 0;
    for (int n = 0; n < g->n_nodes; ++n) need = std::max(need, node_workspace(g->nodes[n]));
    c->sc.grow(need);
}

ggml_backend_i backend_iface() {
    ggml_backend_i i{};
    i.get_name = be_name;
    i.free = be_free;
    i.set_tensor_async = be_set_async;
    i.get_tensor_async = be_get_async;
    i.synchronize = be_sync;
    i.graph_compute = be_compute;
    i.graph_optimize = be_optimize;
    return i;
}

const char *dev_name(ggml_backend_dev_t d) { return ((DevCtx *) d->context)->name.c_str(); }
const char *dev_description(ggml_backend_dev_t d) { return ((DevCtx *) d->context)->description.c_str(); }

void dev_memory(ggml_backend_dev_t d, size_t *free_b, size_t *total_b) {
    cudaSetDevice(((DevCtx *) d->context)->device);
    *free_b = *total_b = 0;
    cudaMemGetInfo(free_b, total_b);
}

enum ggml_backend_dev_type dev_type(ggml_backend_dev_t) { return GGML_BACKEND_DEVICE_TYPE_GPU; }

void dev_props(ggml_backend_dev_t d, ggml_backend_dev_props *p) {
    auto *c = (DevCtx *) d->context;
    p->name = c->name.c_str();
    p->description = c->description.c_str();
    dev_memory(d, &p->memory_free, &p->memory_total);
    p->type = GGML_BACKEND_DEVICE_TYPE_GPU;
    p->device_id = c->pci_id.empty() ? nullptr : c->pci_id.c_str();
    p->caps = {};
    p->caps.async = true;
}

size_t param_size(const char *params, const char *key, size_t dflt) {
    if (!params) return dflt;
    const char *w = std::strstr(params, key);
    return w ? (size_t) std::strtoull(w + std::strlen(key), nullptr, 10) : dflt;
}

// params: "workspace_mb=N" (workspace reserved up front, default 256 MiB).
ggml_backend_t dev_init(ggml_backend_dev_t d, const char *params) {
    auto *dc = (DevCtx *) d->context;
    const size_t mb = param_size(params, "workspace_mb=", kDefaultWorkspaceMb);
    if (!cuda_ok(cudaSetDevice(dc->device), "cudaSetDevice")) return nullptr;
    auto *c = new BackendCtx();
    c->dev = dc;
    bool ok = cuda_ok(cudaStreamCreateWithFlags(&c->stream, cudaStreamDefault), "cudaStreamCreate") &&
              c->sc.init(dc->device, mb);
    auto *be = new ggml_backend{};
    be->guid = backend_guid();
    be->iface = backend_iface();
    be->device = d;
    be->context = c;
    if (!ok) {
        be_free(be);
        return nullptr;
    }
    return be;
}

ggml_backend_buffer_type_t dev_buft(ggml_backend_dev_t d) { return &((DevCtx *) d->context)->buft; }
bool dev_supports_op(ggml_backend_dev_t, const ggml_tensor *op) { return supported_standalone(op); }
bool dev_supports_buft(ggml_backend_dev_t d, ggml_backend_buffer_type_t bt) { return bt == dev_buft(d); }
bool dev_offload_op(ggml_backend_dev_t, const ggml_tensor *) { return false; }

void standalone_devices(ggml_backend_reg_t reg) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    for (int i = 0; i < n; ++i) {
        cudaDeviceProp prop{};
        if (cudaGetDeviceProperties(&prop, i) != cudaSuccess || prop.major != 10) continue;
        auto *dc = new DevCtx();
        dc->device = i;
        dc->name = "QWB" + std::to_string(devices().size());
        dc->description = prop.name;
        char pci[32];
        std::snprintf(pci, sizeof pci, "%04x:%02x:%02x.0", prop.pciDomainID, prop.pciBusID, prop.pciDeviceID);
        dc->pci_id = pci;
        dc->buft.iface.get_name = buft_name;
        dc->buft.iface.alloc_buffer = buft_alloc;
        dc->buft.iface.get_alignment = buft_alignment;
        dc->buft.iface.is_host = buft_is_host;
        dc->buft.device = &dc->dev;
        dc->buft.context = dc;
        ggml_backend_device_i &di = dc->dev.iface;
        di.get_name = dev_name;
        di.get_description = dev_description;
        di.get_memory = dev_memory;
        di.get_type = dev_type;
        di.get_props = dev_props;
        di.init_backend = dev_init;
        di.get_buffer_type = dev_buft;
        di.supports_op = dev_supports_op;
        di.supports_buft = dev_supports_buft;
        di.offload_op = dev_offload_op;
        dc->dev.reg = reg;
        dc->dev.context = dc;
        devices().push_back(dc);
    }
}

// ============================================================== delegating mode

struct DDev {
    ggml_backend_dev_t inner = nullptr;
    int device = 0;
    std::string name, description;
    ggml_backend_device dev{};
};

std::vector<DDev *> &ddevices() {
    static std::vector<DDev *> d;
    return d;
}

// counters of what graph_compute did (ggml_backend_qwb_get_stats)
enum { kStatFused, kStatOwnNodes, kStatInnerNodes, kStatInnerRuns, kStatN };

struct DBackend {
    DDev *dev = nullptr;
    ggml_backend_t inner = nullptr;
    cudaStream_t stream = nullptr;
    cudaEvent_t ev_to_ours = nullptr, ev_to_inner = nullptr;
    Scratch sc;
    bool fuse = true, own_mul_mat = false;
    int64_t fuse_max_tokens = 64;  // larger batches: per-node MUL_MAT_ID (tensor-core GEMMs)
    bool ours_active = false;  // this library's stream holds work the inner stream has not joined
    std::vector<ggml_tensor *> run;
    uint64_t stats[kStatN] = {};
    // fused layers of the graph being computed
    Uses uses;
    std::vector<MoeRegion> regions;
    std::unordered_map<const ggml_tensor *, int> region_of;
    bool analysed = false;
    uint64_t fingerprint = 0;
};

ggml_guid *dbackend_guid() {
    static ggml_guid g = {0x51, 0x57, 0x42, 0x44, 0x65, 0x6c, 0x65, 0x67,
                          0x61, 0x74, 0x65, 0x2d, 0x73, 0x6d, 0x31, 0x30};
    return &g;
}

bool is_dbackend(ggml_backend_t b) { return b && ggml_guid_matches(b->guid, dbackend_guid()); }
ggml_backend_t inner_of(ggml_backend_t b) { return is_dbackend(b) ? ((DBackend *) b->context)->inner : b; }

#ifdef QWB_HANDOFF_FENCE
__global__ void handoff_fence_kernel() {}
#endif

// inner stream -> this library's stream
void to_ours(DBackend *c) {
    if (c->ours_active) return;
    ggml_backend_event e{c->dev->inner, (void *) c->ev_to_ours};
    c->inner->iface.event_record(c->inner, &e);
    cuda_ok(cudaStreamWaitEvent(c->stream, c->ev_to_ours, 0), "cudaStreamWaitEvent");
#ifdef QWB_HANDOFF_FENCE
    handoff_fence_kernel<<<1, 1, 0, c->stream>>>();
#endif
#ifdef QWB_DEBUG_SYNC
    cudaDeviceSynchronize();
#endif
    c->ours_active = true;
}
// this library's stream -> inner stream
void to_inner(DBackend *c) {
    if (!c->ours_active) return;
    cuda_ok(cudaEventRecord(c->ev_to_inner, c->stream), "cudaEventRecord");
    ggml_backend_event e{c->dev->inner, (void *) c->ev_to_inner};
    c->inner->iface.event_wait(c->inner, &e);
#ifdef QWB_DEBUG_SYNC
    cudaDeviceSynchronize();
#endif
    c->ours_active = false;
}

ggml_status flush_run(DBackend *c, ggml_cgraph *g) {
    bool work = false;
    for (const ggml_tensor *t : c->run) work |= !view_op(t->op);
    if (!work) {  // views only: nothing for ggml-cuda to do, no hand-over needed
        c->run.clear();
        return GGML_STATUS_SUCCESS;
    }
    to_inner(c);
    ggml_cgraph sub = ggml_graph_view(g, 0, 0);
    sub.nodes = c->run.data();
    sub.n_nodes = (int) c->run.size();
    const ggml_status st = c->inner->iface.graph_compute(c->inner, &sub);
    c->stats[kStatInnerNodes] += c->run.size();
    c->stats[kStatInnerRuns] += 1;
    c->run.clear();
    return st;
}

// workspace layout of a fused layer: qwb_moe_ffn's workspace, then its outputs (moe_out,
// selection, weights), copied into the graph's tensors where ggml produces them
struct FusedLayout {
    size_t ffn, out, sel, w, total;
};
FusedLayout fused_layout(const MoeRegion &r, const qwb_moe_ffn_desc &d) {
    FusedLayout l{};
    auto up = [](size_t v) { return (v + kAlign - 1) / kAlign * kAlign; };
    l.ffn = up(qwb_moe_ffn_workspace_size(&d));
    l.out = l.ffn;
    l.sel = l.out + up((size_t) (r.H * r.T) * 4);
    l.w = l.sel + up((size_t) (r.n_used * r.T) * 4);
    l.total = l.w + up((size_t) (r.n_used * r.T) * 4);
    return l;
}
qwb_moe_ffn_desc fused_desc(const MoeRegion &r) {
    qwb_moe_ffn_desc d{};
    d.x = (const float *) r.x->data;
    d.norm_w = r.norm_w ? (const float *) r.norm_w->data : nullptr;
    d.norm_eps = r.norm_eps;
    d.residual = r.residual ? (const float *) r.residual->data : nullptr;
    d.router_w = (const float *) r.router_w->data;
    d.g2s = r.g2s;
    d.gate = view_of(r.wg);
    d.up = view_of(r.wu);
    d.down = view_of(r.wd);
    d.H = r.H; d.F = r.F; d.E = r.E; d.n_used = r.n_used; d.T = r.T;
    if (r.sh_d) {
        d.shexp_gate = view_of(r.sh_g);
        d.shexp_up = view_of(r.sh_u);
        d.shexp_down = view_of(r.sh_d);
        d.shexp_gate_inp = r.sh_gate_inp ? (const float *) r.sh_gate_inp->data : nullptr;
    }
    return d;
}

// Structure of a graph: nodes, ops and operands (a graph computed again, QuestWend's
// reused decode graph, keeps its analysis).
uint64_t graph_fingerprint(const ggml_cgraph *g) {
    uint64_t h = 1469598103934665603ull ^ (uint64_t) g->n_nodes;
    auto mix = [&h](uint64_t v) { h = (h ^ v) * 1099511628211ull; };
    for (int i = 0; i < g->n_nodes; ++i) {
        const ggml_tensor *n = g->nodes[i];
        mix((uint64_t) (uintptr_t) n);
        mix((uint64_t) n->op | ((uint64_t) n->flags << 32));
        for (int s = 0; s < 3; ++s) mix((uint64_t) (uintptr_t) n->src[s]);
    }
    return h;
}

void find_regions(DBackend *c, ggml_cgraph *g) {
    const uint64_t fp = graph_fingerprint(g);
    if (c->analysed && fp == c->fingerprint) return;
    c->analysed = true;
    c->fingerprint = fp;
    c->regions.clear();
    c->region_of.clear();
    if (!c->fuse) return;
    c->uses.build(g);
    for (int i = 0; i < g->n_nodes; ++i) {
        ggml_tensor *n = g->nodes[i];
        if (n->op != GGML_OP_MUL_MAT_ID || c->region_of.count(n)) continue;
        MoeRegion r;
        if (!match_moe(c->uses, n, r) || r.T > c->fuse_max_tokens) continue;
        bool overlap = false;
        for (ggml_tensor *m : r.nodes) overlap |= c->region_of.count(m) != 0;
        if (overlap) continue;
        const int id = (int) c->regions.size();
        for (ggml_tensor *m : r.nodes) c->region_of[m] = id;
        c->regions.push_back(std::move(r));
    }
    // A fused layer leaves its results in the workspace until the graph reaches the nodes
    // that produce them; no other workspace user may run in between (in QuestWend's graphs
    // the layer's nodes are consecutive).  Layers that would overlap one are not fused.
    std::vector<int> last(c->regions.size());
    for (size_t k = 0; k < c->regions.size(); ++k) {
        const MoeRegion &r = c->regions[k];
        int l = c->uses.index.at(r.out);
        if (r.sel_out) l = std::max(l, c->uses.index.at(r.sel));
        if (r.weights_out) l = std::max(l, c->uses.index.at(r.weights));
        last[k] = l;
    }
    std::vector<bool> keep(c->regions.size(), true);
    for (size_t k = 0; k < c->regions.size(); ++k) {
        const MoeRegion &r = c->regions[k];
        for (int i = r.first + 1; i <= last[k] && keep[k]; ++i) {
            const ggml_tensor *t = g->nodes[i];
            auto it = c->region_of.find(t);
            if (it != c->region_of.end()) {
                if (it->second != (int) k && c->regions[it->second].first == i) keep[k] = false;
            } else if (node_workspace(t) > 0) {
                keep[k] = false;
            }
        }
    }
    if (std::find(keep.begin(), keep.end(), false) != keep.end()) {
        std::vector<MoeRegion> kept;
        for (size_t k = 0; k < c->regions.size(); ++k)
            if (keep[k]) kept.push_back(std::move(c->regions[k]));
        c->regions = std::move(kept);
        c->region_of.clear();
        for (size_t k = 0; k < c->regions.size(); ++k)
            for (ggml_tensor *m : c->regions[k].nodes) c->region_of[m] = (int) k;
    }
}

size_t graph_workspace(DBackend *c, ggml_cgraph *g) {
    find_regions(c, g);
    size_t need = 0;
    for (const MoeRegion &r : c->regions) need = std::max(need, fused_layout(r, fused_desc(r)).total);
    for (int i = 0; i < g->n_nodes; ++i)
        if (!c->region_of.count(g->nodes[i])) need = std::max(need, node_workspace(g->nodes[i]));
    return need;
}

bool own_node(const DBackend *c, const ggml_tensor *t) {
    switch (t->op) {
        case GGML_OP_MUL_MAT_ID: return supported_mmid(t);
        case GGML_OP_GET_ROWS: return supported_get_rows(t, false);
        case GGML_OP_MUL_MAT: return c->own_mul_mat && supported_mul_mat(t);
        default: return false;
    }
}

ggml_status d_compute(ggml_backend_t be, ggml_cgraph *g) {
    auto *c = (DBackend *) be->context;
    cudaSetDevice(c->dev->device);
    find_regions(c, g);
    std::vector<FusedLayout> layouts;
    for (const MoeRegion &r : c->regions) {
        layouts.push_back(fused_layout(r, fused_desc(r)));
        if (!c->sc.fits(layouts.back().total, r.out)) return GGML_STATUS_ALLOC_FAILED;
    }
    ggml_status st = GGML_STATUS_SUCCESS;
    for (int i = 0; i < g->n_nodes && st == GGML_STATUS_SUCCESS; ++i) {
        ggml_tensor *t = g->nodes[i];
        auto rit = c->region_of.find(t);
        if (rit != c->region_of.end()) {
            const MoeRegion &r = c->regions[rit->second];
            const FusedLayout &l = layouts[rit->second];
            char *ws = (char *) c->sc.ws;
            if (i == r.first) {
                if ((st = flush_run(c, g)) != GGML_STATUS_SUCCESS) break;
                to_ours(c);
                qwb_moe_ffn_desc d = fused_desc(r);
                d.out = (float *) (ws + l.out);
                d.selected = (int32_t *) (ws + l.sel);
                d.weights = (float *) (ws + l.w);
                if (r.direct) {
                    // nothing else runs until the layer's last node: its result tensors hold
                    // no live data now (ggml-alloc gave them memory free from the layer's
                    // first node on, or the residual operand itself, read before written)
                    d.out = (float *) r.out->data;
                    d.weights = r.weights_out ? (float *) r.weights->data : d.weights;
                }
                const qwb_status rc = qwb_moe_ffn(&d, ws, l.ffn, c->sc.status, (qwb_stream_t) c->stream);
                if (rc != QWB_OK) {
                    std::fprintf(stderr, "ggml-qwb: fused MoE layer (%s): %s\n", r.out->name, qwb_status_string(rc));
                    st = GGML_STATUS_FAILED;
                    break;
                }
                c->stats[kStatFused] += 1;
            }
            // the layer's results land in the graph's tensors where ggml would produce them
            // (so ggml-alloc's reuse of their memory before that point stays valid)
            cudaError_t e = cudaSuccess;
            if (r.direct && t != r.sel) {
                // written in place by the fused call
            } else if (t == r.out) {
                to_ours(c);
                e = cudaMemcpyAsync(r.out->data, ws + l.out, (size_t) (r.H * r.T) * 4, cudaMemcpyDeviceToDevice,
                                    c->stream);
            } else if (t == r.sel && r.sel_out) {
                to_ours(c);
                e = cudaMemcpy2DAsync(r.sel->data, r.sel->nb[1], ws + l.sel, (size_t) r.n_used * 4,
                                      (size_t) r.n_used * 4, (size_t) r.T, cudaMemcpyDeviceToDevice, c->stream);
            } else if (t == r.weights && r.weights_out) {
                to_ours(c);
                e = cudaMemcpyAsync(r.weights->data, ws + l.w, (size_t) (r.n_used * r.T) * 4,
                                    cudaMemcpyDeviceToDevice, c->stream);
            }
            if (e != cudaSuccess) {
                std::fprintf(stderr, "ggml-qwb: copy of a fused result: %s\n", cudaGetErrorString(e));
                st = GGML_STATUS_FAILED;
            }
            continue;
        }
        if (ggml_is_empty(t)) continue;
        if (own_node(c, t)) {
            if ((st = flush_run(c, g)) != GGML_STATUS_SUCCESS) break;
            to_ours(c);
            bool short_ws = false;
            const qwb_status rc = run_node(t, c->sc, c->stream, &short_ws);
            if (short_ws) {
                st = GGML_STATUS_ALLOC_FAILED;
                break;
            }
            if (rc != QWB_OK) {
                std::fprintf(stderr, "ggml-qwb: %s (%s): %s\n", ggml_op_name(t->op), t->name, qwb_status_string(rc));
                st = GGML_STATUS_FAILED;
                break;
            }
            c->stats[kStatOwnNodes] += 1;
            continue;
        }
        c->run.push_back(t);
    }
    if (st == GGML_STATUS_SUCCESS) st = flush_run(c, g);
    c->run.clear();
    to_inner(c);  // every call ends with its work on the inner stream
    return st;
}

void d_optimize(ggml_backend_t be, ggml_cgraph *g, ggml_backend_graph_optimize_params *) {
    auto *c = (DBackend *) be->context;
    c->sc.grow(graph_workspace(c, g));
}

const char *d_name(ggml_backend_t be) { return ((DBackend *) be->context)->dev->name.c_str(); }

void d_free(ggml_backend_t be) {
    auto *c = (DBackend *) be->context;
    cudaSetDevice(c->dev->device);
    if (c->inner) ggml_backend_synchronize(c->inner);
    if (c->stream) cudaStreamSynchronize(c->stream);
    c->sc.release();
    if (c->ev_to_ours) cudaEventDestroy(c->ev_to_ours);
    if (c->ev_to_inner) cudaEventDestroy(c->ev_to_inner);
    if (c->stream) cudaStreamDestroy(c->stream);
    if (c->inner) ggml_backend_free(c->inner);
    delete c;
    delete be;
}

void d_set_async(ggml_backend_t be, ggml_tensor *t, const void *src, size_t off, size_t n) {
    ggml_backend_t in = ((DBackend *) be->context)->inner;
    in->iface.set_tensor_async(in, t, src, off, n);
}
void d_get_async(ggml_backend_t be, const ggml_tensor *t, void *dst, size_t off, size_t n) {
    ggml_backend_t in = ((DBackend *) be->context)->inner;
    in->iface.get_tensor_async(in, t, dst, off, n);
}
void d_set_2d_async(ggml_backend_t be, ggml_tensor *t, const void *src, size_t off, size_t size, size_t n,
                    size_t st, size_t sd) {
    ggml_backend_t in = ((DBackend *) be->context)->inner;
    in->iface.set_tensor_2d_async(in, t, src, off, size, n, st, sd);
}
void d_get_2d_async(ggml_backend_t be, const ggml_tensor *t, void *dst, size_t off, size_t size, size_t n,
                    size_t st, size_t sd) {
    ggml_backend_t in = ((DBackend *) be->context)->inner;
    in->iface.get_tensor_2d_async(in, t, dst, off, size, n, st, sd);
}
// either end may be this backend: hand ggml-cuda its own backends
bool d_cpy_async(ggml_backend_t bsrc, ggml_backend_t bdst, const ggml_tensor *src, ggml_tensor *dst) {
    ggml_backend_t is = inner_of(bsrc), id = inner_of(bdst);
    ggml_backend_t exec = is_dbackend(bdst) ? id : is;
    if (!exec->iface.cpy_tensor_async) return false;
    return exec->iface.cpy_tensor_async(is, id, src, dst);
}
void d_sync(ggml_backend_t be) {
    auto *c = (DBackend *) be->context;
    cudaSetDevice(c->dev->device);
    to_inner(c);
    c->inner->iface.synchronize(c->inner);
    c->sc.report(c->stream);
}
void d_event_record(ggml_backend_t be, ggml_backend_event_t ev) {
    auto *c = (DBackend *) be->context;
    to_inner(c);
    ggml_backend_event e{c->dev->inner, ev->context};
    c->inner->iface.event_record(c->inner, &e);
}
void d_event_wait(ggml_backend_t be, ggml_backend_event_t ev) {
    auto *c = (DBackend *) be->context;
    ggml_backend_event e{c->dev->inner, ev->context};
    c->inner->iface.event_wait(c->inner, &e);
}

ggml_backend_i dbackend_iface(ggml_backend_t inner) {
    ggml_backend_i i{};
    i.get_name = d_name;
    i.free = d_free;
    i.set_tensor_async = inner->iface.set_tensor_async ? d_set_async : nullptr;
    i.get_tensor_async = inner->iface.get_tensor_async ? d_get_async : nullptr;
    i.set_tensor_2d_async = inner->iface.set_tensor_2d_async ? d_set_2d_async : nullptr;
    i.get_tensor_2d_async = inner->iface.get_tensor_2d_async ? d_get_2d_async : nullptr;
    i.cpy_tensor_async = inner->iface.cpy_tensor_async ? d_cpy_async : nullptr;
    i.synchronize = d_sync;
    i.graph_compute = d_compute;
    i.event_record = inner->iface.event_record ? d_event_record : nullptr;
    i.event_wait = inner->iface.event_wait ? d_event_wait : nullptr;
    i.graph_optimize = d_optimize;
    return i;
}

const char *dd_name(ggml_backend_dev_t d) { return ((DDev *) d->context)->name.c_str(); }
const char *dd_description(ggml_backend_dev_t d) { return ((DDev *) d->context)->description.c_str(); }
void dd_memory(ggml_backend_dev_t d, size_t *f, size_t *t) { ggml_backend_dev_memory(((DDev *) d->context)->inner, f, t); }
enum ggml_backend_dev_type dd_type(ggml_backend_dev_t) { return GGML_BACKEND_DEVICE_TYPE_GPU; }
void dd_props(ggml_backend_dev_t d, ggml_backend_dev_props *p) {
    auto *c = (DDev *) d->context;
    ggml_backend_dev_get_props(c->inner, p);
    p->name = c->name.c_str();
    p->description = c->description.c_str();
    p->type = GGML_BACKEND_DEVICE_TYPE_GPU;
}

// params: "workspace_mb=N" (default 256), "fuse=0" (no build_moe fusion),
// "fuse_max_tokens=N" (fuse layers of at most N tokens, default 64: the fused layer runs
// its expert GEMVs on the weight-streaming kernel, while per-node MUL_MAT_ID takes the
// tensor-core GEMMs for many tokens per expert), "mul_mat=1" (quantized MUL_MAT on
// libqwb.so too); the rest is passed to ggml-cuda.
ggml_backend_t dd_init(ggml_backend_dev_t d, const char *params) {
    auto *dd = (DDev *) d->context;
    ggml_backend_t inner = ggml_backend_dev_init(dd->inner, params);
    if (!inner) return nullptr;
    if (!cuda_ok(cudaSetDevice(dd->device), "cudaSetDevice")) {
        ggml_backend_free(inner);
        return nullptr;
    }
    auto *c = new DBackend();
    c->dev = dd;
    c->inner = inner;
    c->fuse = param_size(params, "fuse=", 1) != 0;
    c->own_mul_mat = param_size(params, "mul_mat=", 0) != 0;
    c->fuse_max_tokens = (int64_t) param_size(params, "fuse_max_tokens=", 64);
    bool ok = cuda_ok(cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking), "cudaStreamCreate") &&
              cuda_ok(cudaEventCreateWithFlags(&c->ev_to_ours, cudaEventDisableTiming), "cudaEventCreate") &&
              cuda_ok(cudaEventCreateWithFlags(&c->ev_to_inner, cudaEventDisableTiming), "cudaEventCreate") &&
              c->sc.init(dd->device, param_size(params, "workspace_mb=", kDefaultWorkspaceMb));
    auto *be = new ggml_backend{};
    be->guid = dbackend_guid();
    be->iface = dbackend_iface(inner);
    be->device = d;
    be->context = c;
    if (!ok) {
        d_free(be);
        return nullptr;
    }
    return be;
}
ggml_backend_buffer_type_t dd_buft(ggml_backend_dev_t d) {
    return ggml_backend_dev_buffer_type(((DDev *) d->context)->inner);
}
ggml_backend_buffer_type_t dd_host_buft(ggml_backend_dev_t d) {
    return ggml_backend_dev_host_buffer_type(((DDev *) d->context)->inner);
}
ggml_backend_buffer_t dd_from_host_ptr(ggml_backend_dev_t d, void *p, size_t size, size_t max_tensor) {
    return ggml_backend_dev_buffer_from_host_ptr(((DDev *) d->context)->inner, p, size, max_tensor);
}
bool dd_supports_op(ggml_backend_dev_t d, const ggml_tensor *op) {
    auto *c = (DDev *) d->context;
    if ((op->op == GGML_OP_MUL_MAT_ID && supported_mmid(op)) || (op->op == GGML_OP_GET_ROWS && supported_get_rows(op, false)))
        return true;
    return ggml_backend_dev_supports_op(c->inner, op);
}
bool dd_supports_buft(ggml_backend_dev_t d, ggml_backend_buffer_type_t bt) {
    return ggml_backend_dev_supports_buft(((DDev *) d->context)->inner, bt);
}
bool dd_offload_op(ggml_backend_dev_t d, const ggml_tensor *op) {
    return ggml_backend_dev_offload_op(((DDev *) d->context)->inner, op);
}
ggml_backend_event_t dd_event_new(ggml_backend_dev_t d) {
    ggml_backend_event_t e = ggml_backend_event_new(((DDev *) d->context)->inner);
    if (e) e->device = d;  // recorded and waited through this device's backends
    return e;
}
void dd_event_free(ggml_backend_dev_t d, ggml_backend_event_t e) {
    auto *c = (DDev *) d->context;
    e->device = c->inner;
    c->inner->iface.event_free(c->inner, e);
}
void dd_event_sync(ggml_backend_dev_t d, ggml_backend_event_t e) {
    auto *c = (DDev *) d->context;
    ggml_backend_event ie{c->inner, e->context};
    c->inner->iface.event_synchronize(c->inner, &ie);
}

// Loads the stock ggml-cuda backend library without registering it with ggml (its
// devices are reached only through this library's).
ggml_backend_reg_t load_inner() {
    const char *mode = std::getenv("QWB_GGML_MODE");
    if (mode && !std::strcmp(mode, "standalone")) return nullptr;
    std::string path;
    if (const char *p = std::getenv("QWB_GGML_CUDA")) {
        path = p;
    } else {
        Dl_info info{};
        if (!dladdr((void *) &load_inner, &info) || !info.dli_fname) return nullptr;
        path = info.dli_fname;
        const size_t slash = path.rfind('/');
        path = (slash == std::string::npos ? std::string() : path.substr(0, slash + 1)) + "libggml-cuda.so";
    }
    void *h = dlopen(path.c_str(), RTLD_NOW | RTLD_LOCAL);
    if (!h) return nullptr;
    auto init = (ggml_backend_reg_t(*)()) dlsym(h, "ggml_backend_init");
    ggml_backend_reg_t r = init ? init() : nullptr;
    if (!r || r->api_version != GGML_BACKEND_API_VERSION) {
        if (r) std::fprintf(stderr, "ggml-qwb: %s has another backend interface version\n", path.c_str());
        return nullptr;  // the library stays loaded: a registry may already point into it
    }
    return r;
}

void delegating_devices(ggml_backend_reg_t reg, ggml_backend_reg_t inner) {
    for (size_t i = 0; i < ggml_backend_reg_dev_count(inner); ++i) {
        ggml_backend_dev_t idev = ggml_backend_reg_dev_get(inner, i);
        if (ggml_backend_dev_type(idev) != GGML_BACKEND_DEVICE_TYPE_GPU) continue;
        ggml_backend_dev_props p{};
        ggml_backend_dev_get_props(idev, &p);
        int cu = (int) i;
        if (p.device_id) {
            int id = -1;
            if (cudaDeviceGetByPCIBusId(&id, p.device_id) == cudaSuccess) cu = id;
            else cudaGetLastError();
        }
        cudaDeviceProp prop{};
        if (cudaGetDeviceProperties(&prop, cu) != cudaSuccess || prop.major != 10) {
            cudaGetLastError();
            continue;
        }
        auto *dd = new DDev();
        dd->inner = idev;
        dd->device = cu;
        dd->name = "QWB" + std::to_string(ddevices().size());
        dd->description = std::string(prop.name) + " (libqwb MoE kernels over " + ggml_backend_dev_name(idev) + ")";
        ggml_backend_device_i &di = dd->dev.iface;
        di.get_name = dd_name;
        di.get_description = dd_description;
        di.get_memory = dd_memory;
        di.get_type = dd_type;
        di.get_props = dd_props;
        di.init_backend = dd_init;
        di.get_buffer_type = dd_buft;
        di.get_host_buffer_type = idev->iface.get_host_buffer_type ? dd_host_buft : nullptr;
        di.buffer_from_host_ptr = idev->iface.buffer_from_host_ptr ? dd_from_host_ptr : nullptr;
        di.supports_op = dd_supports_op;
        di.supports_buft = dd_supports_buft;
        di.offload_op = idev->iface.offload_op ? dd_offload_op : nullptr;
        di.event_new = idev->iface.event_new ? dd_event_new : nullptr;
        di.event_free = idev->iface.event_free ? dd_event_free : nullptr;
        di.event_synchronize = idev->iface.event_synchronize ? dd_event_sync : nullptr;
        dd->dev.reg = reg;
        dd->dev.context = dd;
        ddevices().push_back(dd);
    }
}

// ---------------------------------------------------------------- registry

bool g_delegating = false;

const char *reg_name(ggml_backend_reg_t) { return "QWB"; }
size_t reg_count(ggml_backend_reg_t) { return g_delegating ? ddevices().size() : devices().size(); }
ggml_backend_dev_t reg_device(ggml_backend_reg_t, size_t i) {
    if (g_delegating) return i < ddevices().size() ? &ddevices()[i]->dev : nullptr;
    return i < devices().size() ? &devices()[i]->dev : nullptr;
}

// Counters since the backend was created: fused MoE layers, nodes run on libqwb.so one at
// a time, nodes handed to ggml-cuda and the sub-graphs they went in.  Returns the count
// written (0 for a backend of the standalone mode).
int qwb_backend_get_stats(ggml_backend_t be, uint64_t *out, int n) {
    if (!is_dbackend(be)) return 0;
    auto *c = (DBackend *) be->context;
    int k = 0;
    for (; k < n && k < kStatN; ++k) out[k] = c->stats[k];
    return k;
}
// Sizes the backend's workspace for a graph (outside graph_compute); true on success.
bool qwb_backend_reserve(ggml_backend_t be, ggml_cgraph *g) {
    if (is_dbackend(be)) {
        auto *c = (DBackend *) be->context;
        cudaSetDevice(c->dev->device);
        return c->sc.grow(graph_workspace(c, g));
    }
    auto *c = (BackendCtx *) be->context;
    size_t need = 0;
    for (int n = 0; n < g->n_nodes; ++n) need = std::max(need, node_workspace(g->nodes[n]));
    return c->sc.grow(need);
}
// 1 when the devices wrap ggml-cuda's (delegating mode), 0 in the standalone mode.
int qwb_backend_is_delegating() { return g_delegating ? 1 : 0; }

void *reg_proc(ggml_backend_reg_t, const char *name) {
    if (!std::strcmp(name, "ggml_backend_qwb_get_stats")) return (void *) qwb_backend_get_stats;
    if (!std::strcmp(name, "ggml_backend_qwb_reserve")) return (void *) qwb_backend_reserve;
    if (!std::strcmp(name, "ggml_backend_qwb_is_delegating")) return (void *) qwb_backend_is_delegating;
    return nullptr;
}

}  // namespace

// The registry of the process's B200 devices ("QWB0", "QWB1", ...): wrapping the stock
// ggml-cuda library's devices when it can be loaded, standalone otherwise; a process
// without a B200 gets a registry with no devices.
QWB_SHIM_API ggml_backend_reg_t ggml_backend_qwb_reg(void) {
    static ggml_backend_reg reg{};
    static std::once_flag once;
    std::call_once(once, [] {
        reg.api_version = GGML_BACKEND_API_VERSION;
        reg.iface.get_name = reg_name;
        reg.iface.get_device_count = reg_count;
        reg.iface.get_device = reg_device;
        reg.iface.get_proc_address = reg_proc;
        reg.context = nullptr;
        if (ggml_backend_reg_t inner = load_inner()) {
            delegating_devices(&reg, inner);
            g_delegating = !ddevices().empty();
        }
        if (!g_delegating) standalone_devices(&reg);
    });
    return &reg;
}

// Entry points of ggml's dynamic backend loader (ggml_backend_load).  The score is above
// the stock ggml-cuda build's so ggml_backend_load_all() prefers this library when both
// are installed as "cuda" variants.
QWB_SHIM_API ggml_backend_reg_t ggml_backend_init(void) { return ggml_backend_qwb_reg(); }
QWB_SHIM_API int ggml_backend_score(void) { return ggml_backend_qwb_reg()->iface.get_device_count(nullptr) ? 100 : 0; }
