// ref_harness.cpp - test/benchmark driver for the REFERENCE ggml CPU backend.
//
// TEST INFRASTRUCTURE ONLY.  This file is linked (by oracle/Makefile) against the
// reference's own ggml sources compiled from the reference tree (vendored llama.cpp
// ggml 1b70350c9).  It builds the same ggml graphs QuestWend builds for the MoE hot path
// and runs them on the ggml CPU backend, so the tests can compare the CUDA path with
// the reference's own arithmetic and bench.py can time the reference CPU path.
// Nothing in the product links this file.
//
// Graphs mirrored (reference core/runtime.cpp):
//   * route_experts        runtime.cpp:2693-2734  softmax -> argsort_top_k -> get_rows ->
//                                                sum_rows -> clamp(6.1035e-5) -> div
//   * build_moe            runtime.cpp:2743-2816  router mul_mat, 3x mul_mat_id,
//                                                swiglu_split, weighted reduce
//                                                (T=1: mul_mat(cont(transpose)), T>1: mul + adds)
//   * in-graph slot remap  runtime.cpp:2769-2778  get_rows(g2s I32 table, selected)
// Ops exercised: ggml_mul_mat_id (ggml.c:3413), ggml_get_rows (ggml.c:3975),
// ggml_argsort_top_k (ggml.c:5462), ggml_swiglu_split (ggml.c:3082).
// The qref_backend_* drivers run MUL_MAT_ID / GET_ROWS graphs on a ggml backend that this
// ggml loads from a shared library (ggml_backend_load), directly and through
// ggml_backend_sched, so the tests check a backend library as a host application uses it.
#include "ggml.h"
#include "ggml-alloc.h"
#include "ggml-backend.h"
#include "ggml-cpu.h"

#include <algorithm>

#include <chrono>
#include <cmath>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <map>
#include <string>
#include <vector>

namespace {

ggml_backend_t g_cpu = nullptr;
int g_threads = 1;

ggml_backend_t cpu() {
    if (!g_cpu) {
        g_cpu = ggml_backend_cpu_init();
        ggml_backend_cpu_set_n_threads(g_cpu, g_threads);
    }
    return g_cpu;
}

struct Graph {
    ggml_context * ctx = nullptr;
    ggml_backend_buffer_t buf = nullptr;
    std::vector<ggml_backend_buffer_t> user_bufs;
    ggml_cgraph * gf = nullptr;

    explicit Graph(size_t n_tensors = 512) {
        ggml_init_params p = { ggml_tensor_overhead() * n_tensors + ggml_graph_overhead_custom(4096, false), nullptr, true };
        ctx = ggml_init(p);
        gf = ggml_new_graph_custom(ctx, 4096, false);
    }
    ~Graph() {
        if (buf) ggml_backend_buffer_free(buf);
        for (auto b : user_bufs) ggml_backend_buffer_free(b);
        if (ctx) ggml_free(ctx);
    }
    // wrap caller memory (weights) without copying when it meets ggml's 32-byte tensor
    // alignment; otherwise the tensor is allocated with the rest and copied in
    std::vector<std::pair<ggml_tensor *, const void *>> copies;
    void bind(ggml_tensor * t, const void * ptr) {
        if (((uintptr_t) ptr) % 32 != 0) { copies.emplace_back(t, ptr); return; }
        ggml_backend_buffer_t b = ggml_backend_cpu_buffer_from_ptr(const_cast<void *>(ptr), ggml_nbytes(t));
        ggml_backend_tensor_alloc(b, t, const_cast<void *>(ptr));
        user_bufs.push_back(b);
    }
    void alloc_rest() {
        buf = ggml_backend_alloc_ctx_tensors(ctx, cpu());
        for (auto & c : copies) ggml_backend_tensor_set(c.first, c.second, 0, ggml_nbytes(c.first));
    }
    // one untimed evaluation (also the result for iters == 0), then `iters` timed ones;
    // returns the mean ms and keeps each evaluation's ms for qref_last_times
    double compute(int iters);
};

std::vector<double> g_last_times;

double Graph::compute(int iters) {
    ggml_backend_graph_compute(cpu(), gf);
    g_last_times.clear();
    if (iters <= 0) return 0.0;
    double total = 0.0;
    for (int i = 0; i < iters; ++i) {
        auto t0 = std::chrono::steady_clock::now();
        ggml_backend_graph_compute(cpu(), gf);
        auto t1 = std::chrono::steady_clock::now();
        g_last_times.push_back(std::chrono::duration<double, std::milli>(t1 - t0).count());
        total += g_last_times.back();
    }
    return total / iters;
}

}  // namespace

extern "C" {

// per-evaluation ms of the last timed call (at most n copied); returns how many it holds
int qref_last_times(double * out, int n) {
    const int have = (int) g_last_times.size();
    for (int i = 0; i < have && i < n; ++i) out[i] = g_last_times[i];
    return have;
}

void qref_set_threads(int n) {
    g_threads = n > 0 ? n : 1;
    if (g_cpu) ggml_backend_cpu_set_n_threads(g_cpu, g_threads);
}

size_t qref_row_size(int type, int64_t n) { return ggml_row_size((ggml_type) type, n); }

// Weight creation exactly as a GGUF converter would: ggml_quantize_chunk (ggml.c:8079),
// no importance matrix (=> the *_ref quantizers).
size_t qref_quantize(int type, const float * src, void * dst, int64_t nrow, int64_t n_per_row) {
    ggml_quantize_init((ggml_type) type);
    return ggml_quantize_chunk((ggml_type) type, src, dst, 0, nrow, n_per_row, nullptr);
}

// The CPU backend's activation quantizer: type_traits_cpu[vec_dot_type].from_float
// (ggml-cpu.c:1609-1644 calls it on src1 rows).  Q8_K -> quantize_row_q8_K,
// Q8_0 -> the x86 SIMD quantize_row_q8_0 (arch/x86/quants.c:302).
int qref_from_float(int type, const float * x, void * y, int64_t nrow, int64_t k) {
    const ggml_type_traits_cpu * tr = ggml_get_type_traits_cpu((ggml_type) type);
    if (!tr || !tr->from_float) return -1;
    const size_t rs = ggml_row_size((ggml_type) type, k);
    for (int64_t r = 0; r < nrow; ++r) tr->from_float(x + r * k, (char *) y + r * rs, k);
    return 0;
}

// Plain dequantize (ggml_get_type_traits(type)->to_float).
int qref_to_float(int type, const void * x, float * y, int64_t nrow, int64_t k) {
    const ggml_type_traits * tr = ggml_get_type_traits((ggml_type) type);
    if (!tr || !tr->to_float) return -1;
    const size_t rs = ggml_row_size((ggml_type) type, k);
    for (int64_t r = 0; r < nrow; ++r) tr->to_float((const char *) x + r * rs, y + r * k, k);
    return 0;
}

// dst[M, n_used, T] = mul_mat_id(as[K, M, n_as], b[K, n_b, T], ids[n_used, T])
// ids_stride: elements between consecutive tokens in ids (>= n_used; a strided view
// like argsort_top_k's when > n_used).
double qref_mul_mat_id(int type, const void * as, int64_t K, int64_t M, int64_t n_as,
                       const float * b, int64_t n_b, int64_t T,
                       const int32_t * ids, int64_t n_used, int64_t ids_stride,
                       float * dst, int iters) {
    Graph g;
    ggml_tensor * tas  = ggml_new_tensor_3d(g.ctx, (ggml_type) type, K, M, n_as);
    ggml_tensor * tb   = ggml_new_tensor_3d(g.ctx, GGML_TYPE_F32, K, n_b, T);
    ggml_tensor * tidf = ggml_new_tensor_2d(g.ctx, GGML_TYPE_I32, ids_stride, T);
    ggml_tensor * tid  = ggml_view_2d(g.ctx, tidf, n_used, T, tidf->nb[1], 0);
    ggml_tensor * out  = ggml_mul_mat_id(g.ctx, tas, tb, tid);
    ggml_build_forward_expand(g.gf, out);
    g.bind(tas, as);
    g.alloc_rest();
    ggml_backend_tensor_set(tb, b, 0, ggml_nbytes(tb));
    ggml_backend_tensor_set(tidf, ids, 0, ggml_nbytes(tidf));
    double ms = g.compute(iters);
    ggml_backend_tensor_get(out, dst, 0, ggml_nbytes(out));
    return ms;
}

// dst[ne0, n] = get_rows(src[ne0, nrows] of `type`, idx[n]); dst type F32 (or I32 for I32 src)
double qref_get_rows(int type, const void * src, int64_t ne0, int64_t nrows,
                     const int32_t * idx, int64_t n, void * dst, int iters) {
    Graph g;
    ggml_tensor * ts = ggml_new_tensor_2d(g.ctx, (ggml_type) type, ne0, nrows);
    ggml_tensor * ti = ggml_new_tensor_1d(g.ctx, GGML_TYPE_I32, n);
    ggml_tensor * out = ggml_get_rows(g.ctx, ts, ti);
    ggml_build_forward_expand(g.gf, out);
    g.bind(ts, src);
    g.alloc_rest();
    ggml_backend_tensor_set(ti, idx, 0, ggml_nbytes(ti));
    double ms = g.compute(iters);
    ggml_backend_tensor_get(out, dst, 0, ggml_nbytes(out));
    return ms;
}

// dst[M, T] = mul_mat(a[K, M] of `type`, b[K, T] f32): ggml_mul_mat (ggml.c:3362) on the
// CPU backend, as the dense FFN / shared expert / output head (runtime.cpp:2825-2833, 3037)
double qref_mul_mat(int type, const void * a, int64_t K, int64_t M, const float * b, int64_t T,
                    float * dst, int iters) {
    Graph g;
    ggml_tensor * ta  = ggml_new_tensor_2d(g.ctx, (ggml_type) type, K, M);
    ggml_tensor * tb  = ggml_new_tensor_2d(g.ctx, GGML_TYPE_F32, K, T);
    ggml_tensor * out = ggml_mul_mat(g.ctx, ta, tb);
    ggml_build_forward_expand(g.gf, out);
    g.bind(ta, a);
    g.alloc_rest();
    ggml_backend_tensor_set(tb, b, 0, ggml_nbytes(tb));
    double ms = g.compute(iters);
    ggml_backend_tensor_get(out, dst, 0, ggml_nbytes(out));
    return ms;
}

// route_experts (runtime.cpp:2693-2734) on given logits [E, T]:
// selected[n_used, T] i32, weights[n_used, T] f32 (renormalised when norm != 0).
double qref_route(const float * logits, int64_t E, int64_t T, int64_t n_used, int norm,
                  float scale, const float * mask, int32_t * selected, float * weights, int iters) {
    Graph g;
    ggml_tensor * tl = ggml_new_tensor_2d(g.ctx, GGML_TYPE_F32, E, T);
    ggml_tensor * tm = mask ? ggml_new_tensor_2d(g.ctx, GGML_TYPE_F32, E, T) : nullptr;
    ggml_tensor * lg = tm ? ggml_add(g.ctx, tl, tm) : tl;
    ggml_tensor * probs = ggml_soft_max(g.ctx, lg);
    ggml_tensor * sel = ggml_argsort_top_k(g.ctx, probs, n_used);
    ggml_tensor * p3 = ggml_reshape_3d(g.ctx, probs, 1, E, T);
    ggml_tensor * w = ggml_get_rows(g.ctx, p3, sel);
    if (norm) {
        w = ggml_reshape_2d(g.ctx, w, n_used, T);
        ggml_tensor * ws = ggml_sum_rows(g.ctx, w);
        ws = ggml_clamp(g.ctx, ws, 6.103515625e-5f, INFINITY);
        w = ggml_div(g.ctx, w, ws);
        w = ggml_reshape_3d(g.ctx, w, 1, n_used, T);
    }
    if (scale != 0.0f && scale != 1.0f) w = ggml_scale(g.ctx, w, scale);
    ggml_tensor * selc = ggml_cont(g.ctx, sel);
    ggml_build_forward_expand(g.gf, w);
    ggml_build_forward_expand(g.gf, selc);
    g.alloc_rest();
    ggml_backend_tensor_set(tl, logits, 0, ggml_nbytes(tl));
    if (tm) ggml_backend_tensor_set(tm, mask, 0, ggml_nbytes(tm));
    double ms = g.compute(iters);
    ggml_backend_tensor_get(selc, selected, 0, ggml_nbytes(selc));
    ggml_backend_tensor_get(w, weights, 0, ggml_nbytes(w));
    return ms;
}

// One MoE FFN layer as build_moe emits it (runtime.cpp:2743-2816), resident branch
// (expert ids used directly) or, when g2s != NULL, the slot-remap branch where each of
// gate/up/down gathers its slot ids through an I32 [1, E] table (runtime.cpp:2769-2778)
// and the expert tensors are slot pools [.., .., n_slots].
//   x        [H, T] f32            router_w [H, E] f32
//   gate/up  [H, F, n_mat] (type_gu)   down [F, H, n_mat] (type_d)
//   g2s      3 x E int32 (gate, up, down tables) or NULL
// outputs: out [H, T], selected [n_used, T], weights [n_used, T]; optional act [F, n_used, T].
// Shared expert of a layer (core/runtime.cpp:2825-2833), or type -1 / null pointers.
struct SharedExpert {
    const void * gate, * up, * down;  // [H, Fs], [H, Fs], [Fs, H] of the routed gate/up, down types
    int64_t Fs;
    const float * gate_inp;           // [H] or null
};

static double moe_layer_graph(const float * x, int64_t H, int64_t T,
                              const float * router_w, int64_t E, int64_t n_used,
                              int type_gu, const void * gate, const void * up,
                              int type_d, const void * down, int64_t F, int64_t n_mat,
                              const int32_t * g2s, const float * mask,
                              float * out, int32_t * selected, float * weights, float * act_out,
                              int iters, const float * norm_w, float norm_eps, const SharedExpert * sh) {
    Graph g(1024);
    ggml_context * ctx = g.ctx;
    ggml_tensor * tx  = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, H, T);
    ggml_tensor * trw = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, H, E);
    ggml_tensor * tg  = ggml_new_tensor_3d(ctx, (ggml_type) type_gu, H, F, n_mat);
    ggml_tensor * tu  = ggml_new_tensor_3d(ctx, (ggml_type) type_gu, H, F, n_mat);
    ggml_tensor * td  = ggml_new_tensor_3d(ctx, (ggml_type) type_d, F, H, n_mat);
    ggml_tensor * tm  = mask ? ggml_new_tensor_2d(ctx, GGML_TYPE_F32, E, T) : nullptr;
    ggml_tensor * tg2s = g2s ? ggml_new_tensor_3d(ctx, GGML_TYPE_I32, 1, E, 3) : nullptr;
    ggml_tensor * tnw = norm_w ? ggml_new_tensor_1d(ctx, GGML_TYPE_F32, H) : nullptr;

    // ffn_in = rms_norm(cur) * ffn_norm.weight (core/runtime.cpp:2979)
    ggml_tensor * xin = tnw ? ggml_mul(ctx, ggml_rms_norm(ctx, tx, norm_eps), tnw) : tx;
    ggml_tensor * logits = ggml_mul_mat(ctx, trw, xin);  // [E, T]
    if (tm) logits = ggml_add(ctx, logits, tm);
    ggml_tensor * probs = ggml_soft_max(ctx, logits);
    ggml_tensor * sel = ggml_argsort_top_k(ctx, probs, n_used);
    ggml_tensor * p3 = ggml_reshape_3d(ctx, probs, 1, E, T);
    ggml_tensor * w = ggml_get_rows(ctx, p3, sel);
    w = ggml_reshape_2d(ctx, w, n_used, T);
    ggml_tensor * ws = ggml_sum_rows(ctx, w);
    ws = ggml_clamp(ctx, ws, 6.103515625e-5f, INFINITY);
    w = ggml_div(ctx, w, ws);
    w = ggml_reshape_3d(ctx, w, 1, n_used, T);
    ggml_build_forward_expand(g.gf, w);

    ggml_tensor *ids_g = sel, *ids_u = sel, *ids_d = sel;
    if (tg2s) {
        auto remap = [&](int role) {
            ggml_tensor * tab = ggml_view_2d(ctx, tg2s, 1, E, tg2s->nb[1], (size_t) role * tg2s->nb[2]);
            ggml_tensor * s = ggml_get_rows(ctx, tab, sel);  // [1, n_used, T] i32
            return ggml_reshape_2d(ctx, s, n_used, T);
        };
        ids_g = remap(0); ids_u = remap(1); ids_d = remap(2);
    }
    ggml_tensor * x3 = ggml_reshape_3d(ctx, xin, H, 1, T);
    ggml_tensor * tup   = ggml_mul_mat_id(ctx, tu, x3, ids_u);
    ggml_tensor * tgate = ggml_mul_mat_id(ctx, tg, x3, ids_g);
    ggml_tensor * act = ggml_swiglu_split(ctx, tgate, tup);  // [F, n_used, T]
    ggml_tensor * experts = ggml_mul_mat_id(ctx, td, act, ids_d);  // [H, n_used, T]
    ggml_tensor * moe;
    if (T == 1) {
        ggml_tensor * et = ggml_cont(ctx, ggml_transpose(ctx, ggml_reshape_2d(ctx, experts, H, n_used)));
        ggml_tensor * w2 = ggml_reshape_2d(ctx, w, n_used, 1);
        moe = ggml_mul_mat(ctx, et, w2);
    } else {
        experts = ggml_mul(ctx, experts, w);
        ggml_build_forward_expand(g.gf, experts);
        moe = ggml_view_2d(ctx, experts, H, T, experts->nb[2], 0);
        for (int64_t i = 1; i < n_used; ++i) {
            ggml_tensor * v = ggml_view_2d(ctx, experts, H, T, experts->nb[2], (size_t) i * experts->nb[1]);
            moe = ggml_add(ctx, moe, v);
        }
        if (n_used == 1) moe = ggml_cont(ctx, moe);
    }
    // shared expert, added to the routed sum (core/runtime.cpp:2825-2833)
    ggml_tensor *tsg = nullptr, *tsu = nullptr, *tsd = nullptr, *tsi = nullptr;
    if (sh) {
        tsg = ggml_new_tensor_2d(ctx, (ggml_type) type_gu, H, sh->Fs);
        tsu = ggml_new_tensor_2d(ctx, (ggml_type) type_gu, H, sh->Fs);
        tsd = ggml_new_tensor_2d(ctx, (ggml_type) type_d, sh->Fs, H);
        ggml_tensor * gs = ggml_mul_mat(ctx, tsg, xin);
        ggml_tensor * us = ggml_mul_mat(ctx, tsu, xin);
        ggml_tensor * shv = ggml_mul_mat(ctx, tsd, ggml_mul(ctx, ggml_silu(ctx, gs), us));
        if (sh->gate_inp) {
            tsi = ggml_new_tensor_1d(ctx, GGML_TYPE_F32, H);
            shv = ggml_mul(ctx, shv, ggml_sigmoid(ctx, ggml_mul_mat(ctx, tsi, xin)));
        }
        moe = ggml_add(ctx, moe, shv);
    }
    ggml_tensor * selc = ggml_cont(ctx, sel);
    ggml_build_forward_expand(g.gf, moe);
    ggml_build_forward_expand(g.gf, selc);
    if (act_out) ggml_build_forward_expand(g.gf, act);

    g.bind(tg, gate); g.bind(tu, up); g.bind(td, down);
    if (sh) { g.bind(tsg, sh->gate); g.bind(tsu, sh->up); g.bind(tsd, sh->down); }
    g.alloc_rest();
    if (tsi) ggml_backend_tensor_set(tsi, sh->gate_inp, 0, ggml_nbytes(tsi));
    ggml_backend_tensor_set(tx, x, 0, ggml_nbytes(tx));
    ggml_backend_tensor_set(trw, router_w, 0, ggml_nbytes(trw));
    if (tm) ggml_backend_tensor_set(tm, mask, 0, ggml_nbytes(tm));
    if (tg2s) ggml_backend_tensor_set(tg2s, g2s, 0, ggml_nbytes(tg2s));
    if (tnw) ggml_backend_tensor_set(tnw, norm_w, 0, ggml_nbytes(tnw));
    double ms = g.compute(iters);
    ggml_backend_tensor_get(moe, out, 0, ggml_nbytes(moe));
    if (selected) ggml_backend_tensor_get(selc, selected, 0, ggml_nbytes(selc));
    if (weights) ggml_backend_tensor_get(w, weights, 0, ggml_nbytes(w));
    if (act_out) ggml_backend_tensor_get(act, act_out, 0, ggml_nbytes(act));
    return ms;
}

double qref_moe_layer(const float * x, int64_t H, int64_t T,
                      const float * router_w, int64_t E, int64_t n_used,
                      int type_gu, const void * gate, const void * up,
                      int type_d, const void * down, int64_t F, int64_t n_mat,
                      const int32_t * g2s, const float * mask,
                      float * out, int32_t * selected, float * weights, float * act_out,
                      int iters, const float * norm_w, float norm_eps) {
    return moe_layer_graph(x, H, T, router_w, E, n_used, type_gu, gate, up, type_d, down, F, n_mat, g2s, mask, out,
                           selected, weights, act_out, iters, norm_w, norm_eps, nullptr);
}

// the layer with a shared expert (sh_gate_inp may be null)
double qref_moe_layer_shexp(const float * x, int64_t H, int64_t T,
                            const float * router_w, int64_t E, int64_t n_used,
                            int type_gu, const void * gate, const void * up,
                            int type_d, const void * down, int64_t F, int64_t n_mat,
                            const float * norm_w, float norm_eps,
                            const void * sh_gate, const void * sh_up, const void * sh_down, int64_t Fs,
                            const float * sh_gate_inp, float * out, int32_t * selected, float * weights) {
    const SharedExpert sh{sh_gate, sh_up, sh_down, Fs, sh_gate_inp};
    return moe_layer_graph(x, H, T, router_w, E, n_used, type_gu, gate, up, type_d, down, F, n_mat, nullptr, nullptr,
                           out, selected, weights, nullptr, 0, norm_w, norm_eps, &sh);
}

// ------------------------------------------------------------------------------------
// Drop-in checks: the same ggml graphs computed by a backend that ggml loads itself from
// a shared library (ggml_backend_load, the path of ggml_backend_load_all()).  The tensors
// are allocated in that backend's buffer type, exactly as a host application would.
// Return 0 on success; -1 the library did not load, -2 it has no device, -3 the backend
// did not initialise, -4 an allocation failed, -5 the graph failed to compute.

static ggml_backend_reg_t load_backend_once(const char * path) {
    static std::map<std::string, ggml_backend_reg_t> loaded;
    auto it = loaded.find(path);
    if (it != loaded.end()) return it->second;
    ggml_backend_reg_t reg = ggml_backend_load(path);
    loaded[path] = reg;
    return reg;
}

static ggml_backend_t backend_open(const char * path, int * rc, const char * params = "workspace_mb=512") {
    ggml_backend_reg_t reg = load_backend_once(path);
    if (!reg) { *rc = -1; return nullptr; }
    if (ggml_backend_reg_dev_count(reg) == 0) { *rc = -2; return nullptr; }
    ggml_backend_t be = ggml_backend_dev_init(ggml_backend_reg_dev_get(reg, 0), params);
    *rc = be ? 0 : -3;
    return be;
}

// Weights in one buffer marked as weights (the model loader marks expert buffers so,
// core/model.cpp:244); everything else in a second buffer of the same backend.
struct BackendGraph {
    ggml_context * wctx = nullptr, * ctx = nullptr;
    ggml_backend_buffer_t wbuf = nullptr, buf = nullptr;
    ggml_cgraph * gf = nullptr;
    BackendGraph() {
        ggml_init_params wp = {ggml_tensor_overhead() * 4, nullptr, true};
        wctx = ggml_init(wp);
        ggml_init_params ip = {ggml_tensor_overhead() * 16 + ggml_graph_overhead(), nullptr, true};
        ctx = ggml_init(ip);
        gf = ggml_new_graph(ctx);
    }
    bool alloc(ggml_backend_t be) {
        ggml_backend_buffer_type_t bt = ggml_backend_get_default_buffer_type(be);
        wbuf = ggml_backend_alloc_ctx_tensors_from_buft(wctx, bt);
        if (!wbuf) return false;
        ggml_backend_buffer_set_usage(wbuf, GGML_BACKEND_BUFFER_USAGE_WEIGHTS);
        buf = ggml_backend_alloc_ctx_tensors_from_buft(ctx, bt);
        return buf != nullptr;
    }
    ~BackendGraph() {
        if (buf) ggml_backend_buffer_free(buf);
        if (wbuf) ggml_backend_buffer_free(wbuf);
        ggml_free(ctx);
        ggml_free(wctx);
    }
};

// qref_mul_mat_id computed by the backend in `path`.
int qref_backend_mul_mat_id(const char * path, int type, const void * as, int64_t K, int64_t M, int64_t n_as,
                            const float * b, int64_t n_b, int64_t T, const int32_t * ids, int64_t n_used,
                            int64_t ids_stride, float * dst) {
    int rc = 0;
    ggml_backend_t be = backend_open(path, &rc);
    if (!be) return rc;
    {
        BackendGraph g;
        ggml_tensor * tas  = ggml_new_tensor_3d(g.wctx, (ggml_type) type, K, M, n_as);
        ggml_tensor * tb   = ggml_new_tensor_3d(g.ctx, GGML_TYPE_F32, K, n_b, T);
        ggml_tensor * tidf = ggml_new_tensor_2d(g.ctx, GGML_TYPE_I32, ids_stride, T);
        ggml_tensor * tid  = ggml_view_2d(g.ctx, tidf, n_used, T, tidf->nb[1], 0);
        ggml_tensor * out  = ggml_mul_mat_id(g.ctx, tas, tb, tid);
        ggml_build_forward_expand(g.gf, out);
        if (!g.alloc(be)) {
            rc = -4;
        } else {
            ggml_backend_tensor_set(tas, as, 0, ggml_nbytes(tas));
            ggml_backend_tensor_set(tb, b, 0, ggml_nbytes(tb));
            ggml_backend_tensor_set(tidf, ids, 0, ggml_nbytes(tidf));
            if (ggml_backend_graph_compute(be, g.gf) != GGML_STATUS_SUCCESS) rc = -5;
            else ggml_backend_tensor_get(out, dst, 0, ggml_nbytes(out));
        }
    }
    ggml_backend_free(be);
    return rc;
}

// qref_mul_mat computed by the backend in `path`.
int qref_backend_mul_mat(const char * path, int type, const void * a, int64_t K, int64_t M, const float * b,
                         int64_t T, float * dst) {
    int rc = 0;
    ggml_backend_t be = backend_open(path, &rc);
    if (!be) return rc;
    {
        BackendGraph g;
        ggml_tensor * ta  = ggml_new_tensor_2d(g.wctx, (ggml_type) type, K, M);
        ggml_tensor * tb  = ggml_new_tensor_2d(g.ctx, GGML_TYPE_F32, K, T);
        ggml_tensor * out = ggml_mul_mat(g.ctx, ta, tb);
        ggml_build_forward_expand(g.gf, out);
        if (!g.alloc(be)) {
            rc = -4;
        } else {
            ggml_backend_tensor_set(ta, a, 0, ggml_nbytes(ta));
            ggml_backend_tensor_set(tb, b, 0, ggml_nbytes(tb));
            if (ggml_backend_graph_compute(be, g.gf) != GGML_STATUS_SUCCESS) rc = -5;
            else ggml_backend_tensor_get(out, dst, 0, ggml_nbytes(out));
        }
    }
    ggml_backend_free(be);
    return rc;
}

// qref_get_rows computed by the backend in `path`.
int qref_backend_get_rows(const char * path, int type, const void * src, int64_t ne0, int64_t nrows,
                          const int32_t * idx, int64_t n, void * dst) {
    int rc = 0;
    ggml_backend_t be = backend_open(path, &rc);
    if (!be) return rc;
    {
        BackendGraph g;
        ggml_tensor * ts = ggml_new_tensor_2d(g.wctx, (ggml_type) type, ne0, nrows);
        ggml_tensor * ti = ggml_new_tensor_1d(g.ctx, GGML_TYPE_I32, n);
        ggml_tensor * out = ggml_get_rows(g.ctx, ts, ti);
        ggml_build_forward_expand(g.gf, out);
        if (!g.alloc(be)) {
            rc = -4;
        } else {
            ggml_backend_tensor_set(ts, src, 0, ggml_nbytes(ts));
            ggml_backend_tensor_set(ti, idx, 0, ggml_nbytes(ti));
            if (ggml_backend_graph_compute(be, g.gf) != GGML_STATUS_SUCCESS) rc = -5;
            else ggml_backend_tensor_get(out, dst, 0, ggml_nbytes(out));
        }
    }
    ggml_backend_free(be);
    return rc;
}

// scale * mul_mat_id(as, b, ids) through ggml_backend_sched over [backend in `path`, CPU]:
// the weights sit in the loaded backend's weight buffer, b and ids are CPU inputs, and
// the scale is an op the loaded backend does not implement.  Reports the number of
// splits and whether the scheduler put MUL_MAT_ID on the loaded backend.
int qref_backend_sched_mul_mat_id(const char * path, int type, const void * as, int64_t K, int64_t M,
                                  int64_t n_as, const float * b, int64_t T, const int32_t * ids, int64_t n_used,
                                  float scale, float * dst, int * n_splits, int * mmid_on_backend) {
    int rc = 0;
    ggml_backend_t be = backend_open(path, &rc);
    if (!be) return rc;
    ggml_backend_t cb = ggml_backend_cpu_init();
    ggml_init_params wp = {ggml_tensor_overhead() * 2, nullptr, true};
    ggml_context * wctx = ggml_init(wp);
    ggml_tensor * ta = ggml_new_tensor_3d(wctx, (ggml_type) type, K, M, n_as);
    ggml_backend_buffer_t wbuf = ggml_backend_alloc_ctx_tensors_from_buft(wctx, ggml_backend_get_default_buffer_type(be));
    ggml_context * ctx = nullptr;
    ggml_backend_sched_t sched = nullptr;
    if (!wbuf) {
        rc = -4;
    } else {
        ggml_backend_buffer_set_usage(wbuf, GGML_BACKEND_BUFFER_USAGE_WEIGHTS);
        ggml_backend_tensor_set(ta, as, 0, ggml_nbytes(ta));
        ggml_init_params ip = {ggml_tensor_overhead() * 16 + ggml_graph_overhead(), nullptr, true};
        ctx = ggml_init(ip);
        ggml_tensor * tb = ggml_new_tensor_3d(ctx, GGML_TYPE_F32, K, 1, T);
        ggml_tensor * tids = ggml_new_tensor_2d(ctx, GGML_TYPE_I32, n_used, T);
        ggml_set_input(tb);
        ggml_set_input(tids);
        ggml_tensor * y = ggml_mul_mat_id(ctx, ta, tb, tids);
        ggml_tensor * z = ggml_scale(ctx, y, scale);
        ggml_set_output(z);
        ggml_cgraph * gf = ggml_new_graph(ctx);
        ggml_build_forward_expand(gf, z);
        ggml_backend_t bes[2] = {be, cb};
        sched = ggml_backend_sched_new(bes, nullptr, 2, GGML_DEFAULT_GRAPH_SIZE, false, true);
        if (!ggml_backend_sched_alloc_graph(sched, gf)) {
            rc = -4;
        } else {
            ggml_backend_tensor_set(tb, b, 0, ggml_nbytes(tb));
            ggml_backend_tensor_set(tids, ids, 0, ggml_nbytes(tids));
            if (ggml_backend_sched_graph_compute(sched, gf) != GGML_STATUS_SUCCESS) rc = -5;
            ggml_backend_sched_synchronize(sched);
            *n_splits = ggml_backend_sched_get_n_splits(sched);
            *mmid_on_backend = ggml_backend_sched_get_tensor_backend(sched, y) == be;
            if (rc == 0) ggml_backend_tensor_get(z, dst, 0, ggml_nbytes(z));
        }
    }
    if (sched) ggml_backend_sched_free(sched);
    if (ctx) ggml_free(ctx);
    if (wbuf) ggml_backend_buffer_free(wbuf);
    ggml_free(wctx);
    ggml_backend_free(cb);
    ggml_backend_free(be);
    return rc;
}


// ------------------------------------------------------------------------------------
// A stack of L decoder MoE FFN blocks as QuestWend builds them (core/runtime.cpp:
// 2972-2993 around build_moe :2743-2816):
//     cur = scale(cur, 1) (a stand-in for the attention block: an op outside the MoE path)
//     ffn_in = rms_norm(cur) * ffn_norm;  cur = build_moe(ffn_in) + cur
// computed by the backend library at `path` (ggml_backend_load), or by the CPU backend
// when path is NULL.  Graph tensors are placed by ggml's graph allocator (gallocr, with
// memory reuse, as QuestWend's runtime does); weights sit in a buffer marked as weights.
//   expert matrices: n_unique distinct byte images per role; expert e of layer l is image
//     (e + l) % n_unique (gate/up [H, F] type_gu, down [F, H] type_d)
//   g2s == NULL: the resident branch, T tokens, expert tensors [.., .., E]
//   g2s != NULL: the expert-cache branch (T = 1): slot pools [.., .., n_slots], one I32
//     table per (layer, role) in g2s_all [1, E, 3L] (g2s: [L][3][E]), and every layer's
//     selection copied into sel_all [n_used, L] (read back into `selected`)
// router_w [L][E][H], norm_w [L][H], x [T][H] -> out [T][H].  Runs the graph once, then
// `iters` timed times (synchronised each time, the input set before each, outside the
// timing): *ms = mean ms per run.  stats (5 values,
// may be NULL): the QWB backend's counters (fused layers, own nodes, delegated nodes,
// delegated runs) and whether it delegates, all zero for other backends.
// Optional shared expert for qref_backend_moe_stack (core/runtime.cpp:2825-2833): one
// byte image per matrix (the same for every layer; gate/up of the routed gate/up type
// [H, Fs], down of the routed down type [Fs, H]) and a sigmoid gate weight per layer
// ([L][H], or null for none).  qref_stack_set_shexp(nullptr, ...) removes it.
static struct {
    const void * gate = nullptr, * up = nullptr, * down = nullptr;
    int64_t Fs = 0;
    const float * gate_inp = nullptr;
} g_stack_sh;

void qref_stack_set_shexp(const void * gate, const void * up, const void * down, int64_t Fs, const float * gate_inp) {
    g_stack_sh.gate = gate;
    g_stack_sh.up = up;
    g_stack_sh.down = down;
    g_stack_sh.Fs = down ? Fs : 0;
    g_stack_sh.gate_inp = down ? gate_inp : nullptr;
}

int qref_backend_moe_stack(const char * path, const char * params, int L, int64_t H, int64_t F, int64_t E,
                           int64_t n_used, int64_t T, int type_gu, const void * gate_u, const void * up_u,
                           int type_d, const void * down_u, int64_t n_unique, const float * router_w,
                           const float * norm_w, const float * x, const int32_t * g2s, int64_t n_slots,
                           float * out, int32_t * selected, int iters, double * ms, uint64_t * stats) {
    int rc = 0;
    ggml_backend_t be = nullptr;
    ggml_backend_reg_t reg = nullptr;
    if (path) {
        be = backend_open(path, &rc, params ? params : "workspace_mb=512");
        if (!be) return rc;
        reg = load_backend_once(path);
    } else {
        be = ggml_backend_cpu_init();
        ggml_backend_cpu_set_n_threads(be, g_threads);
    }
    const bool cache = g2s != nullptr;
    if (cache && T != 1) { ggml_backend_free(be); return -6; }
    const int64_t NE = cache ? n_slots : E;
    const size_t rb_gu = ggml_row_size((ggml_type) type_gu, H), rb_d = ggml_row_size((ggml_type) type_d, F);
    const size_t ex_gu = rb_gu * F, ex_d = rb_d * H;

    ggml_init_params wp = {ggml_tensor_overhead() * (7 * (size_t) L + 8), nullptr, true};
    ggml_context * wctx = ggml_init(wp);
    std::vector<ggml_tensor *> tg(L), tu(L), td(L), trw(L), tnw(L), tsi(L, nullptr);
    const bool sh = g_stack_sh.down != nullptr;
    ggml_tensor * tsg = sh ? ggml_new_tensor_2d(wctx, (ggml_type) type_gu, H, g_stack_sh.Fs) : nullptr;
    ggml_tensor * tsu = sh ? ggml_new_tensor_2d(wctx, (ggml_type) type_gu, H, g_stack_sh.Fs) : nullptr;
    ggml_tensor * tsd = sh ? ggml_new_tensor_2d(wctx, (ggml_type) type_d, g_stack_sh.Fs, H) : nullptr;
    if (sh && g_stack_sh.gate_inp)
        for (int l = 0; l < L; ++l) tsi[l] = ggml_new_tensor_1d(wctx, GGML_TYPE_F32, H);
    for (int l = 0; l < L; ++l) {
        tg[l] = ggml_new_tensor_3d(wctx, (ggml_type) type_gu, H, F, NE);
        tu[l] = ggml_new_tensor_3d(wctx, (ggml_type) type_gu, H, F, NE);
        td[l] = ggml_new_tensor_3d(wctx, (ggml_type) type_d, F, H, NE);
        trw[l] = ggml_new_tensor_2d(wctx, GGML_TYPE_F32, H, E);
        tnw[l] = ggml_new_tensor_1d(wctx, GGML_TYPE_F32, H);
    }
    ggml_tensor * g2s_all = cache ? ggml_new_tensor_3d(wctx, GGML_TYPE_I32, 1, E, 3 * L) : nullptr;
    ggml_tensor * sel_all = cache ? ggml_new_tensor_2d(wctx, GGML_TYPE_I32, n_used, L) : nullptr;
    ggml_backend_buffer_type_t bt = ggml_backend_get_default_buffer_type(be);
    ggml_backend_buffer_t wbuf = ggml_backend_alloc_ctx_tensors_from_buft(wctx, bt);
    ggml_context * ctx = nullptr;
    ggml_gallocr_t galloc = nullptr;
    if (!wbuf) {
        rc = -4;
    } else {
        ggml_backend_buffer_set_usage(wbuf, GGML_BACKEND_BUFFER_USAGE_WEIGHTS);
        const uint8_t * img[3] = {(const uint8_t *) gate_u, (const uint8_t *) up_u, (const uint8_t *) down_u};
        for (int l = 0; l < L; ++l) {
            for (int64_t s = 0; s < NE; ++s) {
                // slot s holds expert e: the identity, or the expert the layer's table sends to s
                int64_t e = s;
                if (cache)
                    for (int64_t k = 0; k < E; ++k)
                        if (g2s[((size_t) l * 3 + 0) * E + k] == s) e = k;
                const int64_t u = (e + l) % n_unique;
                ggml_backend_tensor_set(tg[l], img[0] + u * ex_gu, s * ex_gu, ex_gu);
                ggml_backend_tensor_set(tu[l], img[1] + u * ex_gu, s * ex_gu, ex_gu);
                ggml_backend_tensor_set(td[l], img[2] + u * ex_d, s * ex_d, ex_d);
            }
            ggml_backend_tensor_set(trw[l], router_w + (size_t) l * E * H, 0, ggml_nbytes(trw[l]));
            ggml_backend_tensor_set(tnw[l], norm_w + (size_t) l * H, 0, ggml_nbytes(tnw[l]));
        }
        if (cache) ggml_backend_tensor_set(g2s_all, g2s, 0, ggml_nbytes(g2s_all));
        if (sh) {
            ggml_backend_tensor_set(tsg, g_stack_sh.gate, 0, ggml_nbytes(tsg));
            ggml_backend_tensor_set(tsu, g_stack_sh.up, 0, ggml_nbytes(tsu));
            ggml_backend_tensor_set(tsd, g_stack_sh.down, 0, ggml_nbytes(tsd));
            for (int l = 0; l < L; ++l)
                if (tsi[l]) ggml_backend_tensor_set(tsi[l], g_stack_sh.gate_inp + (size_t) l * H, 0, ggml_nbytes(tsi[l]));
        }

        ggml_init_params ip = {ggml_tensor_overhead() * (64 * (size_t) L + 64) + ggml_graph_overhead_custom(8192, false),
                               nullptr, true};
        ctx = ggml_init(ip);
        ggml_cgraph * gf = ggml_new_graph_custom(ctx, 8192, false);
        ggml_tensor * inp = ggml_new_tensor_2d(ctx, GGML_TYPE_F32, H, T);
        ggml_set_input(inp);
        ggml_tensor * cur = inp;
        for (int l = 0; l < L; ++l) {
            // stand-in for the attention block between MoE blocks (nodes a MoE backend hands
            // on): an identity scale
            cur = ggml_scale(ctx, cur, 1.0f);
            ggml_tensor * ffn_in = ggml_mul(ctx, ggml_rms_norm(ctx, cur, 1e-6f), tnw[l]);
            // route_experts (runtime.cpp:2693-2734): softmax gating, expert_weights_norm
            ggml_tensor * logits = ggml_mul_mat(ctx, trw[l], ffn_in);
            ggml_tensor * probs = ggml_soft_max(ctx, logits);
            ggml_tensor * sel = ggml_argsort_top_k(ctx, probs, n_used);
            ggml_tensor * w = ggml_get_rows(ctx, ggml_reshape_3d(ctx, probs, 1, E, T), sel);
            w = ggml_reshape_2d(ctx, w, n_used, T);
            ggml_tensor * ws = ggml_clamp(ctx, ggml_sum_rows(ctx, w), 6.103515625e-5f, INFINITY);
            w = ggml_reshape_3d(ctx, ggml_div(ctx, w, ws), 1, n_used, T);
            ggml_build_forward_expand(gf, w);
            ggml_tensor * moe;
            if (cache) {
                ggml_tensor * sel_col = ggml_view_2d(ctx, sel_all, n_used, 1, sel_all->nb[1], (size_t) l * sel_all->nb[1]);
                ggml_build_forward_expand(gf, ggml_cpy(ctx, sel, sel_col));
                auto remap = [&](int role) {
                    const int idx = l * 3 + role;
                    ggml_tensor * tab = ggml_view_2d(ctx, g2s_all, 1, E, g2s_all->nb[1], (size_t) idx * g2s_all->nb[2]);
                    return ggml_reshape_2d(ctx, ggml_get_rows(ctx, tab, sel), n_used, 1);
                };
                ggml_tensor * sg = remap(0), * su = remap(1), * sd = remap(2);
                ggml_tensor * x3 = ggml_reshape_3d(ctx, ffn_in, H, 1, 1);
                ggml_tensor * up = ggml_mul_mat_id(ctx, tu[l], x3, su);
                ggml_tensor * gate = ggml_mul_mat_id(ctx, tg[l], x3, sg);
                ggml_tensor * act = ggml_swiglu_split(ctx, gate, up);
                ggml_tensor * experts = ggml_mul_mat_id(ctx, td[l], act, sd);
                ggml_tensor * et = ggml_cont(ctx, ggml_transpose(ctx, ggml_reshape_2d(ctx, experts, H, n_used)));
                moe = ggml_mul_mat(ctx, et, ggml_reshape_2d(ctx, w, n_used, 1));
            } else {
                ggml_tensor * x3 = ggml_reshape_3d(ctx, ffn_in, H, 1, T);
                ggml_tensor * up = ggml_mul_mat_id(ctx, tu[l], x3, sel);
                ggml_tensor * gate = ggml_mul_mat_id(ctx, tg[l], x3, sel);
                ggml_tensor * act = ggml_swiglu_split(ctx, gate, up);
                ggml_tensor * experts = ggml_mul_mat_id(ctx, td[l], act, sel);
                if (T == 1) {
                    ggml_tensor * et = ggml_cont(ctx, ggml_transpose(ctx, ggml_reshape_2d(ctx, experts, H, n_used)));
                    moe = ggml_mul_mat(ctx, et, ggml_reshape_2d(ctx, w, n_used, 1));
                } else {
                    experts = ggml_mul(ctx, experts, w);
                    ggml_build_forward_expand(gf, experts);
                    std::vector<ggml_tensor *> v(n_used);
                    for (int64_t i = 0; i < n_used; ++i) {
                        v[i] = ggml_view_2d(ctx, experts, H, T, experts->nb[2], (size_t) i * experts->nb[1]);
                        ggml_build_forward_expand(gf, v[i]);
                    }
                    moe = v[0];
                    for (int64_t i = 1; i < n_used; ++i) {
                        moe = ggml_add(ctx, moe, v[i]);
                        ggml_build_forward_expand(gf, moe);
                    }
                    if (n_used == 1) moe = ggml_cont(ctx, moe);
                }
            }
            if (sh) {
                // shared expert (runtime.cpp:2825-2833)
                ggml_tensor * gs = ggml_mul_mat(ctx, tsg, ffn_in);
                ggml_tensor * us = ggml_mul_mat(ctx, tsu, ffn_in);
                ggml_tensor * shv = ggml_mul_mat(ctx, tsd, ggml_mul(ctx, ggml_silu(ctx, gs), us));
                if (tsi[l]) shv = ggml_mul(ctx, shv, ggml_sigmoid(ctx, ggml_mul_mat(ctx, tsi[l], ffn_in)));
                moe = ggml_add(ctx, moe, shv);
            }
            cur = ggml_add(ctx, moe, cur);
        }
        ggml_set_output(cur);
        ggml_build_forward_expand(gf, cur);
        galloc = ggml_gallocr_new(bt);
        if (!ggml_gallocr_alloc_graph(galloc, gf)) {
            rc = -4;
        } else {
            ggml_backend_tensor_set(inp, x, 0, ggml_nbytes(inp));
            if (ggml_backend_graph_compute(be, gf) != GGML_STATUS_SUCCESS) rc = -5;
            ggml_backend_synchronize(be);
            double total = 0.0;
            for (int i = 0; i < iters && rc == 0; ++i) {
                // inputs are set before every compute: the graph allocator may reuse an
                // input's memory once its last reader has run
                ggml_backend_tensor_set(inp, x, 0, ggml_nbytes(inp));
                auto t0 = std::chrono::steady_clock::now();
                if (ggml_backend_graph_compute(be, gf) != GGML_STATUS_SUCCESS) rc = -5;
                ggml_backend_synchronize(be);
                total += std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
            }
            if (ms) *ms = iters > 0 ? total / iters : 0.0;
            if (rc == 0) {
                ggml_backend_tensor_get(cur, out, 0, ggml_nbytes(cur));
                if (cache && selected) ggml_backend_tensor_get(sel_all, selected, 0, ggml_nbytes(sel_all));
            }
        }
    }
    if (stats) {
        for (int k = 0; k < 5; ++k) stats[k] = 0;
        if (reg) {
            typedef int (*stats_fn)(ggml_backend_t, uint64_t *, int);
            typedef int (*deleg_fn)();
            if (auto f = (stats_fn) ggml_backend_reg_get_proc_address(reg, "ggml_backend_qwb_get_stats")) f(be, stats, 4);
            if (auto f = (deleg_fn) ggml_backend_reg_get_proc_address(reg, "ggml_backend_qwb_is_delegating")) stats[4] = f();
        }
    }
    if (galloc) ggml_gallocr_free(galloc);
    if (ctx) ggml_free(ctx);
    if (wbuf) ggml_backend_buffer_free(wbuf);
    ggml_free(wctx);
    ggml_backend_free(be);
    return rc;
}


// QuestWend's device choice (core/runtime.cpp:944-957, 996-1010) after loading every
// backend library in `dir` the way ggml_backend_load_all() does: the first GPU device
// that initialises.  Writes its name; returns 0, or -1 when no GPU device initialised.
int qref_dropin_first_gpu(const char * dir, char * name, int cap) {
    ggml_backend_load_all_from_path(dir);
    for (size_t i = 0; i < ggml_backend_dev_count(); ++i) {
        ggml_backend_dev_t dev = ggml_backend_dev_get(i);
        if (ggml_backend_dev_type(dev) != GGML_BACKEND_DEVICE_TYPE_GPU) continue;
        ggml_backend_t be = ggml_backend_dev_init(dev, nullptr);
        if (!be) continue;
        snprintf(name, (size_t) cap, "%s", ggml_backend_dev_name(dev));
        ggml_backend_free(be);
        return 0;
    }
    return -1;
}

}  // extern "C"
