// route.cuh - router / reduction launchers shared by the MoE entry points.
#pragma once

#include "common.cuh"

namespace qwb {

constexpr int kMaxUsed = 32;      // n_expert_used limit of the routing kernels
constexpr int kMaxExperts = 1024; // n_expert limit of the routing kernels
constexpr int kMaxRouterT = 16;   // tokens handled by the fused router GEMV

struct RouterArgs {
    const float *x;         // [T][H]
    const float *router_w;  // [E][H]
    const float *mask;      // [T][E] or null
    int64_t H, E, T, n_used;
    float *logits;          // [T][E] workspace
    unsigned *counter;      // workspace word, zero between launches
    int32_t *selected;      // [T][n_used]
    float *weights;         // [T][n_used]
    Q8Planes xq;            // quantized x out (qs null: skip)
    int kq;                 // 1: Q8_K planes, 0: Q8_0 planes
    int4 *tiles;            // decode tile list out (T == 1) or null
    int *pairs;
    int *n_tiles;
    const float *norm_w;    // [H] ffn_norm weight: route and quantize rms_norm(x) * norm_w
    float norm_eps;
};

cudaError_t launch_route(const float *logits, const float *mask, int64_t E, int64_t T, int64_t k, int norm,
                         float scale, int32_t *selected, float *weights, cudaStream_t s);
cudaError_t launch_router_fused(const RouterArgs &r, cudaStream_t s);
cudaError_t launch_logits_gemm(const float *x, const float *w, float *out, int64_t T, int64_t E, int64_t H,
                               cudaStream_t s);
// y[t] = rms_norm(x[t]) * w  (ggml-cpu/ops.cpp:4107-4162, fused RMS_NORM + MUL)
cudaError_t launch_rmsnorm(const float *x, const float *w, float eps, int64_t T, int64_t H, float *y, cudaStream_t s);
// out = sum_j w_j ex_j (+ sh * sh_scale, the shared expert) (+ res)
cudaError_t launch_weighted_sum(const float *ex, const float *w, const float *res, float *out, int64_t H,
                                int64_t n_used, int64_t T, cudaStream_t s, const float *sh = nullptr,
                                const float *sh_scale = nullptr);
// scale[t] = sigmoid(gw . (rms_norm(x[t]) * norm_w)) (norm_w null: gw . x[t])
cudaError_t launch_shexp_gate(const float *x, const float *norm_w, float eps, const float *gw, int64_t T, int64_t H,
                              float *scale, cudaStream_t s);

}  // namespace qwb
