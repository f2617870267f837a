// moe.cuh - pieces of the MoE layer shared by qwb_moe_ffn (moe_ffn.cu) and
// qwb_moe_ep_layer (ep.cu): the shared expert (core/runtime.cpp:2825-2833) outside the
// pair path.
#pragma once

#include "common.cuh"
#include "kernels.cuh"
#include "mmid.cuh"

namespace qwb {

// A validated shared expert; F == 0: none.
struct Shexp {
    const qwb_tensor *gate, *up, *down;
    const float *gate_inp;
    int64_t F;
};

// Checks the shared-expert operands against the routed experts' types (tg gate/up, td
// down) and the hidden size H: 2-D, contiguous rows, 16-byte aligned data.
qwb_status shexp_check(const qwb_tensor &g, const qwb_tensor &u, const qwb_tensor &d, const float *gate_inp, int tg,
                       int td, int64_t H, Shexp &sh);

// Workspace bytes of shexp_run for T tokens, and where in that workspace it leaves its
// output (sh_out may point there).
size_t shexp_bytes(const Shexp &sh, int64_t H, int64_t T);
float *shexp_out_at(const Shexp &sh, int64_t H, int64_t T, void *ws);

// The shared expert on the expert-GEMV kernels, as one expert that every token selects:
// index, gate/up GEMV with the SwiGLU epilogue (on the layer's quantized ffn_in rows xq),
// act -> Q8, down GEMV into sh_out [T][H]; and sigmoid(gate_inp . ffn_in) into sh_scale
// [T] when gate_inp is set (x and norm_w: the layer input and ffn_norm weight).
cudaError_t shexp_run(const Shexp &sh, const Q8Planes &xq, const float *x, const float *norm_w, float eps, int64_t H,
                      int64_t T, void *ws, float *sh_out, float *sh_scale, qwb_status_block *st, cudaStream_t s);

}  // namespace qwb
