// decode.cuh - the batch-1 decode MoE layer kernels (decode.cu).
#pragma once

#include "common.cuh"

namespace qwb {

// mbarrier chunks of a gate/up CTA's weight copies.  One (two bulk copies: the gate and up
// spans) beat 2-3 chunks (-4 %), 4 (-9 %) and 8 (-19 %) on the 30B-A3B decode stack: each
// bulk copy costs a fixed issue time, and starting the dots on a first chunk gains less.
constexpr int kDecodeChunks = 1;
constexpr int kDecodeThreads = 256;  // gate/up and down CTAs: 8 warps, so both fit one SM together

constexpr int kMaxRouteE = 512;     // experts the decode routing handles
constexpr int kRouterCluster = 16;  // CTAs of the decode router's thread-block cluster
constexpr int kRouterThreads = 256;

struct RouterDecodeArgs {
    const float *x;         // [T][H] layer input (residual stream)
    const float *router_w;  // [E][H]
    const float *mask;      // [T][E] or null
    const float *norm_w;    // [H] or null
    float norm_eps;
    int64_t H, E;
    int n_used;
    int T;                  // tokens: one router cluster each (1 for the batch-1 path)
    const int32_t *g2s;     // [3][E] or null
    int64_t n_slots[3];     // pool sizes (gate, up, down)
    int64_t own_lo, own_n;  // own_n > 0: expert e resolves to slot e - own_lo when it lies in
                            // [own_lo, own_lo + own_n), else to -1 without an error (an expert
                            // another GPU owns)
    int32_t *sel;           // [T][n_used] out
    float *wts;             // [T][n_used] out
    int32_t *slots;         // [3][T][n_used] out: resolved slot ids (-1: invalid / not owned)
    Q8Planes xq;            // Q8 of the normed x (T rows) out
    int kq;
    const float *sh_gate_inp;  // [H] shared-expert gate or null
    float *sh_scale;        // [T] out when set: sigmoid(sh_gate_inp . ffn_in), or 1 without a gate
    qwb_status_block *st;
};

struct GateUpDecodeArgs {
    const uint8_t *Wg, *Wu;
    size_t g_nb2, u_nb2, row_bytes;
    int64_t F, K, n_slots_g, n_slots_u;
    int n_used;
    const int32_t *slots;   // [3][n_used] from the router
    Q8Planes xq;
    float *act;             // [n_used][F]
    qwb_status_block *st;
    size_t partner_smem;    // dynamic shared memory of the down kernel launched after it (0: unknown)
};

struct DownDecodeArgs {
    const uint8_t *W;
    size_t nb2, row_bytes;
    int64_t F, H, n_slots;
    int n_used;
    const int32_t *slots;   // down slots [n_used]
    const float *wts;       // [n_used]
    const float *act;       // [n_used][F]
    float *out;             // [H]
    const float *residual;  // [H] or null
    qwb_status_block *st;
};

cudaError_t launch_router_decode(const RouterDecodeArgs &r, cudaStream_t s);

// ---- decode batches of up to kPairsMaxT tokens as lists of (token, expert) pairs: the
// routed pairs whose three slots are valid (for expert parallelism: owned by this GPU),
// in (token, slot) order, then one shared-expert pair per token when a shared expert is
// given.  Both kernels derive the same list from the router's slot ids.
constexpr int kPairsMaxT = 8;
constexpr int kPairsMaxUsed = 16;
constexpr int kPairsMax = kPairsMaxT * (kPairsMaxUsed + 1);
// routed pairs per launch (expected, for expert parallelism) up to which the pair path is
// taken for decode batches
constexpr int kPairsDirect = 16;

struct PairsCommon {
    int T, n_used;
    const int32_t *slots;     // [3][T][n_used] from the router
    const float *wts;         // [T][n_used]
    int shexp;                // 1: a shared-expert pair per token after the routed pairs
    const float *sh_scale;    // [T] or null (factor 1)
};

struct PairsGateUpArgs {
    PairsCommon pc;
    const uint8_t *Wg, *Wu;   // pools
    size_t g_nb2, u_nb2, row_bytes;
    const uint8_t *Wg_sh, *Wu_sh;  // shared expert [H, F] (same type and row size) or null
    int64_t F, K, n_slots_g, n_slots_u;
    Q8Planes xq;              // [T] rows
    float *act;               // [pairs][F]
    int batch_rows;           // row pairs per copy batch (two batches in flight)
    qwb_status_block *st;
};

struct PairsDownArgs {
    PairsCommon pc;
    const uint8_t *W;
    size_t nb2, row_bytes;
    const uint8_t *W_sh;      // shared expert down [F, H] or null
    int64_t F, H, n_slots;
    const float *act;         // [pairs][F]
    float *out;               // [T][H]
    const float *residual;    // [T][H] or null
    int group;                // pairs whose weight spans are resident at once
    qwb_status_block *st;
};

// eligibility of the pair path (type_gu Q4_K; down Q4_K / Q6_K with F / 256 in {2, 3, 4, 6})
bool pairs_supported(int type_gu, int type_d, int64_t H, int64_t F, int64_t E, int n_used, int T,
                     size_t rb_gu, size_t nb1_g, size_t nb1_u, size_t rb_d, size_t nb1_d);
cudaError_t launch_gateup_pairs(PairsGateUpArgs a, cudaStream_t s);
cudaError_t launch_down_pairs(int type, PairsDownArgs a, cudaStream_t s);

// One MoE layer on the pair path: router (T clusters), gate/up pairs, down pairs, chained
// with programmatic dependent launch.  Workspace pieces: sel / wts [T][n_used], slots
// [3][T][n_used], sh_scale [T], xq (T rows of Q8_K planes), act [T (n_used + 1)][F].
struct PairsLayer {
    const float *x, *router_w, *mask, *norm_w;
    float norm_eps;
    int64_t H, F, E;
    int n_used, T;
    const int32_t *g2s;
    int64_t own_lo, own_n;  // own_n > 0: expert parallelism (this GPU's expert range)
    const qwb_tensor *gate, *up, *down;
    const qwb_tensor *sh_gate, *sh_up, *sh_down;  // shared expert, or null
    const float *sh_gate_inp;
    const float *residual;
    float *out;
    int32_t *sel, *slots;
    float *wts, *sh_scale, *act;
    Q8Planes xq;
    qwb_status_block *st;
};
cudaError_t run_pairs_layer(const PairsLayer &p, cudaStream_t s);
bool gateup_decode_supported(int type, int64_t K, size_t row_bytes, size_t nb1, int64_t F, int n_used);
cudaError_t launch_gateup_decode(const GateUpDecodeArgs &a, cudaStream_t s);
bool down_decode_supported(int type, int64_t F, int64_t H, size_t row_bytes, size_t nb1, int n_used);
cudaError_t launch_down_decode(int type, const DownDecodeArgs &a, cudaStream_t s);
size_t down_decode_smem_bytes(int64_t H, int n_used, size_t row_bytes);

}  // namespace qwb
