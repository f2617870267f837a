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
    const float *x;         // [H] layer input (residual stream)
    const float *router_w;  // [E][H]
    const float *mask;      // [E] or null
    const float *norm_w;    // [H] or null
    float norm_eps;
    int64_t H, E;
    int n_used;
    const int32_t *g2s;     // [3][E] or null
    int64_t n_slots[3];     // pool sizes (gate, up, down)
    int32_t *sel;           // [n_used] out
    float *wts;             // [n_used] out
    int32_t *slots;         // [3][n_used] out: resolved slot ids (-1: invalid)
    Q8Planes xq;            // Q8 of the normed x (one row) out
    int kq;
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
bool gateup_decode_supported(int type, int64_t K, size_t row_bytes, size_t nb1, int64_t F, int n_used);
cudaError_t launch_gateup_decode(const GateUpDecodeArgs &a, cudaStream_t s);
bool down_decode_supported(int type, int64_t F, int64_t H, size_t row_bytes, size_t nb1, int n_used);
cudaError_t launch_down_decode(int type, const DownDecodeArgs &a, cudaStream_t s);
size_t down_decode_smem_bytes(int64_t H, int n_used, size_t row_bytes);

}  // namespace qwb
