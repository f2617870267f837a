// mmid.cuh - shared declarations of the MUL_MAT_ID building blocks.
#pragma once

#include "common.cuh"

namespace qwb {

// Expert-sorted work description written by the index kernel into the workspace.
constexpr int kIndexCounters = 4;

struct MmidIndex {
    int *n_tiles;  // device scalar
    int *work;     // [kIndexCounters] device counters next to n_tiles, zeroed by the index
                   // kernel: chunk counters of the streaming kernels run on this index (one
                   // per kernel: gate/up uses work[0], down work[1])
    int *pairs;    // [P] pair ids p = t*n_used + j, grouped by expert
    int4 *tiles;   // [max_tiles] (expert, first pair, pair count, 0)
    int max_tiles; // host-side upper bound
};

struct GemvArgs {
    const uint8_t *W;        // expert weights [K, M, n_as] (gate when GLU)
    size_t nb1, nb2;
    const uint8_t *W2;       // up weights (GLU only)
    size_t nb1_2, nb2_2;
    size_t row_bytes;
    int64_t M, K;
    Q8Planes act;            // quantized activation rows
    int act_dstride, act_bstride, act_d_off, act_b_off, act_stride;
    const int4 *tiles;
    const int *n_tiles;
    const int *pairs;
    int n_used, n_b;
    float *dst;              // dst[m, j, t] at dst + j*dnb1 + t*dnb2 (bytes) + 4m
    size_t dnb1, dnb2;
    int R, n_rb, wstage, stage_bytes;
    // streaming kernel geometry (stream_geometry): lanes per row, rows per stage, slot
    // bytes, ring slots, consumer warps, ring offset in shared memory, units per lane group
    int lpr, rpw, slot, nslot, nwarps, ring_off, upg;
    int tg, act_off;     // activation rows staged per pass, their shared-memory offset
    int chunks_per_cta;  // > 1: rows are handed out in chunks from *work (load balance)
    int *work;
    // optional expert -> slot remap (the in-graph get_rows of an I32 [1, E] table,
    // core/runtime.cpp:2769-2778); slot ids must lie in [0, n_slots)
    const int32_t *remap, *remap2;
    int64_t n_ids;    // tile expert ids must lie in [0, n_ids) (the remap table length)
    int64_t n_slots;
    qwb_status_block *st;
};

// Q8_0 / Q6_K experts with 8 or more tokens per expert: integer tensor-core kernel (prefill_i8.cu).
struct I8PrefillArgs {
    const uint8_t *W;        // expert weights [K, M, n_as] (16-byte aligned)
    size_t nb1, nb2;
    int64_t M, K, n_as;
    Q8Planes act;            // activation planes (Q8_0 for Q8_0 weights, Q8_K for Q6_K)
    int act_dstride;
    const int4 *tiles;       // index tiles of <= pf_i8_tile_tokens(type, P, n_as) pairs
    const int *n_tiles;
    const int *pairs;
    int n_used, n_b;
    float *dst;
    size_t dnb1, dnb2;
    int *work;               // item counter (zeroed by the index kernel)
    qwb_status_block *st;
    const uint8_t *btiles;   // tcgen05 kernel: activation codes of every tile, gathered in its B layout
    const float *bda;        // tcgen05 kernel: their scales
};
bool pf_i8_eligible(int type, int64_t K, int64_t M, int64_t P, int64_t n_as, const void *W, size_t nb1, size_t nb2);
int pf_i8_tile_tokens(int type, int64_t P, int64_t n_as);
cudaError_t launch_pf_i8(int type, int tile_tokens, const I8PrefillArgs &a, cudaStream_t s);
// Q6_K / Q8_0 experts with many pairs per expert: tcgen05 kind::i8 grouped GEMM
// (prefill_tc8.cu) over index tiles of up to kTc8TileTokens pairs
constexpr int kTc8TileTokens = 128;
cudaError_t launch_pf_tc8(int type, const I8PrefillArgs &a, cudaStream_t s);
// Bytes per index tile of the gathered activation codes / scales that kernel reads, and
// the gather (one pass over the tiles after the index is built).
size_t tc8_btile_stride(int64_t K);
size_t tc8_da_stride(int type, int64_t K);
cudaError_t launch_tc8_gather(int type, Q8Planes act, int act_dstride, int64_t K, const int4 *tiles,
                              const int *n_tiles, int max_tiles, const int *pairs, int n_used, int n_b,
                              uint8_t *btiles, float *bda, cudaStream_t s);

// MUL_MAT_ID of one token (T == 1) on Q4_K / Q6_K experts in one launch (mmid_one.cu): no
// expert index, no quantizer kernel; each CTA quantizes the activation rows it uses while
// its slice of the selected experts' rows is copied.  x: f32 activation rows at stride x_s1.
bool mmid_one_supported(int type, int64_t K, int64_t M, int n_used, int n_b, size_t nb1);
cudaError_t launch_mmid_one(int type, const uint8_t *W, size_t nb2, int64_t M, int64_t K, int64_t n_as,
                            const int32_t *ids, int64_t ids_s0, int n_used, int n_b, const float *x, int64_t x_s1,
                            float *dst, int64_t dst_s1, qwb_status_block *st, cudaStream_t s);

void gemv_geometry(GemvArgs &a, int NT, bool glu);
cudaError_t launch_gemv(int type, bool glu, GemvArgs a, int NT, int max_tiles, cudaStream_t s);
int pick_nt(int64_t pairs, int64_t n_as);
// Weight-streaming MUL_MAT_ID kernel (mmid_stream.cu): one tile per used expert (index
// built with NT >= pairs), every selected expert row read once.  stream_fits is false
// when the rows are too long for its shared-memory stages.
bool stream_fits(int type, int64_t K, size_t nb1, size_t nb1_2, bool glu);
bool stream_geometry(GemvArgs &a, int type, bool glu);
cudaError_t launch_stream(int type, bool glu, const GemvArgs &a, cudaStream_t s);
// An expert FFN (gate/up GLU GEMV, then down GEMV) can use the streaming kernel for both.
bool stream_fits_ffn(int type_gu, int64_t H, size_t nb_g, size_t nb_u, int type_d, int64_t F, size_t nb_d);
// Expert GEMV over the index's tiles: the streaming kernel when `stream` (index built with
// one tile per expert), else the staged GEMV with tiles of <= NT pairs.
cudaError_t launch_expert_gemv(int type, bool glu, GemvArgs a, bool stream, int NT, int max_tiles, int64_t pairs,
                               int64_t n_experts, int *work, cudaStream_t s);
int64_t mmid_max_tiles(int64_t P, int64_t n_as, int NT);
size_t mmid_index_bytes(int64_t P, int64_t n_as, int NT);
MmidIndex mmid_index_at(void *base, int64_t P, int64_t n_as, int NT);
// skip_neg: ids equal to -1 (pairs routed to another GPU's experts) are left out silently;
// every other id outside [0, n_as) is reported (and its dst row zeroed when dst is given).
cudaError_t launch_index(const int32_t *ids, int64_t s0, int64_t s1, int n_used, int T, int n_as, int NT,
                         MmidIndex ix, float *dst, size_t dnb1, size_t dnb2, int64_t M, qwb_status_block *st,
                         cudaStream_t s, int skip_neg = 0);

// allow_prefill: take the tensor-core grouped GEMM when the problem has many tokens per
// expert (its workspace is larger); false keeps the GEMV path for every size.
qwb_status mul_mat_id_impl(const qwb_tensor *as, const qwb_tensor *b, const qwb_tensor *ids, const qwb_tensor *dst,
                           void *ws, size_t ws_bytes, qwb_status_block *st, cudaStream_t s,
                           bool allow_prefill = true);
size_t mul_mat_id_workspace(const qwb_tensor *as, const qwb_tensor *b, const qwb_tensor *ids, bool allow_prefill);

}  // namespace qwb
