// prefill.cuh - grouped expert GEMM for MUL_MAT_ID with many tokens per expert, on the
// 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
#pragma once

#include "common.cuh"
#include "mmid.cuh"

namespace qwb {

// Token tile: up to 128 (token, slot) pairs of one expert; weight tile: 128 rows.
constexpr int kPfTileN = 128;
constexpr int kPfTileM = 128;
// K positions per superblock in the fp16 B tiles: two halves of 128 activation values plus
// 16 block sums each (the min-term columns).
constexpr int kPfHalfK = 144;

// Token columns of a tile of `cnt` pairs (the M=128 MMA takes N in steps of 16).
__host__ __device__ inline int pf_tile_cols(int cnt) { return (cnt + 15) & ~15; }

// Bytes of the B tile buffer for `max_tiles` tiles of a K-long activation.
__host__ __device__ inline size_t pf_btile_stride(int64_t K) { return (size_t) kPfTileN * (size_t) (K / QK_K) * 2 * kPfHalfK * 2; }
__host__ __device__ inline size_t pf_da_stride(int64_t K) { return (size_t) kPfTileN * (size_t) (K / QK_K) * 4; }

struct PrefillArgs {
    const uint8_t *W;       // expert weights [K, M, n_slots]
    size_t nb1, nb2;
    int64_t M, K;
    const int32_t *remap;   // optional expert -> slot table
    int64_t n_ids, n_slots;
    const int4 *tiles;      // (expert, first pair, pair count, 0), count <= kPfTileN
    const int *n_tiles;
    const int *pairs;
    const uint8_t *btiles;  // fp16 B tiles, pf_btile_stride(K) bytes per tile
    const float *da;        // activation scales, [tile][K/256][kPfTileN]
    float *dst;             // dst[m, j, t] at dst + j*dnb1 + t*dnb2 (bytes) + 4m
    size_t dnb1, dnb2;
    int n_used;
    int m_tiles;            // 128-row weight tiles, ceil(M / 128)
    qwb_status_block *st;
};

// Fills the fp16 B tiles and activation scales of every tile from Q8_K planes.
// Pair p = t*n_used + j reads plane row t*n_b + (j % n_b).
cudaError_t launch_pf_gather(Q8Planes act, int64_t K, const int4 *tiles, const int *n_tiles, int max_tiles,
                             const int *pairs, int n_used, int n_b, uint8_t *btiles, float *da, cudaStream_t s);

cudaError_t launch_pf_gemm_q4k(const PrefillArgs &a, cudaStream_t s);

// Whether mul_mat_id takes the tensor-core path for this problem.
bool pf_eligible(int type, int64_t K, int64_t M, int64_t P, int64_t n_as);

}  // namespace qwb
