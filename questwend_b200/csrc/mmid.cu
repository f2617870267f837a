// mmid.cu - GGML_OP_MUL_MAT_ID for Q4_K / Q6_K / Q8_0 expert weights on B200.
//
// Reference: ggml_compute_forward_mul_mat_id (ggml-cpu/ggml-cpu.c:1554-1736) and the op
// contract ggml_mul_mat_id (ggml.c:3401-3437).  Pipeline (all stream-ordered, no host
// synchronisation, no allocation):
//   1. quantize src1 rows into q8 planes (Q8_K / Q8_0-cpu), bit-exact with the CPU's
//      from_float (ggml-cpu.c:1609-1644)                               -> quantize.cu
//   2. index build: one CTA histograms the (slot, token) pairs by expert id, prefix-sums
//      them and emits an expert-sorted pair list plus "tiles" of <= NT pairs of one
//      expert (the role of the CPU's matrix_rows grouping, ggml-cpu.c:1646-1661)
//   3. GEMV over (tile, row-block) work items: each item bulk-copies (cp.async.bulk, the
//      non-tensor TMA) R weight rows of its expert and the tile's activation rows into
//      shared memory behind an mbarrier, two stages deep, and computes R x NT dots from
//      shared memory (dp4a integer sub-block sums, fp32 scale combine).  Weights are
//      streamed from HBM once per tile; the grid is persistent (<= SMs x resident CTAs).
// One token (T == 1, Q4_K / Q6_K): one kernel instead (mmid_one.cu) that reads the ids,
// copies its rows and quantizes the activation rows it uses meanwhile.  Many tokens per expert take the tensor-core grouped
// GEMMs (prefill*.cu) after step 2.
#include <algorithm>

#include "common.cuh"
#include "dot.cuh"
#include "kernels.cuh"
#include "mmid.cuh"
#include "prefill.cuh"

namespace qwb {

// ------------------------------------------------------------------ index build
// ids element (slot j, token t) at ids + t*ids_s1 + j*ids_s0 (elements).
__global__ void __launch_bounds__(1024) mmid_index_kernel(const int32_t *__restrict__ ids, int64_t ids_s0,
                                                          int64_t ids_s1, int n_used, int T, int n_as, int NT,
                                                          MmidIndex ix, float *dst, size_t dnb1, size_t dnb2,
                                                          int64_t M, qwb_status_block *st, int skip_neg) {
    // a kernel launched after this one with programmatic dependent launch may start its
    // prologue now; it reads this kernel's output only after griddepcontrol.wait
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    extern __shared__ int sh[];
    int *cnt = sh;              // [n_as]
    int *off = sh + n_as;       // [n_as] pair offset, later running cursor
    int *toff = sh + 2 * n_as;  // [n_as] tile offset
    const int tid = threadIdx.x, nth = blockDim.x;
    const int P = n_used * T;
    for (int e = tid; e < n_as; e += nth) cnt[e] = 0;
    __syncthreads();
    for (int p = tid; p < P; p += nth) {
        const int t = p / n_used, j = p - t * n_used;
        const int e = ids[(int64_t) t * ids_s1 + (int64_t) j * ids_s0];
        if (e >= 0 && e < n_as) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    {
        // exclusive prefix sums of the pair and tile counts over experts: each thread
        // scans its own contiguous range of experts, then the per-thread totals are
        // scanned across the block (warp shuffles + one value per warp)
        __shared__ int wsum_p[32], wsum_t[32];
        const int per = (n_as + nth - 1) / nth;
        const int e0 = min(n_as, tid * per), e1 = min(n_as, e0 + per);
        int sp = 0, st_ = 0;
        for (int e = e0; e < e1; ++e) {
            sp += cnt[e];
            st_ += (cnt[e] + NT - 1) / NT;
        }
        const int lane = tid & 31, wid = tid >> 5;
        int ip = sp, it = st_;  // inclusive scan within the warp
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int xp = __shfl_up_sync(0xffffffffu, ip, o), xt = __shfl_up_sync(0xffffffffu, it, o);
            if (lane >= o) {
                ip += xp;
                it += xt;
            }
        }
        if (lane == 31) {
            wsum_p[wid] = ip;
            wsum_t[wid] = it;
        }
        __syncthreads();
        if (wid == 0) {
            const int nw = (nth + 31) >> 5;
            int vp = lane < nw ? wsum_p[lane] : 0, vt = lane < nw ? wsum_t[lane] : 0;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int xp = __shfl_up_sync(0xffffffffu, vp, o), xt = __shfl_up_sync(0xffffffffu, vt, o);
                if (lane >= o) {
                    vp += xp;
                    vt += xt;
                }
            }
            if (lane < nw) {
                wsum_p[lane] = vp;  // inclusive totals per warp
                wsum_t[lane] = vt;
            }
            if (lane == nw - 1) *ix.n_tiles = vt;
            if (lane < kIndexCounters) ix.work[lane] = 0;
        }
        __syncthreads();
        int po = ip - sp + (wid ? wsum_p[wid - 1] : 0), to = it - st_ + (wid ? wsum_t[wid - 1] : 0);
        for (int e = e0; e < e1; ++e) {
            off[e] = po;
            toff[e] = to;
            po += cnt[e];
            to += (cnt[e] + NT - 1) / NT;
        }
    }
    __syncthreads();
    for (int p = tid; p < P; p += nth) {
        const int t = p / n_used, j = p - t * n_used;
        const int e = ids[(int64_t) t * ids_s1 + (int64_t) j * ids_s0];
        if (e >= 0 && e < n_as) {
            const int pos = atomicAdd(&off[e], 1);
            ix.pairs[pos] = p;
        } else if (!(skip_neg && e == -1)) {
            report(st, QWB_DEVERR_ID_RANGE, e);
            if (dst) {
                float *o = (float *) ((char *) dst + (size_t) j * dnb1 + (size_t) t * dnb2);
                for (int64_t m = 0; m < M; ++m) o[m] = 0.f;
            }
        }
    }
    __syncthreads();
    // off[e] now holds the END of expert e's pairs
    for (int e = tid; e < n_as; e += nth) {
        const int c = cnt[e];
        const int start = off[e] - c;
        for (int k = 0; k * NT < c; ++k)
            ix.tiles[toff[e] + k] = make_int4(e, start + k * NT, min(NT, c - k * NT), 0);
    }
}

// ------------------------------------------------------------------ GEMV kernel
template <int TYPE, int NT, bool GLU>
__global__ void __launch_bounds__(128) mmid_gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t *bar = (uint64_t *) smem;
    uint8_t *stage0 = smem + 128;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int n_tiles = *a.n_tiles;
    const int64_t total = (int64_t) n_tiles * a.n_rb;
    const int64_t per = ceil_div(total, (int64_t) gridDim.x);
    const int64_t i0 = (int64_t) blockIdx.x * per, i1 = min(total, i0 + per);
    if (i0 >= i1) return;

    const size_t wrow = a.row_bytes;
    const int units = (int) (a.K / 32);

    // issue the copies of item `it` into stage buffer `st` (thread 0 only)
    // expert slot of a tile for the first / second weight tensor; -1 when the remap
    // table holds an id outside [0, n_slots)
    auto slot_of = [&](int e, const int32_t *rm) -> int64_t {
        if (e < 0 || e >= a.n_ids) return -1;
        const int64_t sl = rm ? (int64_t) rm[e] : (int64_t) e;
        return (sl >= 0 && sl < a.n_slots) ? sl : -1;
    };
    auto issue = [&](int64_t it, uint8_t *stg, uint64_t *b) {
        const int4 tile = a.tiles[it / a.n_rb];
        const int rb = (int) (it % a.n_rb);
        const int64_t r0 = (int64_t) rb * a.R;
        const int nr = (int) min((int64_t) a.R, a.M - r0);
        const int64_t e1 = slot_of(tile.x, a.remap), e2 = GLU ? slot_of(tile.x, a.remap2) : 0;
        const bool valid = e1 >= 0 && e2 >= 0;
        const uint8_t *src = a.W + (size_t) (valid ? e1 : 0) * a.nb2 + (size_t) r0 * a.nb1;
        const size_t span = (size_t) (nr - 1) * a.nb1 + wrow;
        uint32_t bytes = valid ? bulk_span_bytes(src, span) : 0u;
        const uint8_t *src2 = nullptr;
        if (GLU) {
            src2 = a.W2 + (size_t) (valid ? e2 : 0) * a.nb2_2 + (size_t) r0 * a.nb1_2;
            if (valid) bytes += bulk_span_bytes(src2, (size_t) (nr - 1) * a.nb1_2 + wrow);
        }
        bytes += (uint32_t) (tile.z * a.act_stride);
        mbar_arrive_expect_tx(b, bytes);
        if (valid) bulk_span_issue(stg, src, span, b);
        if (GLU && valid) bulk_span_issue(stg + a.wstage, src2, (size_t) (nr - 1) * a.nb1_2 + wrow, b);
        uint8_t *act = stg + a.wstage * (GLU ? 2 : 1);
        for (int k = 0; k < tile.z; ++k) {
            const int p = a.pairs[tile.y + k];
            const int t = p / a.n_used, j = p - t * a.n_used;
            const int64_t ar = (int64_t) t * a.n_b + (j % a.n_b);
            uint8_t *dk = act + k * a.act_stride;
            bulk_g2s(dk, a.act.qs + ar * a.K, (uint32_t) a.K, b);
            bulk_g2s(dk + a.act_d_off, a.act.d + ar * a.act_dstride, (uint32_t) (a.act_dstride * 4), b);
            if (a.act.bsum)
                bulk_g2s(dk + a.act_b_off, a.act.bsum + ar * a.act_bstride, (uint32_t) (a.act_bstride * 2), b);
        }
    };

    if (tid == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (tid == 0) issue(i0, stage0, &bar[0]);

    for (int64_t it = i0; it < i1; ++it) {
        const int s = (int) ((it - i0) & 1);
        const uint32_t ph = (uint32_t) (((it - i0) >> 1) & 1);
        uint8_t *stg = stage0 + s * a.stage_bytes;
        const bool has_next = it + 1 < i1;
        if (tid == 0 && has_next) {
            fence_proxy_async_smem();
            issue(it + 1, stage0 + (s ^ 1) * a.stage_bytes, &bar[s ^ 1]);
        }
        bool ok = mbar_wait(&bar[s], ph);
        ok = __syncthreads_and(ok);
        if (!ok) {
            if (tid == 0) {
                report(a.st, QWB_DEVERR_TIMEOUT, (int32_t) it);
                mbar_wait(&bar[s], ph);
                if (has_next) mbar_wait(&bar[s ^ 1], (uint32_t) (((it + 1 - i0) >> 1) & 1));
            }
            return;
        }

        const int4 tile = a.tiles[it / a.n_rb];
        const int rb = (int) (it % a.n_rb);
        const int64_t r0 = (int64_t) rb * a.R;
        const int nr = (int) min((int64_t) a.R, a.M - r0);
        const int64_t e1 = slot_of(tile.x, a.remap), e2 = GLU ? slot_of(tile.x, a.remap2) : 0;
        const int cnt = tile.z;
        if (e1 < 0 || e2 < 0) {  // bad slot id: zero this item's outputs, record it
            if (tid == 0 && rb == 0) report(a.st, QWB_DEVERR_ID_RANGE, tile.x);
            for (int idx = tid; idx < nr * cnt; idx += blockDim.x) {
                const int r = idx / cnt, k = idx - r * cnt;
                const int p = a.pairs[tile.y + k];
                const int t = p / a.n_used, j = p - t * a.n_used;
                ((float *) ((char *) a.dst + (size_t) j * a.dnb1 + (size_t) t * a.dnb2))[r0 + r] = 0.f;
            }
            __syncthreads();
            continue;
        }
        const uint8_t *wbase = stg + ((uintptr_t) (a.W + (size_t) e1 * a.nb2 + (size_t) r0 * a.nb1) & 15);
        const uint8_t *wbase2 = nullptr;
        if (GLU)
            wbase2 = stg + a.wstage + ((uintptr_t) (a.W2 + (size_t) e2 * a.nb2_2 + (size_t) r0 * a.nb1_2) & 15);
        ActSmem A{stg + a.wstage * (GLU ? 2 : 1), a.act_stride, a.act_d_off, a.act_b_off};

        for (int r = warp; r < nr; r += 4) {
            float acc[NT], acc2[NT];
#pragma unroll
            for (int k = 0; k < NT; ++k) { acc[k] = 0.f; acc2[k] = 0.f; }
            const uint8_t *row = wbase + (size_t) r * a.nb1;
            const uint8_t *row2 = GLU ? wbase2 + (size_t) r * a.nb1_2 : nullptr;
            for (int u = lane; u < units; u += 32) {
                unit_dot<TYPE, NT>(row, u, A, cnt, acc);
                if (GLU) unit_dot<TYPE, NT>(row2, u, A, cnt, acc2);
            }
#pragma unroll
            for (int k = 0; k < NT; ++k) {
                if (k < cnt) {
                    float v = warp_sum(acc[k]);
                    if (GLU) v = swiglu1(v, warp_sum(acc2[k]));
                    if (lane == 0) {
                        const int p = a.pairs[tile.y + k];
                        const int t = p / a.n_used, j = p - t * a.n_used;
                        float *o = (float *) ((char *) a.dst + (size_t) j * a.dnb1 + (size_t) t * a.dnb2);
                        o[r0 + r] = v;
                    }
                }
            }
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------ host side
int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

template <int TYPE, int NT, bool GLU>
static cudaError_t launch_gemv_t(const GemvArgs &a, int max_items, cudaStream_t s) {
    auto kern = mmid_gemv_kernel<TYPE, NT, GLU>;
    const size_t smem = 128 + 2 * a.stage_bytes;
    static DeviceSmemLimit limit;
    cudaError_t e = ensure_dyn_smem(kern, smem, limit);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, 128, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int grid = std::max(1, std::min(max_items, per_sm * num_sms()));
    kern<<<grid, 128, smem, s>>>(a);
    return cudaGetLastError();
}

template <int TYPE, bool GLU>
static cudaError_t launch_gemv_nt(const GemvArgs &a, int NT, int max_items, cudaStream_t s) {
    switch (NT) {
        case 1: return launch_gemv_t<TYPE, 1, GLU>(a, max_items, s);
        case 2: return launch_gemv_t<TYPE, 2, GLU>(a, max_items, s);
        case 4: return launch_gemv_t<TYPE, 4, GLU>(a, max_items, s);
        default: return launch_gemv_t<TYPE, 8, GLU>(a, max_items, s);
    }
}

cudaError_t launch_gemv(int type, bool glu, GemvArgs a, int NT, int max_tiles, cudaStream_t s) {
    const int max_items = (int) std::min<int64_t>((int64_t) max_tiles * a.n_rb, 1 << 30);
    if (glu) {
        switch (type) {
            case QWB_TYPE_Q4_K: return launch_gemv_nt<QWB_TYPE_Q4_K, true>(a, NT, max_items, s);
            case QWB_TYPE_Q6_K: return launch_gemv_nt<QWB_TYPE_Q6_K, true>(a, NT, max_items, s);
            default: return launch_gemv_nt<QWB_TYPE_Q8_0, true>(a, NT, max_items, s);
        }
    }
    switch (type) {
        case QWB_TYPE_Q4_K: return launch_gemv_nt<QWB_TYPE_Q4_K, false>(a, NT, max_items, s);
        case QWB_TYPE_Q6_K: return launch_gemv_nt<QWB_TYPE_Q6_K, false>(a, NT, max_items, s);
        default: return launch_gemv_nt<QWB_TYPE_Q8_0, false>(a, NT, max_items, s);
    }
}

// choose rows per item R and fill the smem geometry of GemvArgs
void gemv_geometry(GemvArgs &a, int NT, bool glu) {
    const bool kq = a.act.bsum != nullptr;
    a.act_dstride = (int) plane_d_stride(a.K, kq ? QK_K : QK8_0);
    a.act_bstride = kq ? (int) plane_bsum_stride(a.K) : 0;
    a.act_d_off = (int) a.K;
    a.act_b_off = (int) (a.K + a.act_dstride * 4);
    a.act_stride = (int) align_up((size_t) (a.K + a.act_dstride * 4 + a.act_bstride * 2), 16);
    const size_t nbmax = glu ? std::max(a.nb1, a.nb1_2) : a.nb1;
    // rows per item: as many as keep two stages within ~100 KB (two CTAs per SM)
    int R = 32;
    while (R > 1) {
        const size_t w = align_up((size_t) R * nbmax + 32, 16);
        const size_t st = w * (glu ? 2 : 1) + (size_t) NT * a.act_stride;
        if (2 * st + 128 <= 100 * 1024) break;
        R >>= 1;
    }
    a.R = R;
    a.wstage = (int) align_up((size_t) R * nbmax + 32, 16);
    a.stage_bytes = (int) align_up((size_t) a.wstage * (glu ? 2 : 1) + (size_t) NT * a.act_stride, 128);
    a.n_rb = (int) ceil_div(a.M, R);
}

int pick_nt(int64_t pairs, int64_t n_as) {
    const double per_expert = (double) pairs / (double) std::max<int64_t>(1, std::min<int64_t>(pairs, n_as));
    if (per_expert <= 1.0) return 1;
    if (per_expert <= 2.0) return 2;
    if (per_expert <= 4.0) return 4;
    return 8;
}

int64_t mmid_max_tiles(int64_t P, int64_t n_as, int NT) { return P / NT + std::min<int64_t>(P, n_as) + 1; }

size_t mmid_index_bytes(int64_t P, int64_t n_as, int NT) {
    const int64_t max_tiles = mmid_max_tiles(P, n_as, NT);
    return align_up(256, 256) + align_up((size_t) P * 4, 256) + align_up((size_t) max_tiles * 16, 256);
}
MmidIndex mmid_index_at(void *base, int64_t P, int64_t n_as, int NT) {
    MmidIndex ix;
    char *c = (char *) base;
    ix.n_tiles = (int *) c;
    ix.work = ix.n_tiles + 1;
    c += 256;
    ix.pairs = (int *) c;
    c += align_up((size_t) P * 4, 256);
    ix.tiles = (int4 *) c;
    ix.max_tiles = (int) mmid_max_tiles(P, n_as, NT);
    return ix;
}

cudaError_t launch_index(const int32_t *ids, int64_t s0, int64_t s1, int n_used, int T, int n_as, int NT,
                         MmidIndex ix, float *dst, size_t dnb1, size_t dnb2, int64_t M, qwb_status_block *st,
                         cudaStream_t s, int skip_neg) {
    const size_t smem = (size_t) 3 * n_as * 4;
    static DeviceSmemLimit limit;
    if (smem > 48 * 1024) {
        cudaError_t e = ensure_dyn_smem(mmid_index_kernel, smem, limit);
        if (e != cudaSuccess) return e;
    }
    mmid_index_kernel<<<1, 1024, smem, s>>>(ids, s0, s1, n_used, T, n_as, NT, ix, dst, dnb1, dnb2, M, st, skip_neg);
    return cudaGetLastError();
}

}  // namespace qwb

using namespace qwb;

namespace {

struct MmidPlan {
    int type, vdt;
    int64_t K, M, n_as, n_b, T, n_used, P;
    int NT;
    bool pf;  // tensor-core grouped GEMM (many tokens per expert)
    bool stream;  // weight-streaming kernel (one tile per expert)
    bool pf8;     // Q8_0 / Q6_K integer tensor-core kernel (8 or more tokens per expert)
    size_t planes, index, btiles, da, total;
};

qwb_status plan_mmid(const qwb_tensor *as, const qwb_tensor *b, const qwb_tensor *ids, MmidPlan &p,
                     bool allow_prefill) {
    if (!as || !b || !ids) return QWB_ERR_INVALID_ARG;
    if (as->type != QWB_TYPE_Q4_K && as->type != QWB_TYPE_Q6_K && as->type != QWB_TYPE_Q8_0)
        return QWB_ERR_UNSUPPORTED_TYPE;
    if (b->type != QWB_TYPE_F32 || ids->type != QWB_TYPE_I32) return QWB_ERR_UNSUPPORTED_TYPE;
    for (int i = 0; i < 4; ++i)
        if (as->ne[i] < 0 || b->ne[i] < 0 || ids->ne[i] < 0) return QWB_ERR_INVALID_ARG;
    p.type = as->type;
    p.vdt = as->type == QWB_TYPE_Q8_0 ? QWB_TYPE_Q8_0 : QWB_TYPE_Q8_K;
    p.K = as->ne[0];
    p.M = as->ne[1];
    p.n_as = as->ne[2];
    p.n_b = b->ne[1];
    p.T = b->ne[2];
    p.n_used = ids->ne[0];
    // ggml.c:3401-3437: as 3D, b [K, n_b, T], ids [n_used, T], n_used % n_b == 0
    if (as->ne[3] != 1 || b->ne[3] != 1 || ids->ne[2] != 1 || ids->ne[3] != 1) return QWB_ERR_SHAPE;
    if (b->ne[0] != p.K || ids->ne[1] != p.T) return QWB_ERR_SHAPE;
    if (p.n_b == 0 || p.n_used % p.n_b) return QWB_ERR_SHAPE;
    if (p.K % block_elems(p.type) || p.K % block_elems(p.vdt)) return QWB_ERR_SHAPE;
    p.P = p.n_used * p.T;
    if (p.P > (1 << 24) || p.n_as > 16384 || p.K > (1 << 20) || p.M > (1 << 30)) return QWB_ERR_LIMIT;
    p.pf = allow_prefill && pf_eligible(p.type, p.K, p.M, p.P, p.n_as);
    p.pf8 = allow_prefill && pf_i8_eligible(p.type, p.K, p.M, p.P, p.n_as, as->data, as->nb[1], as->nb[2]);
    p.stream = !p.pf && !p.pf8 && stream_fits(p.type, p.K, as->nb[1], as->nb[1], false);
    p.NT = p.pf    ? kPfTileN
           : p.pf8 ? pf_i8_tile_tokens(p.type, p.P, p.n_as)
           : p.stream ? (int) std::max<int64_t>(1, p.P)
                      : pick_nt(p.P, p.n_as);
    p.planes = planes_bytes(p.n_b * p.T, p.K, p.vdt == QWB_TYPE_Q8_K);
    p.index = mmid_index_bytes(p.P, p.n_as, p.NT);
    p.btiles = p.da = 0;
    if (p.pf) {
        const int64_t max_tiles = mmid_max_tiles(p.P, p.n_as, p.NT);
        p.btiles = align_up((size_t) max_tiles * pf_btile_stride(p.K), 256);
        p.da = align_up((size_t) max_tiles * pf_da_stride(p.K), 256);
    } else if (p.pf8 && p.NT == kTc8TileTokens) {
        const int64_t max_tiles = mmid_max_tiles(p.P, p.n_as, p.NT);
        p.btiles = align_up((size_t) max_tiles * tc8_btile_stride(p.K), 256);
        p.da = align_up((size_t) max_tiles * tc8_da_stride(p.type, p.K), 256);
    }
    // [0, 256) is the control block of the fused kernels
    p.total = kCtrlBytes + p.planes + p.index + p.btiles + p.da;
    return QWB_OK;
}

}  // namespace

size_t qwb::mul_mat_id_workspace(const qwb_tensor *as, const qwb_tensor *b, const qwb_tensor *ids,
                                 bool allow_prefill) {
    MmidPlan p;
    if (plan_mmid(as, b, ids, p, allow_prefill) != QWB_OK) return 0;
    return p.total;
}

extern "C" QWB_API size_t qwb_mul_mat_id_workspace_size(const qwb_tensor *as, const qwb_tensor *b,
                                                        const qwb_tensor *ids) {
    // the larger of the two plans (tensor-core kernels allowed, GEMV kernels only): the
    // GEMV plan's expert index can be the larger one for rows too long to stream
    return std::max(qwb::mul_mat_id_workspace(as, b, ids, true), qwb::mul_mat_id_workspace(as, b, ids, false));
}

qwb_status qwb::mul_mat_id_impl(const qwb_tensor *as, const qwb_tensor *b, const qwb_tensor *ids,
                                const qwb_tensor *dst, void *ws, size_t ws_bytes, qwb_status_block *st,
                                cudaStream_t s, bool allow_prefill) {
    MmidPlan p;
    qwb_status rc = plan_mmid(as, b, ids, p, allow_prefill);
    if (rc != QWB_OK) return rc;
    if (!dst || dst->type != QWB_TYPE_F32) return dst ? QWB_ERR_UNSUPPORTED_TYPE : QWB_ERR_INVALID_ARG;
    if (dst->ne[0] != p.M || dst->ne[1] != p.n_used || dst->ne[2] != p.T || dst->ne[3] != 1) return QWB_ERR_SHAPE;
    if (p.P == 0 || p.M == 0) return QWB_OK;
    if (p.K == 0) return QWB_ERR_SHAPE;
    if (!as->data || !b->data || !ids->data || !dst->data) return QWB_ERR_INVALID_ARG;
    // layouts: rows of as contiguous blocks; b rows contiguous f32; dst rows contiguous
    if (as->nb[0] != row_bytes(p.type, block_elems(p.type))) return QWB_ERR_LAYOUT;
    if (as->nb[1] < row_bytes(p.type, p.K) || as->nb[2] < as->nb[1] * (size_t) p.M) return QWB_ERR_LAYOUT;
    if (b->nb[0] != 4 || dst->nb[0] != 4) return QWB_ERR_LAYOUT;
    if (ids->nb[0] % 4 || ids->nb[1] % 4) return QWB_ERR_ALIGNMENT;
    const uintptr_t walign = (uintptr_t) as->data | as->nb[1] | as->nb[2];
    if (p.type == QWB_TYPE_Q4_K ? walign % 16 : walign % 2) return QWB_ERR_ALIGNMENT;
    if (((uintptr_t) b->data | b->nb[1] | b->nb[2]) % 16) return QWB_ERR_ALIGNMENT;
    if (((uintptr_t) dst->data | dst->nb[1] | dst->nb[2]) % 4) return QWB_ERR_ALIGNMENT;
    if (!ws || ws_bytes < p.total) return QWB_ERR_WORKSPACE;
    if ((uintptr_t) ws % 256) return QWB_ERR_ALIGNMENT;
    if (b->nb[2] != b->nb[1] * (size_t) p.n_b) return QWB_ERR_LAYOUT;  // rows (j, t) at stride nb1

    const bool kq = p.vdt == QWB_TYPE_Q8_K;
    profile_mark(s, 0);
    Q8Planes pl = planes_at((char *) ws + kCtrlBytes, p.n_b * p.T, p.K, kq);
    MmidIndex ix = mmid_index_at((char *) ws + kCtrlBytes + p.planes, p.P, p.n_as, p.NT);
    if (p.T == 1 && !p.pf && !p.pf8 && (uintptr_t) as->data % 16 == 0 && as->nb[2] % 16 == 0 &&
        mmid_one_supported(p.type, p.K, p.M, (int) p.n_used, (int) p.n_b, as->nb[1])) {
        // one token: one launch over the rows of its selected experts (no expert index, the
        // activation rows quantized inside)
        const cudaError_t e1 = launch_mmid_one(p.type, (const uint8_t *) as->data, as->nb[2], p.M, p.K, p.n_as,
                                               (const int32_t *) ids->data, (int64_t) (ids->nb[0] / 4), (int) p.n_used,
                                               (int) p.n_b, (const float *) b->data, (int64_t) (b->nb[1] / 4),
                                               (float *) dst->data, (int64_t) (dst->nb[1] / 4), st, s);
        profile_mark(s, QWB_KERNEL_EXPERT_GEMV);
        return e1 == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
    }
    cudaError_t e = launch_quantize_rows(kq ? 0 : 1, (const float *) b->data, (int64_t) (b->nb[1] / 4),
                                         p.n_b * p.T, p.K, nullptr, pl, nullptr, s);
    if (e != cudaSuccess) return QWB_ERR_CUDA;
    e = launch_index((const int32_t *) ids->data, (int64_t) (ids->nb[0] / 4), (int64_t) (ids->nb[1] / 4),
                     (int) p.n_used, (int) p.T, (int) p.n_as, p.NT, ix, (float *) dst->data, dst->nb[1], dst->nb[2],
                     p.M, st, s);
    if (e != cudaSuccess) return QWB_ERR_CUDA;
    if (p.pf) {
        uint8_t *bt = (uint8_t *) ws + kCtrlBytes + p.planes + p.index;
        float *da = (float *) (bt + p.btiles);
        e = launch_pf_gather(pl, p.K, ix.tiles, ix.n_tiles, ix.max_tiles, ix.pairs, (int) p.n_used, (int) p.n_b, bt,
                             da, s);
        if (e != cudaSuccess) return QWB_ERR_CUDA;
        profile_mark(s, QWB_KERNEL_OTHER);
        PrefillArgs a{};
        a.W = (const uint8_t *) as->data;
        a.nb1 = as->nb[1];
        a.nb2 = as->nb[2];
        a.M = p.M;
        a.K = p.K;
        a.remap = nullptr;
        a.n_ids = p.n_as;
        a.n_slots = p.n_as;
        a.tiles = ix.tiles;
        a.n_tiles = ix.n_tiles;
        a.pairs = ix.pairs;
        a.btiles = bt;
        a.da = da;
        a.dst = (float *) dst->data;
        a.dnb1 = dst->nb[1];
        a.dnb2 = dst->nb[2];
        a.n_used = (int) p.n_used;
        a.m_tiles = (int) ceil_div(p.M, kPfTileM);
        a.st = st;
        e = launch_pf_gemm_q4k(a, s);
        profile_mark(s, QWB_KERNEL_GROUPED_GEMM);
        return e == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
    }
    profile_mark(s, QWB_KERNEL_OTHER);
    if (p.pf8) {
        I8PrefillArgs q{};
        q.W = (const uint8_t *) as->data;
        q.nb1 = as->nb[1];
        q.nb2 = as->nb[2];
        q.M = p.M;
        q.K = p.K;
        q.n_as = p.n_as;
        q.act = pl;
        q.act_dstride = (int) plane_d_stride(p.K, kq ? QK_K : QK8_0);
        q.tiles = ix.tiles;
        q.n_tiles = ix.n_tiles;
        q.pairs = ix.pairs;
        q.n_used = (int) p.n_used;
        q.n_b = (int) p.n_b;
        q.dst = (float *) dst->data;
        q.dnb1 = dst->nb[1];
        q.dnb2 = dst->nb[2];
        q.work = ix.work + 2;
        q.st = st;
        if (p.NT == kTc8TileTokens) {
            uint8_t *bt = (uint8_t *) ws + kCtrlBytes + p.planes + p.index;
            float *bda = (float *) (bt + p.btiles);
            e = launch_tc8_gather(p.type, pl, q.act_dstride, p.K, ix.tiles, ix.n_tiles, ix.max_tiles, ix.pairs,
                                  (int) p.n_used, (int) p.n_b, bt, bda, s);
            if (e != cudaSuccess) return QWB_ERR_CUDA;
            profile_mark(s, QWB_KERNEL_OTHER);
            q.btiles = bt;
            q.bda = bda;
        }
        e = launch_pf_i8(p.type, p.NT, q, s);
        profile_mark(s, QWB_KERNEL_GROUPED_GEMM);
        return e == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
    }
    GemvArgs a{};
    a.W = (const uint8_t *) as->data;
    a.nb1 = as->nb[1];
    a.nb2 = as->nb[2];
    a.row_bytes = row_bytes(p.type, p.K);
    a.M = p.M;
    a.K = p.K;
    a.act = pl;
    a.tiles = ix.tiles;
    a.n_tiles = ix.n_tiles;
    a.pairs = ix.pairs;
    a.n_used = (int) p.n_used;
    a.n_b = (int) p.n_b;
    a.dst = (float *) dst->data;
    a.dnb1 = dst->nb[1];
    a.dnb2 = dst->nb[2];
    a.n_ids = p.n_as;
    a.n_slots = p.n_as;
    a.st = st;
    if (p.stream) {
        // rows cost more with more tokens on their expert: hand out chunks dynamically
        a.chunks_per_cta = 2 * p.P > 3 * std::min(p.P, p.n_as) ? 8 : 4;
        a.work = ix.work;
        if (!stream_geometry(a, p.type, false)) return QWB_ERR_LAYOUT;
        e = launch_stream(p.type, false, a, s);
    } else {
        gemv_geometry(a, p.NT, false);
        e = launch_gemv(p.type, false, a, p.NT, ix.max_tiles, s);
    }
    profile_mark(s, QWB_KERNEL_EXPERT_GEMV);
    return e == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
}

extern "C" QWB_API qwb_status qwb_mul_mat_id(const qwb_tensor *as, const qwb_tensor *b, const qwb_tensor *ids,
                                             const qwb_tensor *dst, void *workspace, size_t workspace_bytes,
                                             qwb_status_block *d_status, qwb_stream_t stream) {
    return qwb::mul_mat_id_impl(as, b, ids, dst, workspace, workspace_bytes, d_status, (cudaStream_t) stream);
}
