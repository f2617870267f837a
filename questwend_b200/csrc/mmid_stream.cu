// mmid_stream.cu - MUL_MAT_ID for few tokens per expert (decode batches of 1-64 tokens):
// a weight-streaming kernel that reads every selected expert row exactly once.
//
// Reference: ggml_compute_forward_mul_mat_id (ggml-cpu/ggml-cpu.c:1554-1736) with the
// CPU dots of dot.cuh (ggml-cpu/quants.c q4_K / q6_K / q8_0 x q8).  The CPU backend walks
// experts and, per expert, every (row, routed token) pair; here the (used expert, row)
// space is cut into chunks handed to persistent CTAs, so each expert row meets all of its
// tokens while it is in shared memory and is read from HBM once.
//
// One CTA per SM: warp NWC is the producer, warps 0..NWC-1 consume.
//   * A stage is a contiguous span of up to SR = NWC * RPW rows of one expert (one bulk
//     copy, tens of KB: the copy engine's cost is per copy, so copies must be large to
//     reach HBM bandwidth).  The ring holds `depth` stages; the producer publishes each
//     stage's (expert tile, first row, row count) in a descriptor before arming its full
//     barrier, and reuses a slot once all NWC consumer warps have released it.
//   * Consumer warp w takes rows [w*RPW, (w+1)*RPW) of every stage: lane = (row, group of
//     superblocks), LPR lanes per row.  It reads the routed tokens' Q8 rows in place from
//     the activation planes (L1-cached global loads), 8 tokens per pass, reduces over the
//     LPR lanes of a row with shuffles and writes dst (GLU: swiglu(gate, up)).
//   * Chunks: CTA b starts with chunk b; when the experts carry several tokens (compute
//     per row varies with the token count) there are more chunks than CTAs and the rest
//     are taken from a counter the index kernel zeroed.
// Every wait is bounded; a timed-out wait records QWB_DEVERR_TIMEOUT, stops the CTA and
// drains the copies already issued before the CTA exits.
#include <algorithm>

#include "common.cuh"
#include "dot.cuh"
#include "kernels.cuh"
#include "mmid.cuh"

namespace qwb {

// Optional phase timestamps (compiled in only with -DQWB_STREAM_TRACE; no effect on the
// default build): one thread per CTA records the global timer at numbered points.
#ifdef QWB_STREAM_TRACE
__device__ unsigned long long g_stream_trace[160][32];
#define ST_TRACE(p)                                                                        \
    do {                                                                                  \
        if (blockIdx.x < 160) g_stream_trace[blockIdx.x][p] = globaltimer_ns();           \
    } while (0)
#else
#define ST_TRACE(p) \
    do {            \
    } while (0)
#endif

namespace {

constexpr int kStreamTok = 8;        // tokens per consumer pass
constexpr int kStreamMaxWarps = 15;  // consumer warps: with the producer, 16 warps (128 registers)
constexpr int kStreamDepth = 3;      // stages in the ring
constexpr size_t kStreamSmemBudget = 216 * 1024;  // ring + staged activations + barriers
constexpr size_t kStreamActBudget = 40 * 1024;    // staged activation rows

struct StreamDesc {
    int tile;  // index into tiles[]
    int r0;    // first weight row of the stage
    int nr;    // rows in the stage (0: end of the stream)
    int off1;  // offset of the first row inside the slot (16-byte widening)
    int off2;  // same, second (up) matrix
    int bad;   // expert slot invalid: outputs are zeroed
    int pad0, pad1;
};

// named barrier over the consumer warps only (the producer keeps running)
__device__ __forceinline__ void consumer_sync(int nthreads) {
    asm volatile("bar.sync 1, %0;" ::"r"(nthreads) : "memory");
}

// Release of a ring slot by a consumer warp.  Relaxed: it only has to follow the warp's
// shared-memory reads of the slot, which have completed once their values were used; a
// release arrive would also wait for the warp's global output stores to be acknowledged.
__device__ __forceinline__ void mbar_arrive_relaxed(uint64_t *bar) {
    asm volatile("mbarrier.arrive.relaxed.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Weight rows are read exactly once: copy them with an L2 evict-first policy so they do
// not displace the activations, the expert index and the kernel's code from L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void bulk_span_issue_ef(void *dst, const void *src, size_t bytes, uint64_t *bar,
                                                   uint64_t pol) {
    const uintptr_t a = (uintptr_t) src & ~(uintptr_t) 15;
    const uint32_t total = bulk_span_bytes(src, bytes);
    for (uint32_t off = 0; off < total; off += 65536u) {
        const uint32_t n = total - off < 65536u ? total - off : 65536u;
        asm volatile(
            "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
                smem_u32((char *) dst + off)),
            "l"((const void *) (a + off)), "r"(n), "r"(smem_u32(bar)), "l"(pol)
            : "memory");
    }
}

// Bounded wait that also gives up as soon as another warp has aborted the CTA.
__device__ __forceinline__ bool stream_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    if (mbar_try_wait_fast(bar, parity)) return true;
    const uint64_t t0 = globaltimer_ns();
    while (true) {
        if (mbar_try_wait_fast(bar, parity)) return true;
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
    }
}

__device__ __forceinline__ int64_t stream_slot_of(const GemvArgs &a, int e, const int32_t *rm) {
    if (e < 0 || e >= a.n_ids) return -1;
    const int64_t sl = rm ? (int64_t) rm[e] : (int64_t) e;
    return (sl >= 0 && sl < a.n_slots) ? sl : -1;
}

// One pass of a lane over its row's superblock groups against NT staged tokens (ng <= NT
// valid), the reduction over the LPR lanes of the row, and the row's outputs.
template <int TYPE, bool GLU, int NT>
__device__ __noinline__ void stream_pass(const uint8_t *row1, const uint8_t *row2, const ActStage &A, int ng,
                                            bool live, bool bad, int LPR, int sl, int n_sb, int units, int UPG,
                                            bool row_ok, const long long *tok_o, float *dst, int row) {
    // every pointer below is into this CTA's shared memory: let the compiler use shared
    // loads (this function is not inlined, so it cannot see where they come from)
    __builtin_assume(__isShared(row1));
    if (GLU) __builtin_assume(__isShared(row2));
    __builtin_assume(__isShared(A.base));
    __builtin_assume(__isShared(tok_o));
    float acc[NT], acc2[NT];
#pragma unroll
    for (int k = 0; k < NT; ++k) {
        acc[k] = 0.f;
        acc2[k] = 0.f;
    }
    if (live) {
        for (int sb = sl; sb < n_sb; sb += LPR) {
            if constexpr (TYPE == QWB_TYPE_Q4_K) {
                sb_q4K<NT>(row1 + (size_t) sb * Q4K_BYTES, sb, A, ng, acc);
                if (GLU) sb_q4K<NT>(row2 + (size_t) sb * Q4K_BYTES, sb, A, ng, acc2);
            } else if constexpr (TYPE == QWB_TYPE_Q6_K) {
                sb_q6K<NT>(row1 + (size_t) sb * Q6K_BYTES, sb, A, ng, acc);
                if (GLU) sb_q6K<NT>(row2 + (size_t) sb * Q6K_BYTES, sb, A, ng, acc2);
            } else {
                const int u1 = min(units, UPG * sb + UPG);
                for (int u = UPG * sb; u < u1; ++u) {
                    unit_dot<TYPE, NT>(row1, u, A, ng, acc);
                    if (GLU) unit_dot<TYPE, NT>(row2, u, A, ng, acc2);
                }
            }
        }
    }
#pragma unroll
    for (int k = 0; k < NT; ++k) {
        for (int o = 1; o < LPR; o <<= 1) {
            acc[k] += __shfl_xor_sync(0xffffffffu, acc[k], o);
            if (GLU) acc2[k] += __shfl_xor_sync(0xffffffffu, acc2[k], o);
        }
        if (k < ng && sl == 0 && row_ok) {
            const float v = bad ? 0.f : (GLU ? swiglu1(acc[k], acc2[k]) : acc[k]);
            ((float *) ((char *) dst + tok_o[k]))[row] = v;
        }
    }
}

template <int TYPE, bool GLU>
__global__ void __launch_bounds__(32 * (kStreamMaxWarps + 1), 1) mmid_stream_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int NS = a.nslot;
    uint64_t *full = (uint64_t *) smem;
    uint64_t *empty = full + NS;
    StreamDesc *desc = (StreamDesc *) (empty + NS);
    volatile int *abort_flag = (volatile int *) (desc + NS);
    long long *tok_o = (long long *) (desc + NS) + 2;   // [kStreamTok] output byte offsets
    int *tok_ar = (int *) (tok_o + kStreamTok);          // [kStreamTok] activation plane rows
    uint8_t *act_buf = smem + a.act_off;                 // [TG][act_stride] staged Q8 rows
    uint8_t *ring = smem + a.ring_off;

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NWC = (int) (blockDim.x >> 5) - 1;
    const int SR = NWC * a.rpw;  // rows per stage
    if (tid == 0) ST_TRACE(0);
    if (tid == 0) {
        for (int i = 0; i < NS; ++i) {
            mbar_init(&full[i], 1);
            mbar_init(&empty[i], (uint32_t) NWC);
        }
        *abort_flag = 0;
    }
    __syncthreads();  // barriers are CTA-local: the block barrier publishes their init
    // launched with programmatic dependent launch: everything above overlapped the index
    // kernel; its output (and the quantized activations before it) is read only below
    asm volatile("griddepcontrol.wait;" ::: "memory");

    if (tid == 0) ST_TRACE(1);
    const int64_t total = (int64_t) (*a.n_tiles) * a.M;
    if (tid == 0) ST_TRACE(2);
    const size_t half = (size_t) a.slot / (GLU ? 2 : 1);
    int issued = 0;  // producer: stages issued

    if (warp == NWC) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            const int64_t n_chunks = (int64_t) gridDim.x * a.chunks_per_cta;
            const int64_t CH = align_up((size_t) ceil_div(max(total, (int64_t) 1), n_chunks), (size_t) SR);
            int64_t chunk = blockIdx.x;
            int64_t next = a.chunks_per_cta > 1 ? (int64_t) gridDim.x + atomicAdd(a.work, 1) : n_chunks;
            int64_t g = chunk * CH, gend = min(total, g + CH);
            int cur_tile = -1;
            int64_t e1 = -1, e2 = -1;
            for (int s = 0;; ++s) {
                while (g >= gend && chunk < n_chunks) {  // chunk done: take the next one
                    chunk = next;
                    if (chunk < n_chunks) {
                        g = chunk * CH;
                        gend = min(total, g + CH);
                        next = (int64_t) gridDim.x + atomicAdd(a.work, 1);
                    }
                }
                const bool real = g < gend;
                const int slot = s % NS;
                const int round = s / NS;
                if (round > 0 && !stream_wait(&empty[slot], (uint32_t) ((round - 1) & 1), abort_flag)) {
                    report(a.st, QWB_DEVERR_TIMEOUT, s);
                    *abort_flag = 1;
                    break;
                }
                // the slot's readers released it through the empty barrier (release-arrive
                // / acquire-wait) before the async-proxy copy below overwrites it
                StreamDesc d{};
                const uint8_t *src1 = nullptr, *src2 = nullptr;
                size_t span1 = 0, span2 = 0;
                uint32_t bytes = 0;
                if (real) {
                    const int i = (int) (g / a.M);
                    const int64_t r = g - (int64_t) i * a.M;
                    const int nr = (int) min((int64_t) SR, min(a.M - r, gend - g));
                    if (i != cur_tile) {
                        cur_tile = i;
                        const int4 t = a.tiles[i];
                        e1 = stream_slot_of(a, t.x, a.remap);
                        e2 = GLU ? stream_slot_of(a, t.x, a.remap2) : 0;
                    }
                    d.tile = i;
                    d.r0 = (int) r;
                    d.nr = nr;
                    d.bad = (e1 < 0 || e2 < 0) ? 1 : 0;
                    if (!d.bad) {
                        src1 = a.W + (size_t) e1 * a.nb2 + (size_t) r * a.nb1;
                        span1 = (size_t) (nr - 1) * a.nb1 + a.row_bytes;
                        d.off1 = (int) ((uintptr_t) src1 & 15);
                        bytes = bulk_span_bytes(src1, span1);
                        if (GLU) {
                            src2 = a.W2 + (size_t) e2 * a.nb2_2 + (size_t) r * a.nb1_2;
                            span2 = (size_t) (nr - 1) * a.nb1_2 + a.row_bytes;
                            d.off2 = (int) ((uintptr_t) src2 & 15);
                            bytes += bulk_span_bytes(src2, span2);
                        }
                    }
                    g += nr;
                }  // else: d.nr == 0 ends the consumers' stream
                desc[slot] = d;
                mbar_arrive_expect_tx(&full[slot], bytes);
                if (bytes) {
                    uint8_t *dst = ring + (size_t) slot * a.slot;
                    bulk_span_issue_ef(dst, src1, span1, &full[slot], pol);
                    if (GLU) bulk_span_issue_ef(dst + half, src2, span2, &full[slot], pol);
                }
                issued = s + 1;
                if (s < 6) ST_TRACE(3 + s);
                if (!real) break;
            }
            ST_TRACE(27);
        }
    } else {
        // ------------------------------------------------------------ consumers
        // The routed tokens' Q8 rows of the current expert (TG at a time) are staged in
        // shared memory by all consumer warps together (one round trip to L2 per expert
        // instead of dependent loads inside every dot); all consumer warps walk the same
        // stage sequence, so they agree on when the staged rows change.
        const int LPR = a.lpr;
        const int rr = warp * a.rpw + lane / LPR, sl = lane % LPR;  // row within the stage
        const int units = (int) (a.K / 32);
        const int UPG = a.upg;  // units per lane group: a K-quant superblock, or 4 Q8_0 blocks
        const int n_sb = (units + UPG - 1) / UPG;
        const int TG = a.tg;
        const int nthr = NWC * 32;
        const bool kq = TYPE != QWB_TYPE_Q8_0;
        const ActStage A{act_buf, a.act_stride, a.act_d_off, a.act_b_off, kq ? 3 : 2};
        const int pq = (int) (a.K / 16), pd = a.act_dstride / 4, pb = a.act_bstride / 8;  // 16-byte pieces
        const int per_tok = pq + pd + pb;
        const int qsh = kq ? 4 : 3;  // log2(16-byte pieces per padded qs group)
        int cur_tile = -1, cur_g0 = -1;
        int4 t = make_int4(0, 0, 0, 0);
        for (int s = 0;; ++s) {
            const int slot = s % NS;
            if (!stream_wait(&full[slot], (uint32_t) ((s / NS) & 1), abort_flag)) {
                if (lane == 0 && !*abort_flag) {
                    report(a.st, QWB_DEVERR_TIMEOUT, s);
                    *abort_flag = 1;
                }
                break;
            }
            if (s < 6 && warp == 0 && lane == 0) ST_TRACE(9 + s);
            const StreamDesc d = desc[slot];
            if (d.nr == 0) break;
            if (d.tile != cur_tile) t = a.tiles[d.tile];  // (expert, first pair, pair count)
            const bool row_ok = rr < d.nr;
            const uint8_t *row1 = ring + (size_t) slot * a.slot + d.off1 + (size_t) rr * a.nb1;
            const uint8_t *row2 = GLU ? ring + (size_t) slot * a.slot + half + d.off2 + (size_t) rr * a.nb1_2 : nullptr;
            for (int g0 = 0; g0 < t.z; g0 += TG) {
                const int ng = min(TG, t.z - g0);
                if (d.tile != cur_tile || g0 != cur_g0) {
                    consumer_sync(nthr);  // every warp is done with the rows staged before
                    if (tid < ng) {
                        const int p = a.pairs[t.y + g0 + tid];
                        const int tt = p / a.n_used, j = p - tt * a.n_used;
                        tok_ar[tid] = tt * a.n_b + j % a.n_b;
                        tok_o[tid] = (long long) ((size_t) j * a.dnb1 + (size_t) tt * a.dnb2);
                    }
                    consumer_sync(nthr);
                    if (s == 0 && g0 == 0 && warp == 0 && lane == 0) ST_TRACE(21);
                    for (int i = tid; i < ng * per_tok; i += nthr) {
                        const int k = i / per_tok, r = i - k * per_tok;
                        const int64_t ar = tok_ar[k];
                        const uint8_t *src;
                        uint8_t *dst = act_buf + (size_t) k * a.act_stride;
                        if (r < pq) {  // qs: 16 spare bytes after each group
                            src = (const uint8_t *) a.act.qs + ar * a.K + 16 * r;
                            dst += (r >> qsh) * ((16 << qsh) + 16) + 16 * (r & ((1 << qsh) - 1));
                        } else if (r < pq + pd) {
                            src = (const uint8_t *) (a.act.d + ar * a.act_dstride) + 16 * (r - pq);
                            dst += a.act_d_off + 16 * (r - pq);
                        } else {  // bsums: 16 spare bytes after each superblock's 32
                            const int rb = r - pq - pd;
                            src = (const uint8_t *) (a.act.bsum + ar * a.act_bstride) + 16 * rb;
                            dst += a.act_b_off + (rb >> 1) * 48 + 16 * (rb & 1);
                        }
                        *(int4 *) dst = *(const int4 *) src;
                    }
                    consumer_sync(nthr);
                    cur_tile = d.tile;
                    cur_g0 = g0;
                    if (s == 0 && g0 == 0 && warp == 0 && lane == 0) ST_TRACE(22);
                }
                // one pass over the staged tokens, instantiated for the pass width
                const bool live = row_ok && !d.bad;
                if (s == 1 && g0 == 0 && warp == 0 && lane == 0) ST_TRACE(28);
                if (ng == 1) stream_pass<TYPE, GLU, 1>(row1, row2, A, ng, live, d.bad, LPR, sl, n_sb, units, UPG, row_ok, tok_o, a.dst, d.r0 + rr);
                else if (ng == 2) stream_pass<TYPE, GLU, 2>(row1, row2, A, ng, live, d.bad, LPR, sl, n_sb, units, UPG, row_ok, tok_o, a.dst, d.r0 + rr);
                else if (ng <= 4) stream_pass<TYPE, GLU, 4>(row1, row2, A, ng, live, d.bad, LPR, sl, n_sb, units, UPG, row_ok, tok_o, a.dst, d.r0 + rr);
                else stream_pass<TYPE, GLU, 8>(row1, row2, A, ng, live, d.bad, LPR, sl, n_sb, units, UPG, row_ok, tok_o, a.dst, d.r0 + rr);
                if (s == 0 && g0 == 0 && warp == 0 && lane == 0) ST_TRACE(23);
                if (s == 1 && g0 == 0 && warp == 0 && lane == 0) ST_TRACE(29);
            }
            if (d.bad && d.r0 == 0 && warp == 0 && lane == 0) report(a.st, QWB_DEVERR_ID_RANGE, t.x);
            __syncwarp();
            if (lane == 0) mbar_arrive_relaxed(&empty[slot]);
            if (s < 6 && warp == 0 && lane == 0) ST_TRACE(15 + s);
        }
        if (warp == 0 && lane == 0) ST_TRACE(24);
    }
    __syncthreads();
    if (tid == 0) ST_TRACE(25);
    // after an abort, copies may still be in flight: wait for every slot's last stage
    if (warp == NWC && lane == 0 && *abort_flag) {
        for (int slot = 0; slot < NS && slot < issued; ++slot) {
            const int last = slot + ((issued - 1 - slot) / NS) * NS;
            mbar_wait(&full[slot], (uint32_t) ((last / NS) & 1));
        }
    }
}

template <int TYPE, bool GLU>
cudaError_t launch_stream_t(const GemvArgs &a, cudaStream_t s) {
    auto kern = mmid_stream_kernel<TYPE, GLU>;
    const size_t smem = (size_t) a.ring_off + (size_t) a.nslot * a.slot;
    static DeviceSmemLimit limit;
    {
        cudaError_t e = ensure_dyn_smem(kern, smem, limit);
        if (e != cudaSuccess) return e;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(num_sms());
    cfg.blockDim = dim3(32 * (a.nwarps + 1));
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

// Lane layout, staged activation rows, consumer warps and stage size for the streaming
// kernel: a warp-step is RPW rows (LPR lanes per row), a stage NWC warp-steps, and
// kStreamDepth stages plus TG staged activation rows must fit the shared-memory budget.
// Returns false when not even two warp-steps fit (very long rows); the caller then keeps
// the staged GEMV kernel.
bool stream_geometry(GemvArgs &a, int type, bool glu) {
    const bool kq = type != QWB_TYPE_Q8_0;
    a.upg = kq ? 8 : 4;
    a.act_dstride = (int) plane_d_stride(a.K, kq ? QK_K : QK8_0);
    a.act_bstride = kq ? (int) plane_bsum_stride(a.K) : 0;
    // staged row: qs groups of 256 (Q8_K) / 128 (Q8_0) bytes each followed by 16 spare
    // bytes, the d plane, then (Q8_K) 48 bytes per superblock of bsums
    const int64_t qgroup = kq ? QK_K : 128;
    const int64_t qs_bytes = ceil_div(a.K, qgroup) * (qgroup + 16);
    a.act_d_off = (int) qs_bytes;
    a.act_b_off = (int) (qs_bytes + a.act_dstride * 4);
    a.act_stride = (int) align_up((size_t) (a.act_b_off + (kq ? (a.K / QK_K) * 48 : 0)), 16);
    a.tg = (int) std::min<size_t>(kStreamTok, kStreamActBudget / (size_t) a.act_stride);
    if (a.tg < 1) return false;
    const int units = (int) (a.K / 32);
    const int n_sb = (units + a.upg - 1) / a.upg;
    int lpr = 1;
    while (lpr < n_sb && lpr < 32) lpr <<= 1;
    a.lpr = lpr;
    a.rpw = 32 / lpr;
    const size_t nb = glu ? std::max(a.nb1, a.nb1_2) : a.nb1;
    auto slot_bytes = [&](int nw) {
        const size_t one = align_up((size_t) (nw * a.rpw - 1) * nb + a.row_bytes + 32, 16);
        return align_up(one * (glu ? 2 : 1), 128);
    };
    const size_t head = align_up((size_t) kStreamDepth * (8 + 8 + sizeof(StreamDesc)) + 16 + kStreamTok * 12, 128);
    const size_t act = align_up((size_t) a.tg * a.act_stride, 128);
    const size_t ring_budget = kStreamSmemBudget - head - act;
    int nw = kStreamMaxWarps;
    while (nw > 1 && kStreamDepth * slot_bytes(nw) > ring_budget) --nw;
    if (nw < 2) return false;
    a.nwarps = nw;
    a.slot = (int) slot_bytes(nw);
    a.nslot = kStreamDepth;
    a.act_off = (int) head;
    a.ring_off = (int) (head + act);
    return true;
}

#ifdef QWB_STREAM_TRACE
extern "C" QWB_API int qwb_debug_stream_trace(void *host, size_t bytes) {
    return (int) cudaMemcpyFromSymbol(host, g_stream_trace, bytes < sizeof(g_stream_trace) ? bytes : sizeof(g_stream_trace));
}
#endif

bool stream_fits(int type, int64_t K, size_t nb1, size_t nb1_2, bool glu) {
    if (K <= 0 || K % 32) return false;
    GemvArgs a{};
    a.K = K;
    a.nb1 = nb1;
    a.nb1_2 = nb1_2;
    a.row_bytes = row_bytes(type, K);
    return stream_geometry(a, type, glu);
}

bool stream_fits_ffn(int type_gu, int64_t H, size_t nb_g, size_t nb_u, int type_d, int64_t F, size_t nb_d) {
    // the Q6_K gate/up (GLU) variant does not fit the register budget: staged GEMV there
    return type_gu != QWB_TYPE_Q6_K && stream_fits(type_gu, H, nb_g, nb_u, true) &&
           stream_fits(type_d, F, nb_d, nb_d, false);
}

cudaError_t launch_expert_gemv(int type, bool glu, GemvArgs a, bool stream, int NT, int max_tiles, int64_t pairs,
                               int64_t n_experts, int *work, cudaStream_t s) {
    if (stream) {
        a.chunks_per_cta = 2 * pairs > 3 * std::min(pairs, n_experts) ? 8 : 4;
        a.work = work;
        if (!stream_geometry(a, type, glu)) return cudaErrorInvalidValue;
        return launch_stream(type, glu, a, s);
    }
    gemv_geometry(a, NT, glu);
    return launch_gemv(type, glu, a, NT, max_tiles, s);
}

cudaError_t launch_stream(int type, bool glu, const GemvArgs &a, cudaStream_t s) {
    if (a.nwarps < 1 || a.nwarps > kStreamMaxWarps) return cudaErrorInvalidConfiguration;
    if (glu) {
        switch (type) {
            case QWB_TYPE_Q4_K: return launch_stream_t<QWB_TYPE_Q4_K, true>(a, s);
            case QWB_TYPE_Q6_K: return launch_stream_t<QWB_TYPE_Q6_K, true>(a, s);
            default: return launch_stream_t<QWB_TYPE_Q8_0, true>(a, s);
        }
    }
    switch (type) {
        case QWB_TYPE_Q4_K: return launch_stream_t<QWB_TYPE_Q4_K, false>(a, s);
        case QWB_TYPE_Q6_K: return launch_stream_t<QWB_TYPE_Q6_K, false>(a, s);
        default: return launch_stream_t<QWB_TYPE_Q8_0, false>(a, s);
    }
}

}  // namespace qwb
