/* qwb.h - C ABI of the B200 (sm_100a) kernel library for QuestWend's quantized MoE
 * expert hot path.
 *
 * What this library replaces.  QuestWend builds ggml graphs whose MoE nodes are
 * GGML_OP_MUL_MAT_ID (ggml.c:3401-3437 op contract) on Q4_K / Q6_K / Q8_0 expert weights
 * and GGML_OP_GET_ROWS (ggml.c:3975-3996), and hands them to a ggml backend through the
 * backend C ABI (ggml-backend-impl.h:122-247).  The entry points below are what a ggml
 * backend for B200 binds from its graph_compute: each names the reference function whose
 * result it reproduces (paths relative to the reference's third_party/ggml/src unless
 * they start with core/).  The ggml backend shim that registers these with ggml is
 * include/qwb_ggml_backend.h.
 *
 * Conventions
 *   - Plain pointers and sizes; tensors are described by qwb_tensor, a copy of the
 *     fields of struct ggml_tensor the kernels need (type, ne[4], nb[4] in bytes, data).
 *     Type ids are ggml's enum ggml_type values.
 *   - Every call is asynchronous on the given cudaStream_t (pass 0 for the legacy
 *     default stream), performs no host synchronisation, no device allocation and no
 *     host read-back of device data, so it can be captured in a CUDA graph.
 *   - Scratch memory is caller-owned ("workspace"); sizes come from the *_workspace_size
 *     queries.  Workspaces must be 256-byte aligned, and their first 256 bytes (a control
 *     block of the fused MoE layer's kernels, which leave it zeroed) must be zero before
 *     the first call that uses them: clear a new workspace once.
 *   - Host-detectable errors (bad type, shape, stride, alignment, workspace) return a
 *     qwb_status and launch nothing.  Data-dependent errors found on the device (an
 *     expert / row id out of range) never fault: the kernel skips the access, writes
 *     zeros for the affected outputs and records the error in an optional device-side
 *     qwb_status_block, read back with qwb_status_block_read.  (The reference's CPU
 *     backend aborts on such ids, ggml-cpu.c:1659 / ops.cpp get_rows asserts.)
 */
#ifndef QWB_H
#define QWB_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(_WIN32)
#define QWB_API __declspec(dllexport)
#else
#define QWB_API __attribute__((visibility("default")))
#endif

typedef struct CUstream_st *qwb_stream_t; /* == cudaStream_t */

#define QWB_ABI_VERSION 1

typedef enum qwb_status {
    QWB_OK = 0,
    QWB_ERR_INVALID_ARG = 1,      /* null pointer, negative size */
    QWB_ERR_UNSUPPORTED_TYPE = 2, /* tensor type not handled by this entry point */
    QWB_ERR_SHAPE = 3,            /* shapes inconsistent with the op contract */
    QWB_ERR_LAYOUT = 4,           /* unsupported strides (permuted / non-contiguous rows) */
    QWB_ERR_ALIGNMENT = 5,        /* pointer or row stride not aligned as required */
    QWB_ERR_WORKSPACE = 6,        /* workspace missing or smaller than required */
    QWB_ERR_CUDA = 7,             /* a CUDA runtime call failed (launch, attribute) */
    QWB_ERR_DEVICE = 8,           /* device not sm_100 */
    QWB_ERR_LIMIT = 9,            /* size beyond a documented maximum */
} qwb_status;

/* ggml_type values used on this path */
enum {
    QWB_TYPE_F32 = 0, QWB_TYPE_F16 = 1, QWB_TYPE_Q8_0 = 8, QWB_TYPE_Q4_K = 12,
    QWB_TYPE_Q6_K = 14, QWB_TYPE_Q8_K = 15, QWB_TYPE_I32 = 26,
};

/* A tensor view with ggml semantics: ne[] element counts, nb[] byte strides. */
typedef struct qwb_tensor {
    void *data;
    int32_t type;
    int32_t reserved;
    int64_t ne[4];
    size_t nb[4];
} qwb_tensor;

/* Device-resident error record.  Allocate it zeroed in device memory; kernels OR flags
 * into it and keep the first offending value.  It is sticky until reset. */
typedef struct qwb_status_block {
    uint32_t flags;       /* QWB_DEVERR_* bits */
    int32_t bad_value;    /* first offending id / row index seen */
    uint32_t count;       /* number of offending accesses */
    uint32_t reserved;
} qwb_status_block;

#define QWB_DEVERR_ID_RANGE 0x1u      /* mul_mat_id expert/slot id outside [0, n_as) */
#define QWB_DEVERR_ROW_RANGE 0x2u     /* get_rows index outside [0, nrows) */
#define QWB_DEVERR_TIMEOUT 0x4u       /* a bounded device wait gave up (copy never landed) */

QWB_API int qwb_abi_version(void);
QWB_API const char *qwb_status_string(qwb_status s);

/* Synchronises `stream`, copies the block to *out and, when reset != 0, zeroes it. */
QWB_API qwb_status qwb_status_block_read(qwb_status_block *d_block, qwb_status_block *out,
                                         int reset, qwb_stream_t stream);

/* ---------------------------------------------------------------- quantizers
 * Activation quantizers, bit-exact with the reference CPU backend's from_float for the
 * weight type's vec_dot_type (ggml-cpu.c:1609-1644 applies them to src1 rows).
 * x: n_rows rows of k floats, row r at x + r*x_row_stride (elements).  y: packed ggml
 * blocks, row r at y + r*row_size(k).  k % 256 == 0 (Q8_K) / k % 32 == 0 (Q8_0). */

/* replaces quantize_row_q8_K (ggml-cpu/arch/x86/quants.c:505 -> ggml-quants.c:2769-2806) */
QWB_API qwb_status qwb_quantize_row_q8_K(const float *x, void *y, int64_t n_rows, int64_t k,
                                         int64_t x_row_stride, qwb_stream_t stream);

#define QWB_Q8_0_CPU 0 /* ggml-cpu/arch/x86/quants.c:302-360: id = 127/amax, round-half-even */
#define QWB_Q8_0_REF 1 /* ggml-quants.c:276-300 quantize_row_q8_0_ref: id = 1/d, roundf     */
/* replaces quantize_row_q8_0 (x86 CPU backend) or quantize_row_q8_0_ref */
QWB_API qwb_status qwb_quantize_row_q8_0(const float *x, void *y, int64_t n_rows, int64_t k,
                                         int64_t x_row_stride, int variant, qwb_stream_t stream);

/* ----------------------------------------------------------------- GET_ROWS
 * replaces ggml_compute_forward_get_rows (ggml-cpu/ops.cpp:5371) incl. get_rows_q
 * (ops.cpp:5204-5240); op contract ggml.c:3975-3996.
 * src0 [ne0, ne01, ne02, ne03] of Q4_K | Q6_K | Q8_0 | F16 | F32 | I32;
 * idx  [n, ne11, ne12] I32 (row ids into src0's ne01, broadcast over ne02 like ggml);
 * dst  [ne0, n, ne11, ne12] F32 (I32 when src0 is I32).  Quantized and F16 rows are
 * dequantized bit-exactly; F32/I32 rows are copied bit-for-bit. */
QWB_API qwb_status qwb_get_rows(const qwb_tensor *src0, const qwb_tensor *idx,
                                const qwb_tensor *dst, qwb_status_block *d_status,
                                qwb_stream_t stream);

/* --------------------------------------------------------------- MUL_MAT_ID
 * replaces ggml_compute_forward_mul_mat_id (ggml-cpu/ggml-cpu.c:1554-1736); op contract
 * ggml.c:3401-3437:
 *   as  [K, M, n_as]      Q4_K | Q6_K | Q8_0 (n_as may be a slot-pool size, ids slot ids)
 *   b   [K, n_b, T]       F32, n_used % n_b == 0 (n_b == 1 broadcasts one row per token)
 *   ids [n_used, T]       I32, may be a strided view (nb[1] != n_used*4)
 *   dst [M, n_used, T]    F32
 * dst[:, j, t] = as[:, :, ids[j, t]] . b[:, j % n_b, t], with b quantized exactly as the
 * CPU backend does (Q8_K for K-quants, Q8_0 CPU variant for Q8_0). */
QWB_API size_t qwb_mul_mat_id_workspace_size(const qwb_tensor *as, const qwb_tensor *b,
                                             const qwb_tensor *ids);
QWB_API qwb_status qwb_mul_mat_id(const qwb_tensor *as, const qwb_tensor *b, const qwb_tensor *ids,
                                  const qwb_tensor *dst, void *workspace, size_t workspace_bytes,
                                  qwb_status_block *d_status, qwb_stream_t stream);

/* MUL_MAT_ID without a workspace, for callers that cannot allocate device memory: a
 * ggml backend inside graph_compute, code running under another framework's CUDA graph
 * capture (where cudaMalloc is not allowed), or a host whose device memory is all
 * committed to its expert-slot pool.  This entry point has no counterpart in the
 * reference.  It always runs the GEMV / weight-streaming kernels (never the tensor-core
 * GEMMs that qwb_mul_mat_id picks for many tokens per expert), so its results match
 * qwb_mul_mat_id's to within fp32 summation order; its scratch is a fixed array of
 * QWB_NOALLOC_SCRATCH_BYTES that the library's device image carries (the CUDA driver
 * reserves it on every GPU that loads the library, until the process exits).
 *   - The limit applies to the workspace of that GEMV plan.  qwb_mul_mat_id_workspace_size
 *     returns the larger of that plan and the tensor-core one, so a problem it sizes at or
 *     below QWB_NOALLOC_SCRATCH_BYTES is always accepted; a larger one may still be.
 *     Problems beyond the limit return QWB_ERR_LIMIT before any work is queued.
 *   - All calls on a device share the array, which keeps the last call's contents (every
 *     byte a call reads it has written first); calls that overlap on the GPU race on it,
 *     so the caller must order them (one stream, or events).
 *   - The first call on each device resolves the array's address with that device
 *     current and keeps it for the life of the process; make it before any stream
 *     capture, and do not use this entry point across a cudaDeviceReset of that device
 *     (the array may be reloaded at another address).
 * No cudaMalloc, cudaFree or other allocating call is made. */
#define QWB_NOALLOC_SCRATCH_BYTES (8u << 20) /* 8 MiB per device */
QWB_API qwb_status qwb_mul_mat_id_noalloc(const qwb_tensor *as, const qwb_tensor *b,
                                          const qwb_tensor *ids, const qwb_tensor *dst,
                                          qwb_status_block *d_status, qwb_stream_t stream);

/* ------------------------------------------------------------------ MUL_MAT
 * replaces ggml_compute_forward_mul_mat (ggml-cpu/ggml-cpu.c:1255-1470) for quantized
 * weights; op contract ggml_mul_mat (ggml.c:3362-3377).  The shared expert and dense FFN
 * matrices (core/runtime.cpp:2825-2833) and the output head (runtime.cpp:3037):
 *   a   [K, M]   Q4_K | Q6_K | Q8_0 (rows contiguous blocks, no batch dimensions)
 *   b   [K, T]   F32 (rows contiguous)
 *   dst [M, T]   F32
 * dst[:, t] = a . b[:, t], b quantized exactly as the CPU backend does (Q8_K / Q8_0-cpu).
 * Same kernels and tolerance as qwb_mul_mat_id (one expert that every token selects). */
QWB_API size_t qwb_mul_mat_workspace_size(const qwb_tensor *a, const qwb_tensor *b);
QWB_API qwb_status qwb_mul_mat(const qwb_tensor *a, const qwb_tensor *b, const qwb_tensor *dst,
                               void *workspace, size_t workspace_bytes, qwb_status_block *d_status,
                               qwb_stream_t stream);

/* ------------------------------------------------------------ small MoE ops */
/* replaces the route_experts subgraph (core/runtime.cpp:2693-2734): soft_max
 * (ops.cpp:5813) -> argsort_top_k (ggml.c:5462) -> get_rows of probs -> sum_rows ->
 * clamp(6.103515625e-5) -> div -> optional scale.  logits [E, T] f32 rows contiguous;
 * mask [E, T] f32 or NULL (added to logits first); selected [n_used, T] i32 and
 * weights [n_used, T] f32, both contiguous.  E <= 512, n_used <= 32. */
QWB_API qwb_status qwb_moe_route(const float *logits, const float *mask, int64_t E, int64_t T,
                                 int64_t n_used, int norm, float scale, int32_t *selected,
                                 float *weights, qwb_stream_t stream);

/* replaces ggml_swiglu_split (ggml.c:3082; ops.cpp:3331-3389): act = silu(gate) * up,
 * n contiguous floats. */
QWB_API qwb_status qwb_swiglu(const float *gate, const float *up, float *act, int64_t n,
                              qwb_stream_t stream);

/* replaces the weighted expert reduction (core/runtime.cpp:2796-2816:
 * T=1 mul_mat(cont(transpose(experts)), w), T>1 mul + (n_used-1) add):
 * out[:, t] = sum_j w[j, t] * experts[:, j, t]; experts [H, n_used, T] contiguous. */
QWB_API qwb_status qwb_moe_weighted_sum(const float *experts, const float *weights, float *out,
                                        int64_t H, int64_t n_used, int64_t T,
                                        qwb_stream_t stream);

/* ---------------------------------------------------------- fused MoE layer
 * replaces the whole build_moe subgraph (core/runtime.cpp:2743-2816, and the cached
 * fast path's slot remap :2769-2778), optionally with the ffn_norm that feeds it (:2979):
 *   x      = rms_norm(x) * norm_w    (when norm_w != NULL; ops.cpp:4107-4162)
 *   logits = router_w . x            (F32 mul_mat, :2750)
 *   selected, weights = route(...)   (as qwb_moe_route, norm on)
 *   slot_r = g2s[r][selected]        (r = gate, up, down; skipped when g2s == NULL)
 *   act    = swiglu(gate . x, up . x)  (mul_mat_id on the pools, Q8_K/Q8_0 activations)
 *   out    = sum_j w_j * (down . act_j) [+ residual]
 * Weight tensors may be slot pools [K, M, n_slots]. */
typedef struct qwb_moe_ffn_desc {
    const float *x;          /* [H, T] f32, contiguous rows */
    const float *router_w;   /* [H, E] f32 (ggml: ffn_gate_inp), contiguous */
    const float *mask;       /* [E, T] f32 added to logits, or NULL */
    const int32_t *g2s;      /* [3][E] i32 expert -> slot tables (gate, up, down), or NULL */
    qwb_tensor gate;         /* [H, F, n_mat] */
    qwb_tensor up;           /* [H, F, n_mat] */
    qwb_tensor down;         /* [F, H, n_mat] */
    int64_t H, F, E, n_used, T;
    const float *residual;   /* [H, T] added to out, or NULL */
    float *out;              /* [H, T] */
    int32_t *selected;       /* [n_used, T] out (logical expert ids), or NULL */
    float *weights;          /* [n_used, T] out, or NULL */
    float *act;              /* [F, n_used, T] out: swiglu(gate, up), the down projection's
                                input (ggml's "act" node), or NULL */
    const float *norm_w;     /* [H] ffn_norm weight, or NULL.  When set the layer input is
                                rms_norm(x, norm_eps) * norm_w (core/runtime.cpp:2979, the
                                ffn_in of build_moe), fused into the router kernel; the
                                residual is still added un-normalised. */
    float norm_eps;
    /* Shared expert (core/runtime.cpp:2825-2833), present when shexp_down.data != NULL:
     *   sh = shexp_down . (silu(shexp_gate . ffn_in) * (shexp_up . ffn_in)),
     *   times sigmoid(shexp_gate_inp . ffn_in) when shexp_gate_inp != NULL,
     * added to the routed experts' weighted sum before the residual.  shexp_gate / up have
     * the routed gate / up type, shexp_down the routed down type, rows contiguous and
     * 16-byte aligned.  With F_sh == F and up to 8 tokens it runs inside the routed
     * experts' gate/up and down kernels (one more (token, expert) pair per token). */
    qwb_tensor shexp_gate;   /* [H, F_sh] */
    qwb_tensor shexp_up;     /* [H, F_sh] */
    qwb_tensor shexp_down;   /* [F_sh, H] */
    const float *shexp_gate_inp; /* [H] f32, or NULL */
} qwb_moe_ffn_desc;

QWB_API size_t qwb_moe_ffn_workspace_size(const qwb_moe_ffn_desc *desc);
QWB_API qwb_status qwb_moe_ffn(const qwb_moe_ffn_desc *desc, void *workspace, size_t workspace_bytes,
                               qwb_status_block *d_status, qwb_stream_t stream);

/* ----------------------------------------------------- expert parallelism (EP)
 * The MoE layer split over N GPUs (no counterpart in the reference, whose multi-GPU
 * plan is a pipeline-style layer split, core/runtime.cpp:1551-1724; the arithmetic per
 * (token, slot) is build_moe's, core/runtime.cpp:2743-2816).  GPU g owns experts
 * [expert_lo, expert_lo + n_local) of every layer, and every GPU holds the hidden states
 * of all T tokens (identical copies).  Per layer:
 *   1. qwb_moe_ep_layer on every GPU: rms_norm * ffn_norm, router and top-k for all T
 *      tokens (replicated: the same ids and weights everywhere), then the SwiGLU expert
 *      FFN of ITS experts over the pairs routed to them:
 *        out[t] = sum over slots j with a local expert of weights[t][j] *
 *                 down(swiglu(gate x_t, up x_t))  (+ residual[t] when residual != NULL)
 *      (zero, or the residual, for a token with no local expert);
 *   2. the caller all-reduces out (sum, f32) over the N GPUs, passing the residual to
 *      exactly one of them: every GPU then holds the layer's output for all tokens.
 * One collective per layer.  Quantization is per row, so every GPU's activation bytes
 * equal a single-GPU run's; only the f32 summation order of the weighted expert outputs
 * differs from qwb_moe_ffn. */
typedef struct qwb_moe_ep_layer_desc {
    const float *x;          /* [T][H] all tokens' rows (the same on every GPU) */
    const float *norm_w;     /* [H] ffn_norm weight, or NULL (no normalisation) */
    float norm_eps;
    int32_t reserved;
    const float *router_w;   /* [E][H] f32 router */
    const float *mask;       /* [T][E] additive logit mask, or NULL */
    qwb_tensor gate, up, down; /* this GPU's experts: [H, F, n_local], [H, F, n_local], [F, H, n_local] */
    int64_t expert_lo;       /* global id of local expert 0 */
    int64_t H, F, E, n_used, T;
    const float *residual;   /* [T][H] added to out, or NULL */
    float *out;              /* [T][H] f32 partial sums (overwritten) */
    int32_t *selected;       /* out: [T][n_used] expert ids, descending probability, or NULL */
    float *weights;          /* out: [T][n_used] renormalised routing weights, or NULL */
    /* the shared expert, as in qwb_moe_ffn_desc: give it to exactly one GPU (the one
       adding the residual), shexp_down.data == NULL on the others */
    qwb_tensor shexp_gate, shexp_up, shexp_down;
    const float *shexp_gate_inp;
} qwb_moe_ep_layer_desc;
QWB_API size_t qwb_moe_ep_layer_workspace_size(const qwb_moe_ep_layer_desc *desc);
QWB_API qwb_status qwb_moe_ep_layer(const qwb_moe_ep_layer_desc *desc, void *workspace, size_t workspace_bytes,
                                    qwb_status_block *d_status, qwb_stream_t stream);

/* The per-layer all-reduce of the partial outputs over peer memory (NVLink / NVSwitch), an
 * alternative to the caller's NCCL all-reduce for decode-sized messages.  One process per
 * GPU of one node, up to 8 GPUs:
 *   1. qwb_ep_comm_create on every GPU (current device): allocates the exchange buffer
 *      (about 16 x max_bytes) and writes its CUDA IPC handle (qwb_ep_comm_handle_size()
 *      bytes) to handle_out;
 *   2. the caller gathers the handles of all GPUs in rank order (any host channel) and
 *      passes them to qwb_ep_comm_connect;
 *   3. qwb_ep_allreduce_f32 (stream-ordered, CUDA-graph capturable): out = the sum over
 *      GPUs of `in` (n floats, n % 4 == 0, 16-byte aligned, n * 4 <= max_bytes; in == out
 *      allowed), added in rank order so every GPU holds the same bits.  Every GPU must
 *      issue the same calls in the same order with the same n.  A peer that does not
 *      arrive within 5 s sets QWB_DEVERR_TIMEOUT in d_status and leaves out unwritten;
 *   4. qwb_ep_comm_destroy after the last call has completed. */
typedef struct qwb_ep_comm qwb_ep_comm;
QWB_API size_t qwb_ep_comm_handle_size(void);
QWB_API qwb_status qwb_ep_comm_create(int world, int rank, size_t max_bytes, qwb_ep_comm **comm, void *handle_out);
QWB_API qwb_status qwb_ep_comm_connect(qwb_ep_comm *comm, const void *handles);
QWB_API qwb_status qwb_ep_allreduce_f32(qwb_ep_comm *comm, const float *in, float *out, int64_t n,
                                        qwb_status_block *d_status, qwb_stream_t stream);
QWB_API void qwb_ep_comm_destroy(qwb_ep_comm *comm);

/* ------------------------------------------------------------- expert pool writes
 * The expert cache keeps each role's experts in a pool tensor [ne0, ne1, n_slots] (one
 * slab of nb[2] bytes per slot; the kernels above read it through slot ids).  A miss
 * copies one expert's slab from host memory into a slot:
 * ExpertCache::fetch_slab (core/expert_cache.cpp:637-723) and the group upload of
 * fetch_parallel (:1357-1377, from a page-locked staging buffer) call
 * ggml_backend_tensor_set(_async)(pool, src, slot * nb2, nb2) once per (role, expert),
 * after checking that the source's nb2 equals the pool's (:643-645, "slab size mismatch").
 *
 * qwb_pool_write_slabs issues those copies on `stream` for n slabs of one pool: copy i
 * writes pool->nb[2] bytes from copies[i].src into slot copies[i].slot, in array order
 * (a slot named twice ends with the later source).  When every source is readable by the
 * device (page-locked host memory from cudaHostAlloc / cudaHostRegister, or this device's
 * memory) and 16-byte aligned, one kernel launch gathers the whole group, reading the
 * sources directly; otherwise one cudaMemcpyAsync per slab (pageable sources are staged
 * by the driver), the odd slots on a second stream of the library's, forked from
 * `stream` and joined back into it with events.  A source inside the pool itself (a slot
 * copied to another slot) makes every copy run in array order on `stream`.  Either way,
 * work queued on `stream` after the call sees every slab.
 * Arguments are checked before the first copy is issued: src_slab_bytes must equal
 * pool->nb[2] (QWB_ERR_SHAPE), every slot must lie in [0, pool->ne[2])
 * (QWB_ERR_INVALID_ARG), so an error writes nothing. */
typedef struct qwb_slab_copy {
    const void *src; /* the slab's bytes (host or device memory) */
    int64_t slot;    /* destination slot in the pool */
} qwb_slab_copy;

QWB_API qwb_status qwb_pool_write_slabs(const qwb_tensor *pool, size_t src_slab_bytes,
                                        const qwb_slab_copy *copies, int n, qwb_stream_t stream);

/* Byte audit of pool slots, on the device.  The reference's audit
 * (core/expert_weight_audit.h:56-66 and :106-125, driven from
 * core/expert_cache.cpp:1712-1731) synchronises, reads every selected slot back to the
 * host and compares it with the authoritative bytes: equal flag, first differing byte
 * and the FNV-1a 64 checksums of both (:82-86).  qwb_pool_audit_slabs computes the same
 * record for n slots on the GPU, without reading the slabs back: expected[i].src holds
 * the bytes slot expected[i].slot should contain, in device memory or page-locked host
 * memory (read by the kernel over the host link; pageable host memory is rejected with
 * QWB_ERR_INVALID_ARG).  results[i] (device memory, n records) is written in stream
 * order; read it back after the stream.  checksums != 0 also computes both FNV-1a 64
 * sums, a serial chain over every byte (milliseconds per megabyte, a diagnostic);
 * checksums == 0 leaves them 0 and only compares, which runs at memory / host-link speed
 * and stops at the first difference. */
typedef struct qwb_slab_audit {
    int32_t equal;             /* 1 when the slot holds exactly the expected bytes */
    int32_t reserved;
    uint64_t first_difference; /* index of the first differing byte; the slab size when equal */
    uint32_t expected_byte;    /* the two bytes at first_difference (0 when equal) */
    uint32_t actual_byte;
    uint64_t expected_fnv1a64; /* FNV-1a 64 of the expected bytes (0 without checksums) */
    uint64_t actual_fnv1a64;   /* FNV-1a 64 of the slot's bytes (0 without checksums) */
} qwb_slab_audit;

QWB_API qwb_status qwb_pool_audit_slabs(const qwb_tensor *pool, const qwb_slab_copy *expected, int n,
                                        int checksums, qwb_slab_audit *results, qwb_stream_t stream);

/* ------------------------------------------------------------- profiling hook
 * Optional per-kernel timing for benchmarks (no counterpart in the reference, whose
 * QWEN_PROF timers are host wall-clock, core/runtime.cpp:3720).  While enabled,
 * qwb_moe_ffn and qwb_mul_mat_id record a CUDA event on their stream before the first
 * kernel ("mark" with tag 0) and after each kernel or group of preparation kernels
 * (tag = QWB_KERNEL_*).  Event records are stream-capture
 * safe: inside a captured CUDA graph they become event-record nodes and are re-recorded
 * on every replay, so after a replay qwb_profile_read returns that replay's durations.
 * Not thread-safe; one profiling session per process. */
#define QWB_KERNEL_ROUTER 1
#define QWB_KERNEL_GATE_UP 2
#define QWB_KERNEL_DOWN 3
#define QWB_KERNEL_OTHER 4
#define QWB_KERNEL_GROUPED_GEMM 5 /* tensor-core grouped expert GEMM (many tokens per expert) */
#define QWB_KERNEL_EXPERT_GEMV 6  /* bandwidth-bound expert GEMV of qwb_mul_mat_id (few tokens per expert) */
QWB_API qwb_status qwb_profile_enable(int max_marks); /* creates the events; 0 disables */
QWB_API qwb_status qwb_profile_reset(void);           /* next mark is mark 0 */
QWB_API int qwb_profile_count(void);                  /* marks recorded since reset */
/* ms[i] = time between mark i and mark i+1, tags[i] = tag of mark i+1, i < n <= count-1.
 * Synchronises on the last mark. */
QWB_API qwb_status qwb_profile_read(float *ms, int32_t *tags, int n);

#ifdef __cplusplus
}
#endif
#endif /* QWB_H */
