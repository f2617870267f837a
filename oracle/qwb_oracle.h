/* qwb_oracle.h - CPU restatement of the reference's quantized MoE hot path.
 *
 * TEST INFRASTRUCTURE ONLY: tests/, __graft_entry__.smoke() and bench.py's
 * cpu_baseline leg use this as the checker.  The product (questwend_b200/) never
 * links or calls it.
 *
 * Every function restates the algorithm of a reference function (vendored ggml,
 * llama.cpp 1b70350c9, paths relative to third_party/ggml/src), cited per function
 * in qwb_oracle.c.  Parity of this restatement with the reference itself is pinned by
 * tests/test_oracle_pin.py against the reference's ggml CPU backend compiled from its
 * own sources (oracle/_ref) and against committed golden fixtures (tests/golden).
 *
 * Type ids are ggml's enum ggml_type values.
 */
#ifndef QWB_ORACLE_H
#define QWB_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
    QO_TYPE_F32 = 0, QO_TYPE_F16 = 1, QO_TYPE_Q8_0 = 8, QO_TYPE_Q4_K = 12,
    QO_TYPE_Q6_K = 14, QO_TYPE_Q8_K = 15, QO_TYPE_I32 = 26,
};

/* Q8_0 activation quantizer variants */
enum { QO_Q8_0_CPU = 0, /* arch/x86/quants.c:302 (what the CPU backend feeds its dots) */
       QO_Q8_0_REF = 1  /* ggml-quants.c:276 quantize_row_q8_0_ref */ };

size_t   qo_row_size(int type, int64_t n);
uint16_t qo_fp32_to_fp16(float f);
float    qo_fp16_to_fp32(uint16_t h);

/* weight quantizers (no importance matrix), as ggml_quantize_chunk uses them */
int  qo_quantize_weights(int type, const float *src, void *dst, int64_t nrow, int64_t n_per_row);
/* activation quantizers as the CPU backend's from_float */
void qo_quantize_row_q8_K(const float *x, void *y, int64_t k);
void qo_quantize_row_q8_0(const float *x, void *y, int64_t k, int variant);
/* dequantize nrow rows of k values */
int  qo_to_float(int type, const void *x, float *y, int64_t nrow, int64_t k);

/* dot of one weight row (type) with one activation row in the type's vec_dot_type */
float qo_vec_dot(int type, int64_t k, const void *w_row, const void *act_row);

/* dst[M, n_used, T] = mul_mat_id(as[K, M, n_as] (type), b[K, n_b, T] f32, ids[n_used, T])
 * ids element (slot j, token t) at ids[t*ids_stride + j].  Returns 0, or -1 on an id out of
 * range (the reference asserts; the restatement reports). */
int qo_mul_mat_id(int type, const void *as, int64_t K, int64_t M, int64_t n_as,
                  const float *b, int64_t n_b, int64_t T,
                  const int32_t *ids, int64_t n_used, int64_t ids_stride,
                  float *dst, int q8_0_variant);

/* dst[ne0, n] = get_rows(src[ne0, nrows], idx[n]); dst f32 (I32 src -> I32 dst) */
int qo_get_rows(int type, const void *src, int64_t ne0, int64_t nrows,
                const int32_t *idx, int64_t n, void *dst);

/* route_experts: softmax -> top-k (descending, ties by lower index) -> gather ->
 * renorm (sum clamped to >= 6.103515625e-5) -> optional scale. mask may be NULL. */
void qo_route(const float *logits, int64_t E, int64_t T, int64_t n_used, int norm, float scale,
              const float *mask, int32_t *selected, float *weights);

/* act[F, n_used, T] = silu(gate) * up, elementwise */
void qo_swiglu(const float *gate, const float *up, float *act, int64_t n);

/* Full MoE FFN layer (build_moe): router GEMV f32, route, 3x mul_mat_id, swiglu, weighted
 * reduce.  g2s (3 x E, gate/up/down) remaps expert ids to pool slots when non-NULL.
 * out[H, T]; selected/weights[n_used, T] and act[F, n_used, T] optional. */
int qo_moe_layer(const float *x, int64_t H, int64_t T,
                 const float *router_w, int64_t E, int64_t n_used,
                 int type_gu, const void *gate, const void *up,
                 int type_d, const void *down, int64_t F, int64_t n_mat,
                 const int32_t *g2s, const float *mask,
                 float *out, int32_t *selected, float *weights, float *act_out);

/* ggml_rms_norm(x, eps) * w per row of H (ggml-cpu/ops.cpp:4107-4162) */
void qo_rms_norm_mul(const float *x, const float *w, float eps, int64_t T, int64_t H, float *y);

/* Expert pool byte audit: FNV-1a 64 (core/expert_weight_audit.h:83-87) and the audit
 * record of ExpertWeightAudit::compare (:106-125): equal flag, first differing byte (n
 * when equal), the two bytes there, both checksums. */
uint64_t qo_fnv1a64(const uint8_t *p, size_t n);
void qo_slab_audit(const uint8_t *expected, const uint8_t *actual, size_t n, int32_t *equal,
                   uint64_t *first_difference, uint32_t *expected_byte, uint32_t *actual_byte,
                   uint64_t *expected_fnv, uint64_t *actual_fnv);

#ifdef __cplusplus
}
#endif
#endif
