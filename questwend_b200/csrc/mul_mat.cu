// mul_mat.cu - quantized GGML_OP_MUL_MAT: the shared expert and dense FFN matrices
// (core/runtime.cpp:2825-2833) and the output head (runtime.cpp:3037), on the MUL_MAT_ID
// kernels as one expert that every token selects.
//
// Reference: ggml_compute_forward_mul_mat (ggml-cpu/ggml-cpu.c:1255-1470), op contract
// ggml_mul_mat (ggml.c:3362-3377): dst[:, n] = a[:, :] . b[:, n] with b quantized to the
// weight type's vec_dot type exactly as the CPU backend does.  The same dots as
// MUL_MAT_ID, so the results match the CPU backend to the same fp32 summation-order
// tolerance; few tokens take the weight-streaming kernel (every weight row read once for
// all tokens), many tokens on Q4_K the tensor-core grouped GEMM.
#include <cuda_runtime.h>

#include "common.cuh"
#include "kernels.cuh"
#include "mmid.cuh"

namespace {

struct MmViews {
    qwb_tensor as, b, ids, dst;
    size_t ids_bytes;
};

// a [K, M] -> as [K, M, 1]; b [K, T] -> [K, 1, T]; ids [1, T] (zeros, in the workspace);
// dst [M, T] -> [M, 1, T].  Only the 2-D form (no batch dimensions).
qwb_status mm_views(const qwb_tensor *a, const qwb_tensor *b, const qwb_tensor *dst, MmViews &v) {
    if (!a || !b) return QWB_ERR_INVALID_ARG;
    for (int i = 0; i < 4; ++i)
        if (a->ne[i] < 0 || b->ne[i] < 0) return QWB_ERR_INVALID_ARG;
    if (a->ne[2] != 1 || a->ne[3] != 1 || b->ne[2] != 1 || b->ne[3] != 1) return QWB_ERR_SHAPE;
    if (b->ne[0] != a->ne[0]) return QWB_ERR_SHAPE;
    const int64_t M = a->ne[1], T = b->ne[1];
    v.as = *a;
    v.as.nb[2] = a->nb[1] * (size_t) (M > 0 ? M : 1);
    v.as.nb[3] = v.as.nb[2];
    v.b = *b;
    v.b.ne[1] = 1;
    v.b.ne[2] = T;
    v.b.nb[2] = b->nb[1];
    v.b.nb[3] = b->nb[1] * (size_t) (T > 0 ? T : 1);
    v.ids = qwb_tensor{};
    v.ids.type = QWB_TYPE_I32;
    v.ids.ne[0] = 1;
    v.ids.ne[1] = T;
    v.ids.ne[2] = v.ids.ne[3] = 1;
    v.ids.nb[0] = v.ids.nb[1] = 4;
    v.ids.nb[2] = v.ids.nb[3] = (size_t) 4 * (T > 0 ? T : 1);
    v.ids_bytes = qwb::align_up((size_t) (T > 0 ? T : 1) * 4, 256);
    if (dst) {
        if (dst->ne[0] != M || dst->ne[1] != T || dst->ne[2] != 1 || dst->ne[3] != 1) return QWB_ERR_SHAPE;
        v.dst = *dst;
        v.dst.ne[1] = 1;
        v.dst.ne[2] = T;
        v.dst.nb[2] = dst->nb[1];
        v.dst.nb[3] = dst->nb[1] * (size_t) (T > 0 ? T : 1);
    }
    return QWB_OK;
}

}  // namespace

extern "C" QWB_API size_t qwb_mul_mat_workspace_size(const qwb_tensor *a, const qwb_tensor *b) {
    MmViews v;
    if (mm_views(a, b, nullptr, v) != QWB_OK) return 0;
    const size_t w = qwb::mul_mat_id_workspace(&v.as, &v.b, &v.ids, true);
    return w ? v.ids_bytes + w : 0;
}

extern "C" QWB_API qwb_status qwb_mul_mat(const qwb_tensor *a, const qwb_tensor *b, const qwb_tensor *dst,
                                          void *workspace, size_t workspace_bytes, qwb_status_block *d_status,
                                          qwb_stream_t stream) {
    MmViews v;
    if (!dst) return QWB_ERR_INVALID_ARG;
    qwb_status rc = mm_views(a, b, dst, v);
    if (rc != QWB_OK) return rc;
    if (b->ne[1] == 0 || a->ne[1] == 0) return QWB_OK;
    if (!workspace || workspace_bytes < v.ids_bytes) return QWB_ERR_WORKSPACE;
    if ((uintptr_t) workspace % 256) return QWB_ERR_ALIGNMENT;
    cudaStream_t s = (cudaStream_t) stream;
    // every token selects expert 0: the ids column is zeros
    if (cudaMemsetAsync(workspace, 0, (size_t) b->ne[1] * 4, s) != cudaSuccess) return QWB_ERR_CUDA;
    v.ids.data = workspace;
    return qwb::mul_mat_id_impl(&v.as, &v.b, &v.ids, &v.dst, (char *) workspace + v.ids_bytes,
                                workspace_bytes - v.ids_bytes, d_status, s, true);
}
