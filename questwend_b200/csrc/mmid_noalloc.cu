// mmid_noalloc.cu - MUL_MAT_ID for callers that cannot allocate device memory.
//
// qwb_mul_mat_id needs a caller-provided workspace (quantized activation rows and the
// expert-sorted index).  Some callers have no way to provide one: a ggml backend's
// graph_compute may not allocate, a plugin running inside another framework's CUDA
// graph capture cannot call cudaMalloc (it is not capturable), and a host that has
// handed all device memory to its expert-slot pool has nothing left to carve from.
// qwb_mul_mat_id_noalloc serves them from a fixed scratch array that lives in this
// library's own device image: the CUDA driver reserves it when the library's kernels are
// loaded on a device and it stays reserved until the process exits.  No call here
// allocates: there is no cudaMalloc, cudaFree or allocating library routine.
//
// Contract (also in include/qwb.h):
//   - it always takes the GEMV / weight-streaming kernels, and the scratch holds at most
//     QWB_NOALLOC_SCRATCH_BYTES: a problem whose workspace for that plan is larger is
//     rejected with QWB_ERR_LIMIT (qwb_mul_mat_id_workspace_size also plans for the
//     tensor-core GEMMs, so it can report more for a problem this entry point accepts);
//   - the address lookup below is cached per device for the life of the process: do not
//     use this entry point on a device across a cudaDeviceReset of it;
//   - every call on a device shares the one array and it keeps the previous call's
//     contents; the kernels write every byte they later read, so nothing needs
//     clearing between calls, but calls whose executions overlap on the GPU (different
//     streams, no ordering between them) race on it and must be serialised by the caller;
//   - the first call on a device looks up the array's device address for that device
//     (cudaGetSymbolAddress, with the device current); make that first call before any
//     stream capture.
#include <mutex>

#include "common.cuh"
#include "kernels.cuh"
#include "mmid.cuh"

namespace qwb {

// The scratch array.  In host code `g_noalloc_scratch` names a host-side shadow, not
// device memory: host code must use the address cudaGetSymbolAddress returns.
static __device__ __align__(256) uint8_t g_noalloc_scratch[QWB_NOALLOC_SCRATCH_BYTES];

namespace {
constexpr int kMaxDevices = 64;
std::mutex g_mu;
void *g_scratch_ptr[kMaxDevices] = {};
}  // namespace

static qwb_status noalloc_scratch(void **out) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return QWB_ERR_CUDA;
    if (dev < 0 || dev >= kMaxDevices) return QWB_ERR_DEVICE;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_scratch_ptr[dev]) {
        void *p = nullptr;
        // with `dev` current: the address of this device's copy of the array
        if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return QWB_ERR_CUDA;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return QWB_OK;
}

}  // namespace qwb

extern "C" QWB_API qwb_status qwb_mul_mat_id_noalloc(const qwb_tensor *as, const qwb_tensor *b,
                                                     const qwb_tensor *ids, const qwb_tensor *dst,
                                                     qwb_status_block *d_status, qwb_stream_t stream) {
    // the GEMV path at every size: its workspace stays small enough for the scratch array
    const size_t need = qwb::mul_mat_id_workspace(as, b, ids, false);
    if (need == 0) {
        // malformed arguments: let the regular entry point report the precise status
        return qwb::mul_mat_id_impl(as, b, ids, dst, nullptr, 0, d_status, (cudaStream_t) stream, false);
    }
    if (need > (size_t) QWB_NOALLOC_SCRATCH_BYTES) return QWB_ERR_LIMIT;
    void *scratch = nullptr;
    const qwb_status rc = qwb::noalloc_scratch(&scratch);
    if (rc != QWB_OK) return rc;
    return qwb::mul_mat_id_impl(as, b, ids, dst, scratch, (size_t) QWB_NOALLOC_SCRATCH_BYTES, d_status,
                                (cudaStream_t) stream, false);
}
