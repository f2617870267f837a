// kernels.cuh - declarations shared between the qwb translation units.
#pragma once

#include "common.cuh"

namespace qwb {

// Every workspace starts with this many bytes of control words (the fused router's
// completion counter).  They must be zero before the first call on a workspace and are
// left at zero by every kernel.
constexpr size_t kCtrlBytes = 256;

// q8-plane row strides (elements), padded to 16 bytes so each plane row is a whole
// number of 16-byte units (bulk-copyable)
__host__ __device__ inline int64_t plane_d_stride(int64_t K, int blk) { return (int64_t) align_up((size_t) (K / blk), 4); }
__host__ __device__ inline int64_t plane_bsum_stride(int64_t K) { return (int64_t) align_up((size_t) (K / 16), 8); }

// bytes of q8 planes for n_rows rows of length K (vec-dot type: Q8_K when kq, else Q8_0)
inline size_t planes_bytes(int64_t n_rows, int64_t K, bool kq) {
    size_t b = align_up((size_t) (n_rows * K), 256);
    b += align_up((size_t) n_rows * plane_d_stride(K, kq ? QK_K : QK8_0) * 4, 256);
    if (kq) b += align_up((size_t) n_rows * plane_bsum_stride(K) * 2, 256);
    return b;
}
inline Q8Planes planes_at(void *base, int64_t n_rows, int64_t K, bool kq) {
    Q8Planes p;
    char *c = (char *) base;
    p.K = K;
    p.qs = (int8_t *) c;
    c += align_up((size_t) (n_rows * K), 256);
    p.d = (float *) c;
    c += align_up((size_t) n_rows * plane_d_stride(K, kq ? QK_K : QK8_0) * 4, 256);
    p.bsum = kq ? (int16_t *) c : nullptr;
    return p;
}

// kind: 0 = Q8_K, 1 = Q8_0 (CPU variant), 2 = Q8_0 (ref variant).  Either output may be
// null.  row_map (device, optional): source row of output row r.
cudaError_t launch_quantize_rows(int kind, const float *x, int64_t x_stride, int64_t n_rows, int64_t K,
                                 uint8_t *packed, Q8Planes planes, const int32_t *row_map, cudaStream_t s);

int num_sms();

// cudaFuncSetAttribute changes a kernel's attribute on the current device only, so a
// process that drives several GPUs must set it on each.  A launcher keeps one of these
// per kernel: the largest dynamic shared-memory limit it has set, per device.
constexpr int kAttrDevices = 64;
struct DeviceSmemLimit {
    size_t bytes[kAttrDevices] = {};
};
template <class Kernel>
inline cudaError_t ensure_dyn_smem(Kernel kern, size_t smem, DeviceSmemLimit &limit) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kAttrDevices) return cudaErrorInvalidDevice;
    if (smem <= limit.bytes[dev]) return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int) smem);
    if (e == cudaSuccess) limit.bytes[dev] = smem;
    return e;
}

// records a profiling mark when qwb_profile_enable is active (api.cu)
void profile_mark(cudaStream_t s, int tag);

}  // namespace qwb
