// ep_comm.cu - the expert-parallel layer's exchange: a one-shot all-reduce of the GPUs'
// partial layer outputs over peer memory (NVLink / NVSwitch), for the small messages of
// decode (T tokens x hidden f32: 8 KB to 1 MB).
//
// Each GPU allocates one exchange buffer, exports it with a CUDA IPC handle, and maps
// every peer's buffer (qwb_ep_comm_connect).  A buffer holds, for two alternating calls
// (parity = call number & 1), one slot per source GPU of 8-byte words: (call number << 32)
// | float bits, one word per element.  qwb_ep_allreduce_f32: CTA b of every GPU owns the
// same slice of the message and
//   1. writes each element of its input slice, tagged with the call number, into slot
//      [parity][own rank] of every GPU's buffer: one 64-bit peer store per element and
//      destination (a naturally aligned 64-bit access is seen whole or not at all, so the
//      tag validates the value in the same word: no fence, no separate flag);
//   2. reads slot [parity][r] of its own buffer for every source r, polling each word
//      until it carries the call number (bounded: QWB_DEVERR_TIMEOUT after kCommWaitNs),
//      and sums the sources in rank order 0..N-1, so every GPU computes the same bits.
// Two parities suffice: CTA b of a GPU can only start call k+2 (overwriting parity k's
// slice b on a peer) after every peer's CTA b has written call k+1, that is after it has
// finished reading call k's slice b.  The call number is kept per CTA in device memory
// (each CTA increments its own), so the kernel can be captured in a CUDA graph and
// replayed.  Launched with programmatic dependent launch: it starts while the kernel
// before it (the layer's down projection) finishes and waits for it on the device, and
// lets the kernel after it (the next layer's router) start prefetching at once.
// Every GPU must issue the same sequence of calls with the same size.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"
#include "kernels.cuh"

namespace qwb {
namespace {

constexpr int kCommMaxRanks = 8;
constexpr int kCommCtas = 32;                      // CTAs (slices) per call
constexpr int kCommThreads = 512;
constexpr uint64_t kCommWaitNs = 5000000000ull;    // 5 s: peers of one job, in lockstep

struct CommLayout {
    size_t slot;       // bytes of one source slot: 8 per element of the largest message
    size_t off_epoch;  // call counters [kCommCtas] uint32 (this GPU only)
    size_t total;
};
CommLayout comm_layout(size_t max_bytes) {
    CommLayout l{};
    l.slot = align_up(2 * max_bytes, 256);
    l.off_epoch = 2 * kCommMaxRanks * l.slot;
    l.total = l.off_epoch + align_up((size_t) kCommCtas * 4, 256);
    return l;
}

struct CommPeers {
    char *buf[kCommMaxRanks];  // every GPU's exchange buffer, mapped into this GPU's space
};

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

__global__ void __launch_bounds__(kCommThreads) ep_allreduce_kernel(const CommPeers peers, int world, int rank,
                                                                    size_t slot, size_t off_epoch,
                                                                    const float *in, float *out, int64_t n,
                                                                    qwb_status_block *st) {
    __shared__ uint32_t s_epoch;
    __shared__ int s_abort;
    volatile int *abort_flag = &s_abort;
    const int b = blockIdx.x, tid = threadIdx.x;
    char *own = peers.buf[rank];
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");  // the next kernel may prefetch
    // `in` is the previous kernel's output, and when that kernel is the previous call its
    // CTAs must have advanced their call numbers: read nothing before this wait
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (tid == 0) {
        uint32_t *ep = (uint32_t *) (own + off_epoch) + b;
        s_epoch = *ep + 1;  // this CTA's call number (only this CTA touches its counter)
        *ep = s_epoch;
        s_abort = 0;
    }
    __syncthreads();
    const uint64_t tag = (uint64_t) s_epoch << 32;
    const int par = (int) (s_epoch & 1u);
    const int64_t s0 = n * b / gridDim.x, s1 = n * (b + 1) / gridDim.x;
    // 1. the tagged input slice into slot [par][rank] of every GPU
    for (int64_t i = s0 + tid; i < s1; i += blockDim.x) {
        const uint64_t w = tag | __float_as_uint(in[i]);
        for (int r = 0; r < world; ++r)
            st_relaxed_sys_u64((uint64_t *) (peers.buf[r] + ((size_t) par * kCommMaxRanks + rank) * slot) + i, w);
    }
    // 2. every source's word of each element, summed in rank order
    const uint64_t t0 = globaltimer_ns();
    for (int64_t i = s0 + tid; i < s1; i += blockDim.x) {
        float acc = 0.f;
        bool ok = true;
        for (int r = 0; r < world && ok; ++r) {
            const uint64_t *p = (const uint64_t *) (own + ((size_t) par * kCommMaxRanks + r) * slot) + i;
            uint64_t w = ld_relaxed_sys_u64(p);
            for (uint32_t spin = 0; (w & 0xffffffff00000000ull) != tag; ++spin) {
                if ((spin & 255u) == 255u && (*abort_flag || globaltimer_ns() - t0 > kCommWaitNs)) {
                    ok = false;
                    break;
                }
                w = ld_relaxed_sys_u64(p);
            }
            const float v = __uint_as_float((uint32_t) w);
            acc = r == 0 ? v : __fadd_rn(acc, v);
        }
        if (!ok) {
            if (!*abort_flag) report(st, QWB_DEVERR_TIMEOUT, b);
            *abort_flag = 1;
            break;
        }
        out[i] = acc;
    }
}

}  // namespace
}  // namespace qwb

using namespace qwb;

struct qwb_ep_comm {
    int world, rank, device;
    size_t max_bytes;
    CommLayout lay;
    char *own;
    CommPeers peers;
    bool opened[kCommMaxRanks];
};

extern "C" QWB_API size_t qwb_ep_comm_handle_size(void) { return sizeof(cudaIpcMemHandle_t); }

extern "C" QWB_API qwb_status qwb_ep_comm_create(int world, int rank, size_t max_bytes, qwb_ep_comm **out,
                                                 void *handle_out) {
    if (!out || !handle_out) return QWB_ERR_INVALID_ARG;
    *out = nullptr;
    if (world < 1 || rank < 0 || rank >= world || max_bytes == 0) return QWB_ERR_INVALID_ARG;
    if (world > kCommMaxRanks || max_bytes > ((size_t) 1 << 30)) return QWB_ERR_LIMIT;
    qwb_ep_comm *c = new qwb_ep_comm();
    c->world = world;
    c->rank = rank;
    c->max_bytes = max_bytes;
    c->lay = comm_layout(max_bytes);
    if (cudaGetDevice(&c->device) != cudaSuccess || cudaMalloc(&c->own, c->lay.total) != cudaSuccess) {
        delete c;
        return QWB_ERR_CUDA;
    }
    if (cudaMemset(c->own, 0, c->lay.total) != cudaSuccess ||
        cudaIpcGetMemHandle((cudaIpcMemHandle_t *) handle_out, c->own) != cudaSuccess ||
        cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(c->own);
        delete c;
        return QWB_ERR_CUDA;
    }
    for (int r = 0; r < kCommMaxRanks; ++r) {
        c->peers.buf[r] = nullptr;
        c->opened[r] = false;
    }
    c->peers.buf[rank] = c->own;
    *out = c;
    return QWB_OK;
}

extern "C" QWB_API qwb_status qwb_ep_comm_connect(qwb_ep_comm *c, const void *handles) {
    if (!c || !handles) return QWB_ERR_INVALID_ARG;
    for (int r = 0; r < c->world; ++r) {
        if (r == c->rank || c->opened[r]) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, (const char *) handles + (size_t) r * sizeof(h), sizeof(h));
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return QWB_ERR_CUDA;
        c->peers.buf[r] = (char *) p;
        c->opened[r] = true;
    }
    return QWB_OK;
}

extern "C" QWB_API qwb_status qwb_ep_allreduce_f32(qwb_ep_comm *c, const float *in, float *out, int64_t n,
                                                   qwb_status_block *st, qwb_stream_t stream) {
    if (!c || n < 0) return QWB_ERR_INVALID_ARG;
    if (n == 0) return QWB_OK;
    if (!in || !out) return QWB_ERR_INVALID_ARG;
    for (int r = 0; r < c->world; ++r)
        if (!c->peers.buf[r]) return QWB_ERR_INVALID_ARG;  // not connected
    if ((size_t) n * 4 > c->max_bytes) return QWB_ERR_LIMIT;
    if (n % 4 || ((uintptr_t) in | (uintptr_t) out) % 16) return QWB_ERR_ALIGNMENT;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(kCommCtas);
    cfg.blockDim = dim3(kCommThreads);
    cfg.stream = (cudaStream_t) stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, ep_allreduce_kernel, c->peers, c->world, c->rank, c->lay.slot,
                                             c->lay.off_epoch, in, out, n, st);
    return e == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
}

extern "C" QWB_API void qwb_ep_comm_destroy(qwb_ep_comm *c) {
    if (!c) return;
    for (int r = 0; r < kCommMaxRanks; ++r)
        if (c->opened[r]) cudaIpcCloseMemHandle(c->peers.buf[r]);
    cudaFree(c->own);
    delete c;
}
