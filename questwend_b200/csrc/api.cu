// api.cu - library-level entry points: version, status strings, device status block.
#include "common.cuh"

extern "C" QWB_API int qwb_abi_version(void) { return QWB_ABI_VERSION; }

extern "C" QWB_API const char *qwb_status_string(qwb_status s) {
    switch (s) {
        case QWB_OK: return "ok";
        case QWB_ERR_INVALID_ARG: return "invalid argument";
        case QWB_ERR_UNSUPPORTED_TYPE: return "unsupported tensor type";
        case QWB_ERR_SHAPE: return "shape mismatch";
        case QWB_ERR_LAYOUT: return "unsupported tensor layout";
        case QWB_ERR_ALIGNMENT: return "misaligned pointer or stride";
        case QWB_ERR_WORKSPACE: return "workspace missing or too small";
        case QWB_ERR_CUDA: return "CUDA runtime error";
        case QWB_ERR_DEVICE: return "unsupported device (sm_100 required)";
        case QWB_ERR_LIMIT: return "size beyond supported limit";
    }
    return "unknown status";
}

extern "C" QWB_API qwb_status qwb_status_block_read(qwb_status_block *d_block, qwb_status_block *out, int reset,
                                                   qwb_stream_t stream) {
    if (!d_block || !out) return QWB_ERR_INVALID_ARG;
    cudaStream_t s = (cudaStream_t) stream;
    if (cudaMemcpyAsync(out, d_block, sizeof(*out), cudaMemcpyDeviceToHost, s) != cudaSuccess) return QWB_ERR_CUDA;
    if (cudaStreamSynchronize(s) != cudaSuccess) return QWB_ERR_CUDA;
    if (reset && cudaMemsetAsync(d_block, 0, sizeof(*d_block), s) != cudaSuccess) return QWB_ERR_CUDA;
    return QWB_OK;
}

// ------------------------------------------------------------------ profiling
#include <vector>

namespace qwb {
namespace {
std::vector<cudaEvent_t> g_events;
std::vector<int32_t> g_tags;
int g_next = 0;
}  // namespace

void profile_mark(cudaStream_t s, int tag) {
    if (g_events.empty() || g_next >= (int) g_events.size()) return;
    // under stream capture the record must become an external event-record node, or it
    // is only a capture-time dependency and never records on replay
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(s, &cs);
    const unsigned flags = cs == cudaStreamCaptureStatusActive ? cudaEventRecordExternal : cudaEventRecordDefault;
    if (cudaEventRecordWithFlags(g_events[g_next], s, flags) == cudaSuccess) g_tags[g_next++] = tag;
}
}  // namespace qwb

extern "C" QWB_API qwb_status qwb_profile_enable(int max_marks) {
    using namespace qwb;
    for (cudaEvent_t e : g_events) cudaEventDestroy(e);
    g_events.clear();
    g_tags.clear();
    g_next = 0;
    if (max_marks < 0) return QWB_ERR_INVALID_ARG;
    for (int i = 0; i < max_marks; ++i) {
        cudaEvent_t e;
        if (cudaEventCreate(&e) != cudaSuccess) return QWB_ERR_CUDA;
        g_events.push_back(e);
    }
    g_tags.assign((size_t) max_marks, 0);
    return QWB_OK;
}

extern "C" QWB_API qwb_status qwb_profile_reset(void) {
    qwb::g_next = 0;
    return QWB_OK;
}

extern "C" QWB_API int qwb_profile_count(void) { return qwb::g_next; }

extern "C" QWB_API qwb_status qwb_profile_read(float *ms, int32_t *tags, int n) {
    using namespace qwb;
    if (n < 0 || n > g_next - 1 || (n && (!ms || !tags))) return QWB_ERR_INVALID_ARG;
    if (n == 0) return QWB_OK;
    if (cudaEventSynchronize(g_events[n]) != cudaSuccess) return QWB_ERR_CUDA;
    for (int i = 0; i < n; ++i) {
        if (cudaEventElapsedTime(&ms[i], g_events[i], g_events[i + 1]) != cudaSuccess) return QWB_ERR_CUDA;
        tags[i] = g_tags[i + 1];
    }
    return QWB_OK;
}
