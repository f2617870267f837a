// ggml-qwb.cpp - a ggml backend (interface version 3) for B200 that runs QuestWend's MoE
// hot path through libqwb.so: GGML_OP_MUL_MAT_ID on Q4_K / Q6_K / Q8_0 expert tensors
// (slot-pool tensors with slot ids included), GGML_OP_MUL_MAT on 2-D Q4_K / Q6_K / Q8_0
// weights (shared expert, dense FFN, output head) and GGML_OP_GET_ROWS on Q4_K / Q6_K /
// Q8_0 / F16 / F32 / I32 rows.  Every other compute op is reported unsupported, so ggml's
// scheduler places it on another backend (ggml-cuda or the CPU).
//
// The vtables are the ones of ggml-backend-impl.h (buffer type / buffer :17-85, backend
// :122-164, device :177-225, registry :231-247).  Loading is ggml's dynamic-backend path
// (ggml_backend_load -> ggml_backend_init / ggml_backend_score, ggml-backend-reg.cpp),
// which QuestWend reaches through ggml_backend_load_all() (core/backend_loader.h:21-24).
//
// Behaviour kept from the C ABI (include/qwb.h): graph_compute only queues work on the
// backend's stream (no host synchronisation, no host read-back of ids).  The MUL_MAT_ID
// workspace is reserved by init_backend (params "workspace_mb=N", default 256) and grown
// only outside stream capture.  Expert or row ids out of range never fault the device:
// the affected outputs are zeroed and synchronize reports them from the status block
// (the reference CPU backend aborts on such ids instead).
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "ggml-backend-impl.h"
#include "ggml.h"
#include "qwb.h"
#include "qwb_ggml_backend.h"

#define QWB_SHIM_API extern "C" __attribute__((visibility("default")))

namespace {

constexpr size_t kAlign = 256;
constexpr size_t kDefaultWorkspaceMb = 256;

struct DevCtx {
    int device = 0;
    std::string name, description, pci_id;
    ggml_backend_buffer_type buft{};
    ggml_backend_device dev{};
};

struct BufCtx {
    void *ptr = nullptr;
    int device = 0;
};

struct BackendCtx {
    DevCtx *dev = nullptr;
    cudaStream_t stream = nullptr;
    void *ws = nullptr;
    size_t ws_bytes = 0;
    qwb_status_block *status = nullptr;
};

std::vector<DevCtx *> &devices() {
    static std::vector<DevCtx *> d;
    return d;
}

bool cuda_ok(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return true;
    std::fprintf(stderr, "ggml-qwb: %s: %s\n", what, cudaGetErrorString(e));
    return false;
}

qwb_tensor view_of(const ggml_tensor *t) {
    qwb_tensor q{};
    q.data = t->data;
    q.type = (int32_t) t->type;
    for (int i = 0; i < 4; ++i) {
        q.ne[i] = t->ne[i];
        q.nb[i] = t->nb[i];
    }
    return q;
}

// ------------------------------------------------------------------ buffer

void buf_free(ggml_backend_buffer_t b) {
    auto *c = (BufCtx *) b->context;
    cudaSetDevice(c->device);
    cuda_ok(cudaFree(c->ptr), "cudaFree");
    delete c;
}

void *buf_base(ggml_backend_buffer_t b) { return ((BufCtx *) b->context)->ptr; }

// Host copies are ordered after all work queued on the device: the backend's stream is a
// blocking stream, so the legacy default stream used here waits for it.
void buf_memset(ggml_backend_buffer_t b, ggml_tensor *t, uint8_t v, size_t off, size_t n) {
    cudaSetDevice(((BufCtx *) b->context)->device);
    cuda_ok(cudaMemset((char *) t->data + off, v, n), "cudaMemset");
}

void buf_set(ggml_backend_buffer_t b, ggml_tensor *t, const void *src, size_t off, size_t n) {
    cudaSetDevice(((BufCtx *) b->context)->device);
    cuda_ok(cudaMemcpy((char *) t->data + off, src, n, cudaMemcpyHostToDevice), "set_tensor");
}

void buf_get(ggml_backend_buffer_t b, const ggml_tensor *t, void *dst, size_t off, size_t n) {
    cudaSetDevice(((BufCtx *) b->context)->device);
    cuda_ok(cudaMemcpy(dst, (const char *) t->data + off, n, cudaMemcpyDeviceToHost), "get_tensor");
}

const char *buft_name(ggml_backend_buffer_type_t bt);

bool is_qwb_buffer(ggml_backend_buffer_t b) { return b && b->buft && b->buft->iface.get_name == buft_name; }

bool buf_cpy(ggml_backend_buffer_t b, const ggml_tensor *src, ggml_tensor *dst) {
    ggml_backend_buffer_t sb = src->view_src ? src->view_src->buffer : src->buffer;
    if (!is_qwb_buffer(sb)) return false;
    cudaSetDevice(((BufCtx *) b->context)->device);
    return cuda_ok(cudaMemcpy(dst->data, src->data, ggml_nbytes(src), cudaMemcpyDefault), "cpy_tensor");
}

void buf_clear(ggml_backend_buffer_t b, uint8_t v) {
    cudaSetDevice(((BufCtx *) b->context)->device);
    cuda_ok(cudaMemset(((BufCtx *) b->context)->ptr, v, b->size), "clear");
}

ggml_backend_buffer_i buffer_iface() {
    ggml_backend_buffer_i i{};
    i.free_buffer = buf_free;
    i.get_base = buf_base;
    i.init_tensor = nullptr;
    i.memset_tensor = buf_memset;
    i.set_tensor = buf_set;
    i.get_tensor = buf_get;
    i.set_tensor_2d = nullptr;
    i.get_tensor_2d = nullptr;
    i.cpy_tensor = buf_cpy;
    i.clear = buf_clear;
    i.reset = nullptr;
    return i;
}

// ------------------------------------------------------------- buffer type

const char *buft_name(ggml_backend_buffer_type_t bt) { return ((DevCtx *) bt->context)->name.c_str(); }

ggml_backend_buffer_t buft_alloc(ggml_backend_buffer_type_t bt, size_t size) {
    auto *d = (DevCtx *) bt->context;
    cudaSetDevice(d->device);
    void *p = nullptr;
    // ggml asks for 0-byte buffers for graphs without tensors; hand out one aligned unit
    if (!cuda_ok(cudaMalloc(&p, size ? size : kAlign), "cudaMalloc")) return nullptr;
    auto *c = new BufCtx{p, d->device};
    return ggml_backend_buffer_init(bt, buffer_iface(), c, size);
}

size_t buft_alignment(ggml_backend_buffer_type_t) { return kAlign; }
bool buft_is_host(ggml_backend_buffer_type_t) { return false; }

// ---------------------------------------------------------------- support

bool weight_type(ggml_type t) { return t == GGML_TYPE_Q4_K || t == GGML_TYPE_Q6_K || t == GGML_TYPE_Q8_0; }

bool supported(const ggml_tensor *op) {
    switch (op->op) {
        case GGML_OP_NONE:
        case GGML_OP_RESHAPE:
        case GGML_OP_VIEW:
        case GGML_OP_PERMUTE:
        case GGML_OP_TRANSPOSE:
            return true;
        case GGML_OP_MUL_MAT_ID: {
            const ggml_tensor *a = op->src[0], *b = op->src[1], *ids = op->src[2];
            if (!weight_type(a->type) || b->type != GGML_TYPE_F32 || ids->type != GGML_TYPE_I32 ||
                op->type != GGML_TYPE_F32)
                return false;
            // b rows and dst rows contiguous, weight rows packed blocks
            if (b->nb[0] != sizeof(float) || op->nb[0] != sizeof(float)) return false;
            if (a->nb[0] != ggml_type_size(a->type)) return false;
            qwb_tensor qa = view_of(a), qb = view_of(b), qi = view_of(ids);
            return qwb_mul_mat_id_workspace_size(&qa, &qb, &qi) > 0;
        }
        case GGML_OP_MUL_MAT: {
            const ggml_tensor *a = op->src[0], *b = op->src[1];
            if (!weight_type(a->type) || b->type != GGML_TYPE_F32 || op->type != GGML_TYPE_F32) return false;
            if (b->nb[0] != sizeof(float) || op->nb[0] != sizeof(float) || a->nb[0] != ggml_type_size(a->type))
                return false;
            qwb_tensor qa = view_of(a), qb = view_of(b);
            return qwb_mul_mat_workspace_size(&qa, &qb) > 0;
        }
        case GGML_OP_GET_ROWS: {
            const ggml_tensor *s = op->src[0], *i = op->src[1];
            const bool rows = weight_type(s->type) || s->type == GGML_TYPE_F16 || s->type == GGML_TYPE_F32 ||
                              s->type == GGML_TYPE_I32;
            const ggml_type out = s->type == GGML_TYPE_I32 ? GGML_TYPE_I32 : GGML_TYPE_F32;
            return rows && i->type == GGML_TYPE_I32 && op->type == out && op->nb[0] == ggml_type_size(out) &&
                   s->nb[0] == ggml_type_size(s->type) && i->ne[3] == 1;
        }
        default:
            return false;
    }
}

// ----------------------------------------------------------------- backend

ggml_guid *backend_guid() {
    static ggml_guid g = {0x51, 0x57, 0x42, 0x32, 0x30, 0x30, 0x6d, 0x6f,
                          0x65, 0x2d, 0x73, 0x6d, 0x31, 0x30, 0x30, 0x61};
    return &g;
}

const char *be_name(ggml_backend_t be) { return ((BackendCtx *) be->context)->dev->name.c_str(); }

void be_free(ggml_backend_t be) {
    auto *c = (BackendCtx *) be->context;
    cudaSetDevice(c->dev->device);
    if (c->stream) cudaStreamSynchronize(c->stream);
    if (c->ws) cudaFree(c->ws);
    if (c->status) cudaFree(c->status);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
    delete be;
}

void be_set_async(ggml_backend_t be, ggml_tensor *t, const void *src, size_t off, size_t n) {
    auto *c = (BackendCtx *) be->context;
    cuda_ok(cudaMemcpyAsync((char *) t->data + off, src, n, cudaMemcpyHostToDevice, c->stream), "set_tensor_async");
}

void be_get_async(ggml_backend_t be, const ggml_tensor *t, void *dst, size_t off, size_t n) {
    auto *c = (BackendCtx *) be->context;
    cuda_ok(cudaMemcpyAsync(dst, (const char *) t->data + off, n, cudaMemcpyDeviceToHost, c->stream),
            "get_tensor_async");
}

// Waits for the stream, then reports (and clears) device-side id errors recorded by the
// kernels since the last synchronize.
void be_sync(ggml_backend_t be) {
    auto *c = (BackendCtx *) be->context;
    cudaSetDevice(c->dev->device);
    qwb_status_block h{};
    if (qwb_status_block_read(c->status, &h, 1, (qwb_stream_t) c->stream) != QWB_OK) {
        std::fprintf(stderr, "ggml-qwb: synchronize failed: %s\n", cudaGetErrorString(cudaGetLastError()));
        return;
    }
    if (h.flags)
        std::fprintf(stderr, "ggml-qwb: %u out-of-range %s (first: %d); affected outputs were zeroed\n", h.count,
                     (h.flags & QWB_DEVERR_ID_RANGE) ? "expert ids" : "row ids", h.bad_value);
}

bool reserve_workspace(BackendCtx *c, size_t need) {
    if (need <= c->ws_bytes) return true;
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(c->stream, &cs);
    if (cs != cudaStreamCaptureStatusNone) {
        std::fprintf(stderr,
                     "ggml-qwb: MUL_MAT_ID needs %zu workspace bytes but %zu are reserved and the stream is being "
                     "captured; raise workspace_mb\n",
                     need, c->ws_bytes);
        return false;
    }
    if (!cuda_ok(cudaStreamSynchronize(c->stream), "cudaStreamSynchronize")) return false;
    if (c->ws) cudaFree(c->ws);
    c->ws = nullptr;
    c->ws_bytes = 0;
    if (!cuda_ok(cudaMalloc(&c->ws, need), "cudaMalloc(workspace)")) return false;
    c->ws_bytes = need;
    return true;
}

ggml_status be_compute(ggml_backend_t be, ggml_cgraph *g) {
    auto *c = (BackendCtx *) be->context;
    cudaSetDevice(c->dev->device);
    for (int n = 0; n < ggml_graph_n_nodes(g); ++n) {
        ggml_tensor *t = ggml_graph_node(g, n);
        if (ggml_is_empty(t)) continue;
        qwb_status rc = QWB_OK;
        switch (t->op) {
            case GGML_OP_NONE:
            case GGML_OP_RESHAPE:
            case GGML_OP_VIEW:
            case GGML_OP_PERMUTE:
            case GGML_OP_TRANSPOSE:
                continue;
            case GGML_OP_MUL_MAT_ID: {
                qwb_tensor a = view_of(t->src[0]), b = view_of(t->src[1]), ids = view_of(t->src[2]), d = view_of(t);
                if (!reserve_workspace(c, qwb_mul_mat_id_workspace_size(&a, &b, &ids))) return GGML_STATUS_ALLOC_FAILED;
                rc = qwb_mul_mat_id(&a, &b, &ids, &d, c->ws, c->ws_bytes, c->status, (qwb_stream_t) c->stream);
                break;
            }
            case GGML_OP_MUL_MAT: {
                qwb_tensor a = view_of(t->src[0]), b = view_of(t->src[1]), d = view_of(t);
                if (!reserve_workspace(c, qwb_mul_mat_workspace_size(&a, &b))) return GGML_STATUS_ALLOC_FAILED;
                rc = qwb_mul_mat(&a, &b, &d, c->ws, c->ws_bytes, c->status, (qwb_stream_t) c->stream);
                break;
            }
            case GGML_OP_GET_ROWS: {
                qwb_tensor s = view_of(t->src[0]), i = view_of(t->src[1]), d = view_of(t);
                rc = qwb_get_rows(&s, &i, &d, c->status, (qwb_stream_t) c->stream);
                break;
            }
            default:
                std::fprintf(stderr, "ggml-qwb: op %s (%s) is not supported\n", ggml_op_name(t->op), t->name);
                return GGML_STATUS_FAILED;
        }
        if (rc != QWB_OK) {
            std::fprintf(stderr, "ggml-qwb: %s (%s): %s\n", ggml_op_name(t->op), t->name, qwb_status_string(rc));
            return GGML_STATUS_FAILED;
        }
    }
    return GGML_STATUS_SUCCESS;
}

ggml_backend_i backend_iface() {
    ggml_backend_i i{};
    i.get_name = be_name;
    i.free = be_free;
    i.set_tensor_async = be_set_async;
    i.get_tensor_async = be_get_async;
    i.synchronize = be_sync;
    i.graph_compute = be_compute;
    return i;
}

// ------------------------------------------------------------------ device

const char *dev_name(ggml_backend_dev_t d) { return ((DevCtx *) d->context)->name.c_str(); }
const char *dev_description(ggml_backend_dev_t d) { return ((DevCtx *) d->context)->description.c_str(); }

void dev_memory(ggml_backend_dev_t d, size_t *free_b, size_t *total_b) {
    cudaSetDevice(((DevCtx *) d->context)->device);
    *free_b = *total_b = 0;
    cudaMemGetInfo(free_b, total_b);
}

enum ggml_backend_dev_type dev_type(ggml_backend_dev_t) { return GGML_BACKEND_DEVICE_TYPE_GPU; }

void dev_props(ggml_backend_dev_t d, ggml_backend_dev_props *p) {
    auto *c = (DevCtx *) d->context;
    p->name = c->name.c_str();
    p->description = c->description.c_str();
    dev_memory(d, &p->memory_free, &p->memory_total);
    p->type = GGML_BACKEND_DEVICE_TYPE_GPU;
    p->device_id = c->pci_id.empty() ? nullptr : c->pci_id.c_str();
    p->caps = {};
    p->caps.async = true;
}

// params: "workspace_mb=N" (MUL_MAT_ID workspace reserved up front, default 256 MiB).
ggml_backend_t dev_init(ggml_backend_dev_t d, const char *params) {
    auto *dc = (DevCtx *) d->context;
    size_t mb = kDefaultWorkspaceMb;
    if (params) {
        const char *w = std::strstr(params, "workspace_mb=");
        if (w) mb = (size_t) std::strtoull(w + 13, nullptr, 10);
    }
    if (!cuda_ok(cudaSetDevice(dc->device), "cudaSetDevice")) return nullptr;
    auto *c = new BackendCtx();
    c->dev = dc;
    bool ok = cuda_ok(cudaStreamCreateWithFlags(&c->stream, cudaStreamDefault), "cudaStreamCreate") &&
              cuda_ok(cudaMalloc((void **) &c->status, sizeof(qwb_status_block)), "cudaMalloc(status)") &&
              cuda_ok(cudaMemset(c->status, 0, sizeof(qwb_status_block)), "cudaMemset(status)");
    if (ok && mb) {
        ok = cuda_ok(cudaMalloc(&c->ws, mb << 20), "cudaMalloc(workspace)");
        if (ok) c->ws_bytes = mb << 20;
    }
    auto *be = new ggml_backend{};
    be->guid = backend_guid();
    be->iface = backend_iface();
    be->device = d;
    be->context = c;
    if (!ok) {
        be_free(be);
        return nullptr;
    }
    return be;
}

ggml_backend_buffer_type_t dev_buft(ggml_backend_dev_t d) { return &((DevCtx *) d->context)->buft; }
bool dev_supports_op(ggml_backend_dev_t, const ggml_tensor *op) { return supported(op); }
bool dev_supports_buft(ggml_backend_dev_t d, ggml_backend_buffer_type_t bt) { return bt == dev_buft(d); }
bool dev_offload_op(ggml_backend_dev_t, const ggml_tensor *) { return false; }

// ---------------------------------------------------------------- registry

const char *reg_name(ggml_backend_reg_t) { return "QWB"; }
size_t reg_count(ggml_backend_reg_t) { return devices().size(); }
ggml_backend_dev_t reg_device(ggml_backend_reg_t, size_t i) { return i < devices().size() ? &devices()[i]->dev : nullptr; }
void *reg_proc(ggml_backend_reg_t, const char *) { return nullptr; }

}  // namespace

// The registry of B200 (sm_100) devices visible to this process; a process without one
// gets a registry with no devices.
QWB_SHIM_API ggml_backend_reg_t ggml_backend_qwb_reg(void) {
    static ggml_backend_reg reg{};
    static std::once_flag once;
    std::call_once(once, [] {
        reg.api_version = GGML_BACKEND_API_VERSION;
        reg.iface.get_name = reg_name;
        reg.iface.get_device_count = reg_count;
        reg.iface.get_device = reg_device;
        reg.iface.get_proc_address = reg_proc;
        reg.context = nullptr;
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess) {
            cudaGetLastError();
            n = 0;
        }
        for (int i = 0; i < n; ++i) {
            cudaDeviceProp prop{};
            if (cudaGetDeviceProperties(&prop, i) != cudaSuccess || prop.major != 10) continue;
            auto *dc = new DevCtx();
            dc->device = i;
            dc->name = "QWB" + std::to_string(devices().size());
            dc->description = prop.name;
            char pci[32];
            std::snprintf(pci, sizeof pci, "%04x:%02x:%02x.0", prop.pciDomainID, prop.pciBusID, prop.pciDeviceID);
            dc->pci_id = pci;
            dc->buft.iface.get_name = buft_name;
            dc->buft.iface.alloc_buffer = buft_alloc;
            dc->buft.iface.get_alignment = buft_alignment;
            dc->buft.iface.is_host = buft_is_host;
            dc->buft.device = &dc->dev;
            dc->buft.context = dc;
            ggml_backend_device_i &di = dc->dev.iface;
            di.get_name = dev_name;
            di.get_description = dev_description;
            di.get_memory = dev_memory;
            di.get_type = dev_type;
            di.get_props = dev_props;
            di.init_backend = dev_init;
            di.get_buffer_type = dev_buft;
            di.supports_op = dev_supports_op;
            di.supports_buft = dev_supports_buft;
            di.offload_op = dev_offload_op;
            dc->dev.reg = &reg;
            dc->dev.context = dc;
            devices().push_back(dc);
        }
    });
    return &reg;
}

// Entry points of ggml's dynamic backend loader (ggml_backend_load).
QWB_SHIM_API ggml_backend_reg_t ggml_backend_init(void) { return ggml_backend_qwb_reg(); }
QWB_SHIM_API int ggml_backend_score(void) { return ggml_backend_qwb_reg()->iface.get_device_count(nullptr) ? 100 : 0; }
