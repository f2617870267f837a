// pool.cu - expert pool writes (host slabs -> pool slots) and the device-side byte audit
// of pool slots.
//
// Pool write: ExpertCache::fetch_slab (core/expert_cache.cpp:637-723) and fetch_parallel's
// group upload (:1357-1377) copy one expert's slab of nb2 bytes into slot s of a pool
// tensor with ggml_backend_tensor_set(_async)(pool, src, s * nb2, nb2), after checking
// that the source's nb2 equals the pool's (:643-645).  Here the whole group is one call:
// arguments are checked first (nothing is written on an error), then one asynchronous
// copy per slab.  Slabs are not merged into larger copies even when their addresses
// line up: adjacent addresses may belong to two separate page-locked allocations, and
// one copy may not span both.  Copy-engine copies queued back to back leave a set-up gap
// each (0.67-0.84 of one large copy's rate for 24 slabs of ~1 MB), so when every source
// is readable by the device (page-locked host memory or this device's memory) and
// 16-byte aligned, one gather kernel moves the whole group: each CTA copies a 64 KB chunk
// of one slab with 16-byte loads straight from the source (over the host link for host
// memory) and stores into the slot.  A slot named twice keeps only its last source (the
// one a sequence of copies would leave).  Otherwise (pageable or unaligned sources) one
// cudaMemcpyAsync per slab, the odd slots on a second stream of the library's, forked
// from and joined back into the caller's stream with events.
//
// Byte audit: ExpertWeightAudit::destination / compare (core/expert_weight_audit.h:62-66,
// :106-125) read each slot back to the host and compare it with the authoritative bytes,
// logging the equal flag, the first differing byte and both FNV-1a 64 checksums (:83-87).
// pool_audit_kernel computes that record on the GPU, one CTA per slab: the CTA stages
// 8 KB chunks of the expected and actual bytes in shared memory, every thread compares
// its 32-byte segment (until the first difference is known), and, when checksums are
// asked for, two threads run the two checksum chains, which are serial by definition
// (h = (h ^ byte) * prime per byte): ~18 cycles per byte on one thread, milliseconds per
// megabyte, so the compare alone (no checksums) stops at the first difference and runs at
// the bandwidth of the slower source.
#include <cuda_runtime.h>

#include <algorithm>
#include <mutex>
#include <unordered_set>
#include <vector>

#include "common.cuh"

namespace qwb {

namespace {

constexpr int kAuditThreads = 256;
constexpr int kAuditChunk = 8192;  // bytes staged per buffer per pass
constexpr int kAuditBatch = 128;   // slabs per launch (pointer table in the kernel parameters)

// FNV-1a 64 (Fowler / Noll / Vo): offset basis and prime of the published algorithm,
// the constants core/expert_weight_audit.h:84-85 uses
constexpr unsigned long long kFnvBasis = 14695981039346656037ull;
constexpr unsigned long long kFnvPrime = 1099511628211ull;

struct AuditBatch {
    const uint8_t *expected[kAuditBatch];
    const uint8_t *actual[kAuditBatch];
};

// One FNV-1a step on h = (hi, lo): h ^= byte; h *= 2^40 + 0x1b3 (the prime), written in
// 32-bit halves so the dependent chain is one xor and one multiply-add per byte:
//   lo' = (lo ^ byte) * 0x1b3                (mod 2^32)
//   hi' = hi * 0x1b3 + umulhi(lo ^ byte, 0x1b3) + ((lo ^ byte) << 8)   (mod 2^32)
struct Fnv {
    uint32_t lo, hi;
};
static_assert(kFnvPrime == (1ull << 40) + 0x1b3ull, "FNV-1a 64 prime");

__device__ __forceinline__ void fnv_byte(Fnv &h, uint32_t byte) {
    const uint32_t x = h.lo ^ byte;
    h.hi = h.hi * 0x1b3u + __umulhi(x, 0x1b3u) + (x << 8);
    h.lo = x * 0x1b3u;
}

__device__ __forceinline__ void fnv_word(Fnv &h, uint32_t w) {
#pragma unroll
    for (int k = 0; k < 4; ++k) fnv_byte(h, (w >> (8 * k)) & 0xffu);
}

// FNV-1a over n staged bytes (16-byte aligned shared buffer)
__device__ void fnv_bytes(Fnv &h, const uint8_t *s, int n) {
    int i = 0;
    for (; i + 16 <= n; i += 16) {
        const uint4 w = *(const uint4 *) (s + i);
        fnv_word(h, w.x);
        fnv_word(h, w.y);
        fnv_word(h, w.z);
        fnv_word(h, w.w);
    }
    for (; i < n; ++i) fnv_byte(h, s[i]);
}

__global__ void __launch_bounds__(kAuditThreads) pool_audit_kernel(const __grid_constant__ AuditBatch b,
                                                                   unsigned long long bytes, bool vec, bool sums,
                                                                   qwb_slab_audit *__restrict__ res) {
    __shared__ __align__(16) uint8_t se[kAuditChunk];
    __shared__ __align__(16) uint8_t sa[kAuditChunk];
    __shared__ unsigned long long first;
    const int tid = threadIdx.x;
    const uint8_t *exp = b.expected[blockIdx.x], *act = b.actual[blockIdx.x];
    if (tid == 0) first = bytes;
    Fnv h{(uint32_t) kFnvBasis, (uint32_t) (kFnvBasis >> 32)};  // thread 0: expected, thread 32: actual
    __syncthreads();
    for (unsigned long long off = 0; off < bytes; off += kAuditChunk) {
        const int n = (int) (bytes - off < (unsigned long long) kAuditChunk ? bytes - off : kAuditChunk);
        // read before this chunk's compare phase lowers it: every thread takes the same branch
        const bool searching = first == bytes;
        if (!searching && !sums) break;  // the record is complete
        if (vec) {  // both slabs 16-byte aligned and bytes % 16 == 0
            for (int i = tid; i < n / 16; i += kAuditThreads) {
                ((uint4 *) se)[i] = ((const uint4 *) (exp + off))[i];
                ((uint4 *) sa)[i] = ((const uint4 *) (act + off))[i];
            }
        } else {
            for (int i = tid; i < n; i += kAuditThreads) {
                se[i] = exp[off + i];
                sa[i] = act[off + i];
            }
        }
        __syncthreads();
        if (searching) {  // no difference found in earlier chunks: compare this one
            const int lo = 32 * tid, hi = min(lo + 32, n);
            for (int i = lo; i < hi; ++i) {
                if (se[i] != sa[i]) {
                    atomicMin(&first, off + (unsigned long long) i);
                    break;
                }
            }
        }
        if (sums && tid == 0) fnv_bytes(h, se, n);
        if (sums && tid == 32) fnv_bytes(h, sa, n);
        __syncthreads();  // the buffers are free, `first` is final for this chunk
    }
    qwb_slab_audit &r = res[blockIdx.x];
    if (tid == 0) {
        const unsigned long long f = first;
        r.equal = f == bytes;
        r.reserved = 0;
        r.first_difference = f;
        r.expected_byte = f < bytes ? exp[f] : 0u;
        r.actual_byte = f < bytes ? act[f] : 0u;
        r.expected_fnv1a64 = sums ? ((unsigned long long) h.hi << 32) | h.lo : 0ull;
    }
    if (tid == 32) r.actual_fnv1a64 = sums ? ((unsigned long long) h.hi << 32) | h.lo : 0ull;
}

// Second copy stream and its fork / join events, one set per device, created on first use.
struct SideStream {
    cudaStream_t s = nullptr;
    cudaEvent_t fork = nullptr, join = nullptr;
};
constexpr int kMaxDevices = 64;
SideStream g_side[kMaxDevices];
std::mutex g_side_mu;  // also serialises the fork / copies / join sequence of concurrent callers

bool side_ready(SideStream &ss) {
    if (ss.s) return true;
    if (cudaStreamCreateWithFlags(&ss.s, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&ss.join, cudaEventDisableTiming) != cudaSuccess) {
        (void) cudaGetLastError();
        return false;
    }
    return true;
}

constexpr int kGatherThreads = 256;
constexpr int kGatherChunk = 65536;  // bytes of one slab per CTA
constexpr int kGatherBatch = 128;    // slabs per launch (pointer table in the kernel parameters)

struct GatherBatch {
    const uint4 *src[kGatherBatch];
    uint4 *dst[kGatherBatch];
};

// CTA (slab i, chunk c) copies bytes [c * 64 KB, (c + 1) * 64 KB) of slab i; every thread
// keeps four 16-byte loads in flight before it stores them.
__global__ void __launch_bounds__(kGatherThreads) pool_gather_kernel(const __grid_constant__ GatherBatch b,
                                                                     int chunks, long long words) {
    const int i = blockIdx.x / chunks, c = blockIdx.x - i * chunks;
    const uint4 *src = b.src[i];
    uint4 *dst = b.dst[i];
    constexpr int kw = kGatherChunk / 16;
    const long long w0 = (long long) c * kw, w1 = min(w0 + kw, words);
    long long w = w0 + threadIdx.x;
    for (; w + 3 * kGatherThreads < w1; w += 4 * kGatherThreads) {
        uint4 v[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) v[k] = src[w + k * kGatherThreads];
#pragma unroll
        for (int k = 0; k < 4; ++k) dst[w + k * kGatherThreads] = v[k];
    }
    for (; w < w1; w += kGatherThreads) dst[w] = src[w];
}

bool pool_ok(const qwb_tensor *pool) { return pool && pool->data && pool->ne[2] >= 1 && pool->nb[2] > 0; }

// A pointer the current device can dereference: device memory of this device, managed
// memory, or page-locked host memory (its device alias).  Pageable host memory and other
// devices' memory give nullptr.
const void *device_view(const void *p, int dev) {
    cudaPointerAttributes at{};
    if (cudaPointerGetAttributes(&at, p) != cudaSuccess) {
        (void) cudaGetLastError();
        return nullptr;
    }
    switch (at.type) {
        case cudaMemoryTypeDevice: return at.device == dev ? p : nullptr;
        case cudaMemoryTypeManaged: return p;
        case cudaMemoryTypeHost: return at.devicePointer;
        default: return nullptr;
    }
}

}  // namespace

}  // namespace qwb

extern "C" QWB_API qwb_status qwb_pool_write_slabs(const qwb_tensor *pool, size_t src_slab_bytes,
                                                   const qwb_slab_copy *copies, int n, qwb_stream_t stream) {
    if (!qwb::pool_ok(pool) || n < 0 || (n > 0 && !copies)) return QWB_ERR_INVALID_ARG;
    const size_t nb2 = pool->nb[2];
    if (src_slab_bytes != nb2) return QWB_ERR_SHAPE;  // "slab size mismatch (pool vs source)"
    for (int i = 0; i < n; ++i)
        if (!copies[i].src || copies[i].slot < 0 || copies[i].slot >= pool->ne[2]) return QWB_ERR_INVALID_ARG;
    if (n == 0) return QWB_OK;
    cudaStream_t s = (cudaStream_t) stream;
    char *base = (char *) pool->data;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= qwb::kMaxDevices) return QWB_ERR_CUDA;
    // A source inside the pool (a slot copied to another slot) may be overwritten by an
    // earlier entry: then every copy runs in array order on the caller's stream.
    const uintptr_t lo = (uintptr_t) base, hi = lo + (uintptr_t) pool->ne[2] * nb2;
    bool in_order = false;
    for (int i = 0; i < n && !in_order; ++i) {
        const uintptr_t a0 = (uintptr_t) copies[i].src;
        in_order = a0 < hi && a0 + nb2 > lo;
    }
    if (!in_order) {
        // gather kernel: every source device-readable and 16-byte aligned, the slots too
        std::vector<const void *> view(n, nullptr);
        bool gather = nb2 % 16 == 0 && (uintptr_t) base % 16 == 0 && qwb::device_view(base, dev) == base;
        for (int i = 0; i < n && gather; ++i) {
            view[i] = qwb::device_view(copies[i].src, dev);
            gather = view[i] && (uintptr_t) view[i] % 16 == 0;
        }
        if (gather) {
            // the last entry of each slot wins; the others would be overwritten
            std::vector<int> keep;
            keep.reserve(n);
            std::unordered_set<int64_t> seen;
            for (int i = n - 1; i >= 0; --i)
                if (seen.insert(copies[i].slot).second) keep.push_back(i);
            const int chunks = (int) ((nb2 + qwb::kGatherChunk - 1) / qwb::kGatherChunk);
            for (size_t k0 = 0; k0 < keep.size(); k0 += qwb::kGatherBatch) {
                const int cnt = (int) std::min(keep.size() - k0, (size_t) qwb::kGatherBatch);
                qwb::GatherBatch b{};
                for (int k = 0; k < cnt; ++k) {
                    const int i = keep[k0 + k];
                    b.src[k] = (const uint4 *) view[i];
                    b.dst[k] = (uint4 *) (base + (size_t) copies[i].slot * nb2);
                }
                qwb::pool_gather_kernel<<<cnt * chunks, qwb::kGatherThreads, 0, s>>>(b, chunks,
                                                                                   (long long) (nb2 / 16));
                if (cudaGetLastError() != cudaSuccess) return QWB_ERR_CUDA;
            }
            return QWB_OK;
        }
        (void) cudaGetLastError();
    }
    auto issue = [&](int i, cudaStream_t st) {
        return cudaMemcpyAsync(base + (size_t) copies[i].slot * nb2, copies[i].src, nb2, cudaMemcpyDefault, st) ==
               cudaSuccess;
    };
    std::lock_guard<std::mutex> lk(qwb::g_side_mu);
    qwb::SideStream &ss = qwb::g_side[dev];
    bool ok;
    if (n == 1 || in_order || !qwb::side_ready(ss)) {
        ok = true;
        for (int i = 0; i < n && ok; ++i) ok = issue(i, s);
    } else {
        ok = cudaEventRecord(ss.fork, s) == cudaSuccess && cudaStreamWaitEvent(ss.s, ss.fork, 0) == cudaSuccess;
        for (int i = 0; i < n && ok; ++i) ok = issue(i, (copies[i].slot & 1) ? ss.s : s);
        // join even after a failed copy, so the caller's stream never runs ahead of copies
        // already issued on the side stream
        const bool joined = cudaEventRecord(ss.join, ss.s) == cudaSuccess &&
                            cudaStreamWaitEvent(s, ss.join, 0) == cudaSuccess;
        ok = ok && joined;
    }
    if (!ok) {
        (void) cudaGetLastError();  // the error belongs to this call, not to later launches
        return QWB_ERR_CUDA;
    }
    return QWB_OK;
}

extern "C" QWB_API qwb_status qwb_pool_audit_slabs(const qwb_tensor *pool, const qwb_slab_copy *expected, int n,
                                                   int checksums, qwb_slab_audit *results, qwb_stream_t stream) {
    if (!qwb::pool_ok(pool) || n < 0 || (n > 0 && (!expected || !results))) return QWB_ERR_INVALID_ARG;
    for (int i = 0; i < n; ++i)
        if (!expected[i].src || expected[i].slot < 0 || expected[i].slot >= pool->ne[2]) return QWB_ERR_INVALID_ARG;
    if (n == 0) return QWB_OK;
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return QWB_ERR_CUDA;
    const char *base = (const char *) qwb::device_view(pool->data, dev);
    qwb_slab_audit *res = (qwb_slab_audit *) qwb::device_view(results, dev);
    if (!base || !res) return QWB_ERR_INVALID_ARG;
    const size_t nb2 = pool->nb[2];
    cudaStream_t s = (cudaStream_t) stream;
    for (int i0 = 0; i0 < n; i0 += qwb::kAuditBatch) {
        const int cnt = std::min(n - i0, qwb::kAuditBatch);
        qwb::AuditBatch b{};
        bool vec = nb2 % 16 == 0;
        for (int k = 0; k < cnt; ++k) {
            const uint8_t *e = (const uint8_t *) qwb::device_view(expected[i0 + k].src, dev);
            if (!e) return QWB_ERR_INVALID_ARG;  // pageable host memory or another device's
            b.expected[k] = e;
            b.actual[k] = (const uint8_t *) base + (size_t) expected[i0 + k].slot * nb2;
            vec = vec && ((uintptr_t) b.expected[k] % 16 == 0) && ((uintptr_t) b.actual[k] % 16 == 0);
        }
        qwb::pool_audit_kernel<<<cnt, qwb::kAuditThreads, 0, s>>>(b, (unsigned long long) nb2, vec, checksums != 0,
                                                                   res + i0);
        if (cudaGetLastError() != cudaSuccess) return QWB_ERR_CUDA;
    }
    return QWB_OK;
}
