// route.cu - router top-k, SwiGLU and the weighted expert reduction.
//
// route_experts (core/runtime.cpp:2693-2734) on the CPU backend is
//   probs   = soft_max(logits [+ mask])              ggml-cpu/ops.cpp:5813 (exp(x-max),
//                                                    sum in double, scale by 1/sum)
//   sel     = argsort_top_k(probs, k)                ggml.c:5462 (descending argsort view)
//   w       = get_rows(probs, sel); w /= clamp(sum_rows(w), 6.103515625e-5, inf) [* scale]
// One CTA routes one token: softmax in shared memory, then a rank-based top-k (each
// expert counts the experts that beat it: larger probability, or equal probability and a
// lower index) so the k winners land directly at their rank.  The CPU's std::sort leaves
// the order of exactly equal probabilities unspecified; with distinct values the
// selection and its order are identical.
#include "common.cuh"
#include "kernels.cuh"
#include "quant_dev.cuh"
#include "route.cuh"

namespace qwb {

__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    float r = red[0];
    for (int i = 1; i < nw; ++i) r = fmaxf(r, red[i]);
    return r;
}
__device__ __forceinline__ double block_sum_d(double v, double *red) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    __syncthreads();
    if ((threadIdx.x & 31) == 0) red[w] = v;
    __syncthreads();
    double r = 0.0;
    for (int i = 0; i < nw; ++i) r += red[i];
    return r;
}

// Route one token with the whole CTA.  lg: E logits (global), mk: E mask values or null.
// sp: shared scratch of E floats.  Writes sel[0..k) and w[0..k).
__device__ void route_token(const float *lg, const float *mk, int E, int k, int norm, float scale, int32_t *sel,
                            float *w, float *sp, int *ssel, float *redf, double *redd) {
    // a NaN logit ranks last (as -inf) so the top-k is a total order and every one of
    // the k slots is written
    for (int j = threadIdx.x; j < k; j += blockDim.x) ssel[j] = j;
    float lmax = -INFINITY;
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        float v = __ldcg(lg + i);
        if (mk) v = __fadd_rn(v, __ldcg(mk + i));
        if (isnan(v)) v = -INFINITY;
        sp[i] = v;
        lmax = fmaxf(lmax, v);
    }
    const float mx = block_max(lmax, redf);
    double ls = 0.0;
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        float e = expf(__fsub_rn(sp[i], mx));
        if (isnan(e)) e = 0.f;  // every logit -inf: all probabilities 0
        sp[i] = e;
        ls += (double) e;
    }
    const double sum = block_sum_d(ls, redd);
    const float inv = sum > 0.0 ? (float) (1.0 / sum) : 0.f;
    for (int i = threadIdx.x; i < E; i += blockDim.x) sp[i] = __fmul_rn(sp[i], inv);
    __syncthreads();
    for (int i = threadIdx.x; i < E; i += blockDim.x) {
        const float pi = sp[i];
        int rank = 0;
        for (int j = 0; j < E; ++j) {
            const float pj = sp[j];
            rank += (pj > pi) || (pj == pi && j < i);
        }
        if (rank < k) ssel[rank] = i;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float ws = 0.f;
        for (int j = 0; j < k; ++j) ws = __fadd_rn(ws, sp[ssel[j]]);
        if (ws < 6.103515625e-5f) ws = 6.103515625e-5f;
        for (int j = 0; j < k; ++j) {
            float v = sp[ssel[j]];
            if (norm) v = __fdiv_rn(v, ws);
            if (scale != 0.0f && scale != 1.0f) v = __fmul_rn(v, scale);
            sel[j] = ssel[j];
            w[j] = v;
        }
    }
    __syncthreads();
}

// one CTA per token
__global__ void __launch_bounds__(256) route_kernel(const float *logits, const float *mask, int E, int k, int norm,
                                                    float scale, int32_t *selected, float *weights) {
    extern __shared__ float sp[];
    __shared__ int ssel[kMaxUsed];
    __shared__ float redf[8];
    __shared__ double redd[8];
    const int64_t t = blockIdx.x;
    route_token(logits + t * E, mask ? mask + t * E : nullptr, E, k, norm, scale, selected + t * k,
                weights + t * k, sp, ssel, redf, redd);
}

cudaError_t launch_route(const float *logits, const float *mask, int64_t E, int64_t T, int64_t k, int norm,
                         float scale, int32_t *selected, float *weights, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    route_kernel<<<(unsigned) T, 128, (size_t) E * 4, s>>>(logits, mask, (int) E, (int) k, norm, scale, selected,
                                                          weights);
    return cudaGetLastError();
}

// ------------------------------------------------------- fused router (small T)
// CTA e computes logits[t][e] = router_w[e] . x[t] for all t (4 warps split H), and,
// as side work, quantizes 256-chunks of x into q8 planes.  The last CTA to finish (an
// atomicInc on a workspace counter that wraps back to zero) routes every token and,
// for decode (T == 1), writes the GEMV tile list: one tile per selected expert.
// sum of squares of a warp's slice of a row, each square rounded to f32 and accumulated
// in f64 as ggml's rms_norm does (ggml-cpu/ops.cpp:4140-4144)
__device__ __forceinline__ double warp_sumsq(const float *x, int64_t n, int lane) {
    double acc = 0.0;
    for (int64_t h = 4 * lane; h < n; h += 128) {
        const float4 b = *(const float4 *) (x + h);
        acc += (double) __fmul_rn(b.x, b.x);
        acc += (double) __fmul_rn(b.y, b.y);
        acc += (double) __fmul_rn(b.z, b.z);
        acc += (double) __fmul_rn(b.w, b.w);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    return acc;
}
// scale = 1 / sqrtf(mean + eps), mean = (float)(sum / H)  (ops.cpp:4146-4147)
__device__ __forceinline__ float rms_scale(double sum, int64_t H, float eps) {
    const float mean = (float) (sum / (double) H);
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
}

__global__ void __launch_bounds__(128) router_fused_kernel(const RouterArgs r) {
    extern __shared__ float sp[];
    __shared__ float part[4][kMaxRouterT];
    __shared__ double dpart[4][kMaxRouterT];
    __shared__ float s_scale[kMaxRouterT];
    __shared__ int ssel[kMaxUsed];
    __shared__ float redf[8];
    __shared__ double redd[8];
    __shared__ int s_last;
    const int e = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t q = r.H / 4;  // H % 1024 == 0 checked on the host

    // ffn_norm: every CTA derives the per-token RMS scale itself (x rows are a few KB)
    if (r.norm_w) {
        for (int t = 0; t < r.T; ++t) {
            const double v = warp_sumsq(r.x + (int64_t) t * r.H + warp * q, q, lane);
            if (lane == 0) dpart[warp][t] = v;
        }
        __syncthreads();
        if (threadIdx.x < r.T) {
            const int t = threadIdx.x;
            s_scale[t] = rms_scale(((dpart[0][t] + dpart[1][t]) + dpart[2][t]) + dpart[3][t], r.H, r.norm_eps);
        }
        __syncthreads();
    }

    // side work: quantize (normed) x (T rows of H) into q8 planes, one 256-chunk per warp
    if (r.xq.qs) {
        const int64_t chunks = (int64_t) r.T * (r.H / 256);
        for (int64_t c = (int64_t) blockIdx.x * 4 + warp; c < chunks; c += (int64_t) gridDim.x * 4) {
            const int64_t t = c / (r.H / 256), cc = c % (r.H / 256);
            quantize_chunk_warp(r.kq ? 0 : 1, r.x + t * r.H + cc * 256, r.xq, t, cc * 256, r.H,
                                r.norm_w ? s_scale[t] : 1.f, r.norm_w ? r.norm_w + cc * 256 : nullptr);
        }
    }
    // logits
    const float *wr = r.router_w + (int64_t) e * r.H + warp * q;
    const float *gw = r.norm_w ? r.norm_w + warp * q : nullptr;
    for (int t = 0; t < r.T; ++t) {
        const float *xr = r.x + (int64_t) t * r.H + warp * q;
        float acc = 0.f;
        if (gw) {
            const float sc = s_scale[t];
            for (int64_t h = 4 * lane; h < q; h += 128) {
                const float4 a = *(const float4 *) (wr + h);
                const float4 b = *(const float4 *) (xr + h);
                const float4 g = *(const float4 *) (gw + h);
                acc = fmaf(a.x, __fmul_rn(__fmul_rn(b.x, sc), g.x), acc);
                acc = fmaf(a.y, __fmul_rn(__fmul_rn(b.y, sc), g.y), acc);
                acc = fmaf(a.z, __fmul_rn(__fmul_rn(b.z, sc), g.z), acc);
                acc = fmaf(a.w, __fmul_rn(__fmul_rn(b.w, sc), g.w), acc);
            }
        } else {
            for (int64_t h = 4 * lane; h < q; h += 128) {
                const float4 a = *(const float4 *) (wr + h);
                const float4 b = *(const float4 *) (xr + h);
                acc = fmaf(a.x, b.x, acc);
                acc = fmaf(a.y, b.y, acc);
                acc = fmaf(a.z, b.z, acc);
                acc = fmaf(a.w, b.w, acc);
            }
        }
        acc = warp_sum(acc);
        if (lane == 0) part[warp][t] = acc;
    }
    __syncthreads();
    if (threadIdx.x < r.T) {
        const int t = threadIdx.x;
        r.logits[(int64_t) t * r.E + e] = (part[0][t] + part[1][t]) + (part[2][t] + part[3][t]);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicInc(r.counter, gridDim.x - 1) == gridDim.x - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int t = 0; t < r.T; ++t) {
        int32_t *sel = r.selected + (int64_t) t * r.n_used;
        float *w = r.weights + (int64_t) t * r.n_used;
        route_token(r.logits + (int64_t) t * r.E, r.mask ? r.mask + (int64_t) t * r.E : nullptr, (int) r.E,
                    (int) r.n_used, 1, 0.0f, sel, w, sp, ssel, redf, redd);
        if (r.tiles && threadIdx.x < r.n_used) {  // decode: one tile per slot j (T == 1)
            const int j = threadIdx.x;
            r.tiles[j] = make_int4(ssel[j], j, 1, 0);
            r.pairs[j] = j;
        }
    }
    if (r.tiles && threadIdx.x == 0) *r.n_tiles = (int) r.n_used;
}

cudaError_t launch_router_fused(const RouterArgs &r, cudaStream_t s) {
    router_fused_kernel<<<(unsigned) r.E, 128, (size_t) r.E * 4, s>>>(r);
    return cudaGetLastError();
}

// ------------------------------------------------------- logits, up to 512 tokens
// One CTA per expert e: its router row staged in shared memory, one warp per token
// (lanes stride over h, warp-shuffle sum), so E CTAs stream the router weights once.
__global__ void __launch_bounds__(256) logits_rows_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                          float *__restrict__ out, int64_t T, int64_t E, int64_t H) {
    extern __shared__ float ws_row[];
    const int64_t e = blockIdx.x;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    for (int64_t h = tid; h < H; h += blockDim.x) ws_row[h] = w[e * H + h];
    __syncthreads();
    for (int64_t t = warp; t < T; t += blockDim.x >> 5) {
        const float *xr = x + t * H;
        float acc = 0.f;
        for (int64_t h = lane; h < H; h += 32) acc = fmaf(xr[h], ws_row[h], acc);
        acc = warp_sum(acc);
        if (lane == 0) out[t * E + e] = acc;
    }
}

// ------------------------------------------------------- logits GEMM (large T)
// logits[t][e] = sum_h x[t][h] * w[e][h]; 64x64 output tile per CTA, 256 threads, 4x4
// outputs per thread, K chunks of 16 staged in shared memory.
__global__ void __launch_bounds__(256) logits_gemm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                          float *__restrict__ out, int64_t T, int64_t E, int64_t H) {
    __shared__ float xs[16][64 + 4];
    __shared__ float ws[16][64 + 4];
    const int tid = threadIdx.x;
    const int64_t t0 = (int64_t) blockIdx.y * 64, e0 = (int64_t) blockIdx.x * 64;
    const int tr = tid / 16, tc = tid % 16;  // thread's 4x4 block: tokens tr*4.., experts tc*4..
    float acc[4][4] = {};
    for (int64_t h0 = 0; h0 < H; h0 += 16) {
        for (int i = tid; i < 64 * 16; i += 256) {
            const int rr = i / 16, kk = i % 16;
            const int64_t tt = t0 + rr, ee = e0 + rr;
            xs[kk][rr] = (tt < T && h0 + kk < H) ? x[tt * H + h0 + kk] : 0.f;
            ws[kk][rr] = (ee < E && h0 + kk < H) ? w[ee * H + h0 + kk] : 0.f;
        }
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) { a[i] = xs[kk][tr * 4 + i]; b[i] = ws[kk][tc * 4 + i]; }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t tt = t0 + tr * 4 + i, ee = e0 + tc * 4 + j;
            if (tt < T && ee < E) out[tt * E + ee] = acc[i][j];
        }
}

cudaError_t launch_logits_gemm(const float *x, const float *w, float *out, int64_t T, int64_t E, int64_t H,
                               cudaStream_t s) {
    if (T <= 512 && H * 4 <= 48 * 1024) {
        logits_rows_kernel<<<(unsigned) E, 256, (size_t) H * 4, s>>>(x, w, out, T, E, H);
        return cudaGetLastError();
    }
    dim3 grid((unsigned) ceil_div(E, 64), (unsigned) ceil_div(T, 64));
    logits_gemm_kernel<<<grid, 256, 0, s>>>(x, w, out, T, E, H);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ rms norm
// one CTA (128 threads) per row
__global__ void __launch_bounds__(128) rmsnorm_kernel(const float *__restrict__ x, const float *__restrict__ w,
                                                      float eps, int64_t H, float *__restrict__ y) {
    __shared__ double dpart[4];
    __shared__ float s_sc;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int64_t q = H / 4;
    const float *xr = x + (int64_t) blockIdx.x * H;
    const double v = warp_sumsq(xr + warp * q, q, lane);
    if (lane == 0) dpart[warp] = v;
    __syncthreads();
    if (threadIdx.x == 0) s_sc = rms_scale(((dpart[0] + dpart[1]) + dpart[2]) + dpart[3], H, eps);
    __syncthreads();
    const float sc = s_sc;
    float *yr = y + (int64_t) blockIdx.x * H;
    for (int64_t h = threadIdx.x; h < H; h += blockDim.x) yr[h] = __fmul_rn(__fmul_rn(xr[h], sc), w[h]);
}

cudaError_t launch_rmsnorm(const float *x, const float *w, float eps, int64_t T, int64_t H, float *y, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    rmsnorm_kernel<<<(unsigned) T, 128, 0, s>>>(x, w, eps, H, y);
    return cudaGetLastError();
}

// ------------------------------------------------------------------ swiglu
__global__ void swiglu_kernel(const float *__restrict__ g, const float *__restrict__ u, float *__restrict__ a,
                              int64_t n) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
}

// ------------------------------------------------- weighted expert reduction
// out[t][h] = sum_j w[t][j] * ex[t][j][h], j ascending, then + sh[t][h] (* sh_scale[t]),
// then + res[t][h] (the order of the reference graph: the routed sum, the shared expert's
// ggml_add, the layer's residual add)
__global__ void weighted_sum_kernel(const float *__restrict__ ex, const float *__restrict__ w,
                                    const float *__restrict__ sh, const float *__restrict__ sh_scale,
                                    const float *__restrict__ res, float *__restrict__ out, int64_t H, int n_used,
                                    int64_t T) {
    const int64_t i = (int64_t) blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= H * T) return;
    const int64_t t = i / H, h = i % H;
    const float *e = ex + t * n_used * H + h;
    const float *wt = w + t * n_used;
    float acc = 0.f;
    for (int j = 0; j < n_used; ++j) acc = fmaf(wt[j], e[(int64_t) j * H], acc);
    if (sh) acc = __fadd_rn(acc, sh_scale ? __fmul_rn(sh[i], sh_scale[t]) : sh[i]);
    if (res) acc += res[i];
    out[i] = acc;
}

cudaError_t launch_weighted_sum(const float *ex, const float *w, const float *res, float *out, int64_t H,
                                int64_t n_used, int64_t T, cudaStream_t s, const float *sh, const float *sh_scale) {
    const int64_t n = H * T;
    if (n == 0) return cudaSuccess;
    weighted_sum_kernel<<<(unsigned) ceil_div(n, 256), 256, 0, s>>>(ex, w, sh, sh_scale, res, out, H, (int) n_used, T);
    return cudaGetLastError();
}

// ------------------------------------------------- shared-expert gate
// scale[t] = sigmoid(gw . ffn_in[t]), ffn_in = rms_norm(x) * norm_w (or x): the
// ffn_gate_inp_shexp factor of core/runtime.cpp:2831-2832 (ggml_sigmoid_f32:
// 1 / (1 + exp(-v))).  One CTA (128 threads) per token; the normalisation is
// rmsnorm_kernel's.
__global__ void __launch_bounds__(128) shexp_gate_kernel(const float *__restrict__ x, const float *__restrict__ nw,
                                                         float eps, const float *__restrict__ gw, int64_t H,
                                                         float *__restrict__ scale) {
    __shared__ double dpart[4];
    __shared__ float fpart[4];
    __shared__ float s_sc;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const float *xr = x + (int64_t) blockIdx.x * H;
    if (nw) {
        const int64_t q = H / 4;
        const double v = warp_sumsq(xr + warp * q, q, lane);
        if (lane == 0) dpart[warp] = v;
        __syncthreads();
        if (threadIdx.x == 0) s_sc = rms_scale(((dpart[0] + dpart[1]) + dpart[2]) + dpart[3], H, eps);
        __syncthreads();
    }
    const float sc = nw ? s_sc : 1.f;
    float acc = 0.f;
    for (int64_t h = threadIdx.x; h < H; h += blockDim.x) {
        const float xi = nw ? __fmul_rn(__fmul_rn(xr[h], sc), nw[h]) : xr[h];
        acc = fmaf(gw[h], xi, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0) fpart[warp] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
        const float v = ((fpart[0] + fpart[1]) + fpart[2]) + fpart[3];
        scale[blockIdx.x] = 1.f / (1.f + expf(-v));
    }
}

cudaError_t launch_shexp_gate(const float *x, const float *norm_w, float eps, const float *gw, int64_t T, int64_t H,
                              float *scale, cudaStream_t s) {
    if (T == 0) return cudaSuccess;
    shexp_gate_kernel<<<(unsigned) T, 128, 0, s>>>(x, norm_w, eps, gw, H, scale);
    return cudaGetLastError();
}

}  // namespace qwb

using namespace qwb;

extern "C" QWB_API qwb_status qwb_moe_route(const float *logits, const float *mask, int64_t E, int64_t T,
                                            int64_t n_used, int norm, float scale, int32_t *selected,
                                            float *weights, qwb_stream_t stream) {
    if (E <= 0 || T < 0 || n_used <= 0) return QWB_ERR_INVALID_ARG;
    if (E > kMaxExperts || n_used > kMaxUsed || n_used > E) return QWB_ERR_LIMIT;
    if (T > 0x7fffffff) return QWB_ERR_LIMIT;
    if (T == 0) return QWB_OK;
    if (!logits || !selected || !weights) return QWB_ERR_INVALID_ARG;
    return launch_route(logits, mask, E, T, n_used, norm, scale, selected, weights, (cudaStream_t) stream) ==
                   cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
}

extern "C" QWB_API qwb_status qwb_swiglu(const float *gate, const float *up, float *act, int64_t n,
                                         qwb_stream_t stream) {
    if (n < 0) return QWB_ERR_INVALID_ARG;
    if (n == 0) return QWB_OK;
    if (!gate || !up || !act) return QWB_ERR_INVALID_ARG;
    swiglu_kernel<<<(unsigned) ceil_div(n, 256), 256, 0, (cudaStream_t) stream>>>(gate, up, act, n);
    return cudaGetLastError() == cudaSuccess ? QWB_OK : QWB_ERR_CUDA;
}

extern "C" QWB_API qwb_status qwb_moe_weighted_sum(const float *experts, const float *weights, float *out, int64_t H,
                                                   int64_t n_used, int64_t T, qwb_stream_t stream) {
    if (H < 0 || n_used <= 0 || T < 0) return QWB_ERR_INVALID_ARG;
    if (H == 0 || T == 0) return QWB_OK;
    if (!experts || !weights || !out) return QWB_ERR_INVALID_ARG;
    return launch_weighted_sum(experts, weights, nullptr, out, H, n_used, T, (cudaStream_t) stream) == cudaSuccess
                   ? QWB_OK : QWB_ERR_CUDA;
}
