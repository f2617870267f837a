/* qwb_oracle.c - CPU restatement of the reference's quantized MoE hot path.
 *
 * TEST INFRASTRUCTURE ONLY (the checker for tests/, smoke() and bench.py's
 * cpu_baseline leg).  Written from the algorithms of vendored ggml (llama.cpp
 * 1b70350c9); each function names the reference function and file:line it restates
 * (paths relative to third_party/ggml/src).  Scalar C, single thread: fast enough for
 * the small parity cases, not a performance baseline.
 *
 * Parity pinning: tests/test_oracle_pin.py compares every function here with the
 * reference's own ggml CPU backend (built from the reference sources by
 * oracle/Makefile into oracle/_ref) and with the committed golden fixtures.
 */
#include "qwb_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#define QK_K 256
#define QK8_0 32

/* Block layouts: ggml-common.h:251-255 (q8_0), :327-337 (q4_K), :362-367 (q6_K),
 * :370-375 (q8_K).  Same field order and sizes: the formats are the contract. */
typedef struct { uint16_t d; int8_t qs[QK8_0]; } blk_q8_0;                       /* 34 B  */
typedef struct { uint16_t d, dmin; uint8_t scales[12]; uint8_t qs[QK_K / 2]; } blk_q4_K; /* 144 B */
typedef struct { uint8_t ql[QK_K / 2]; uint8_t qh[QK_K / 4]; int8_t scales[QK_K / 16]; uint16_t d; } blk_q6_K; /* 210 B */
typedef struct { float d; int8_t qs[QK_K]; int16_t bsums[QK_K / 16]; } blk_q8_K;  /* 292 B */

_Static_assert(sizeof(blk_q8_0) == 34, "q8_0");
_Static_assert(sizeof(blk_q4_K) == 144, "q4_K");
_Static_assert(sizeof(blk_q6_K) == 210, "q6_K");
_Static_assert(sizeof(blk_q8_K) == 292, "q8_K");

size_t qo_row_size(int type, int64_t n) {
    switch (type) {
        case QO_TYPE_F32: case QO_TYPE_I32: return (size_t) n * 4;
        case QO_TYPE_F16: return (size_t) n * 2;
        case QO_TYPE_Q8_0: return (size_t) (n / QK8_0) * sizeof(blk_q8_0);
        case QO_TYPE_Q4_K: return (size_t) (n / QK_K) * sizeof(blk_q4_K);
        case QO_TYPE_Q6_K: return (size_t) (n / QK_K) * sizeof(blk_q6_K);
        case QO_TYPE_Q8_K: return (size_t) (n / QK_K) * sizeof(blk_q8_K);
        default: return 0;
    }
}

/* ---------------------------------------------------------------- IEEE half */
/* binary32 -> binary16, round to nearest, ties to even (IEEE 754 conversion rule; the
 * reference's GGML_FP32_TO_FP16 / F16C vcvtps2ph with imm 0 implement the same rule). */
uint16_t qo_fp32_to_fp16(float f) {
    uint32_t x; memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) {                       /* inf / nan */
        return (uint16_t) (sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u | ((ax >> 13) & 0x3ffu) : 0));
    }
    const int e = (int) (ax >> 23) - 127;          /* unbiased exponent */
    if (e > 15) return (uint16_t) (sign | 0x7c00u); /* overflow -> inf */
    uint32_t mant = (ax & 0x7fffffu) | 0x800000u;  /* 24-bit significand */
    int shift;                                     /* bits to drop from the 24-bit significand */
    uint32_t hexp;
    if (e >= -14) { shift = 13; hexp = (uint32_t) (e + 15); }
    else {
        if (ax == 0) return (uint16_t) sign;
        shift = 13 + (-14 - e);                    /* subnormal half */
        hexp = 0;
        if (shift > 24) return (uint16_t) sign;    /* rounds to zero */
    }
    uint32_t q = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (q & 1u))) q++;
    uint32_t h;
    if (hexp == 0) h = q;                          /* q may carry into the normal range: fine */
    else {
        h = (hexp << 10) + (q - 0x400u);           /* q in [0x400, 0x800]; carry bumps exponent */
    }
    return (uint16_t) (sign | h);
}

float qo_fp16_to_fp32(uint16_t h) {
    const uint32_t sign = (uint32_t) (h & 0x8000u) << 16;
    const uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) x = sign;
        else {                                     /* subnormal: value m * 2^-24 */
            float v = (float) m * 5.9604644775390625e-08f;
            memcpy(&x, &v, 4); x |= sign;
        }
    } else if (e == 31) x = sign | 0x7f800000u | (m << 13);
    else x = sign | ((e + 112u) << 23) | (m << 13);
    float f; memcpy(&f, &x, 4); return f;
}

/* ggml-quants.c:621-626 nearest_int: round to nearest, ties to even, by adding 1.5*2^23
 * (valid for |f| <= 4194303). */
static inline int nearest_int(float f) {
    float v = f + 12582912.f;
    int32_t i; memcpy(&i, &v, 4);
    return (i & 0x007fffff) - 0x00400000;
}

static inline int imin(int a, int b) { return a < b ? a : b; }
static inline int imax(int a, int b) { return a > b ? a : b; }

/* --------------------------------------------------------- weight quantizers */
/* ggml-quants.c:799-875 make_qkx2_quants: affine (scale, min) fit of n values to
 * [0, nmax] with a weighted least-squares search over nstep+1 candidate scales. */
static float make_qkx2(int n, int nmax, const float *x, const float *w, uint8_t *L,
                       float *the_min, uint8_t *Laux, float rmin, float rdelta, int nstep) {
    float mn = x[0], mx = x[0];
    float sum_w = w[0], sum_x = sum_w * x[0];
    for (int i = 1; i < n; ++i) {
        if (x[i] < mn) mn = x[i];
        if (x[i] > mx) mx = x[i];
        float wi = w[i];
        sum_w += wi;
        sum_x += wi * x[i];
    }
    if (mn > 0) mn = 0;
    if (mx == mn) {
        for (int i = 0; i < n; ++i) L[i] = 0;
        *the_min = -mn;
        return 0.f;
    }
    float iscale = nmax / (mx - mn);
    float scale = 1 / iscale;
    float best = 0;
    for (int i = 0; i < n; ++i) {
        int l = nearest_int(iscale * (x[i] - mn));
        L[i] = (uint8_t) imax(0, imin(nmax, l));
        float diff = scale * L[i] + mn - x[i];
        diff = diff * diff;
        best += w[i] * diff;
    }
    for (int is = 0; is <= nstep; ++is) {
        iscale = (rmin + rdelta * is + nmax) / (mx - mn);
        float sum_l = 0, sum_l2 = 0, sum_xl = 0;
        for (int i = 0; i < n; ++i) {
            int l = nearest_int(iscale * (x[i] - mn));
            l = imax(0, imin(nmax, l));
            Laux[i] = (uint8_t) l;
            float wi = w[i];
            sum_l += wi * l;
            sum_l2 += wi * l * l;
            sum_xl += wi * l * x[i];
        }
        float D = sum_w * sum_l2 - sum_l * sum_l;
        if (D > 0) {
            float this_scale = (sum_w * sum_xl - sum_x * sum_l) / D;
            float this_min = (sum_l2 * sum_x - sum_l * sum_xl) / D;
            if (this_min > 0) {
                this_min = 0;
                this_scale = sum_xl / sum_l2;
            }
            float cur = 0;
            for (int i = 0; i < n; ++i) {
                float diff = this_scale * Laux[i] + this_min - x[i];
                diff = diff * diff;
                cur += w[i] * diff;
            }
            if (cur < best) {
                for (int i = 0; i < n; ++i) L[i] = Laux[i];
                best = cur;
                scale = this_scale;
                mn = this_min;
            }
        }
    }
    *the_min = -mn;
    return scale;
}

/* ggml-quants.c:880-887 get_scale_min_k4: 6-bit scale j and min j from the 12 packed bytes */
static inline void scale_min_k4(int j, const uint8_t *q, uint8_t *d, uint8_t *m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t) ((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t) ((q[j + 4] >> 4) | ((q[j - 0] >> 6) << 4));
    }
}

/* ggml-quants.c:1458-1528 quantize_row_q4_K_ref */
static void quantize_q4_K_row(const float *x, blk_q4_K *y, int64_t k) {
    const int64_t nb = k / QK_K;
    uint8_t L[QK_K], Laux[32];
    float wts[32], mins[QK_K / 32], scales[QK_K / 32];
    for (int64_t i = 0; i < nb; ++i) {
        float max_scale = 0, max_min = 0;
        for (int j = 0; j < QK_K / 32; ++j) {
            float sum_x2 = 0;
            for (int l = 0; l < 32; ++l) sum_x2 += x[32 * j + l] * x[32 * j + l];
            float av_x = sqrtf(sum_x2 / 32);
            for (int l = 0; l < 32; ++l) wts[l] = av_x + fabsf(x[32 * j + l]);
            scales[j] = make_qkx2(32, 15, x + 32 * j, wts, L + 32 * j, &mins[j], Laux, -1.f, 0.1f, 20);
            if (scales[j] > max_scale) max_scale = scales[j];
            if (mins[j] > max_min) max_min = mins[j];
        }
        float inv_scale = max_scale > 0 ? 63.f / max_scale : 0.f;
        float inv_min = max_min > 0 ? 63.f / max_min : 0.f;
        memset(y[i].scales, 0, 12);
        for (int j = 0; j < QK_K / 32; ++j) {
            uint8_t ls = (uint8_t) nearest_int(inv_scale * scales[j]);
            uint8_t lm = (uint8_t) nearest_int(inv_min * mins[j]);
            if (ls > 63) ls = 63;
            if (lm > 63) lm = 63;
            if (j < 4) {
                y[i].scales[j] = ls;
                y[i].scales[j + 4] = lm;
            } else {
                y[i].scales[j + 4] = (uint8_t) ((ls & 0xF) | ((lm & 0xF) << 4));
                y[i].scales[j - 4] |= (uint8_t) ((ls >> 4) << 6);
                y[i].scales[j - 0] |= (uint8_t) ((lm >> 4) << 6);
            }
        }
        y[i].d = qo_fp32_to_fp16(max_scale / 63.f);
        y[i].dmin = qo_fp32_to_fp16(max_min / 63.f);
        for (int j = 0; j < QK_K / 32; ++j) {
            uint8_t sc, m;
            scale_min_k4(j, y[i].scales, &sc, &m);
            const float d = qo_fp16_to_fp32(y[i].d) * sc;
            if (!d) continue;
            const float dm = qo_fp16_to_fp32(y[i].dmin) * m;
            for (int ii = 0; ii < 32; ++ii) {
                int l = nearest_int((x[32 * j + ii] + dm) / d);
                L[32 * j + ii] = (uint8_t) imax(0, imin(15, l));
            }
        }
        uint8_t *q = y[i].qs;
        for (int j = 0; j < QK_K; j += 64) {
            for (int l = 0; l < 32; ++l) q[l] = (uint8_t) (L[j + l] | (L[j + l + 32] << 4));
            q += 32;
        }
        x += QK_K;
    }
}

/* ggml-quants.c:628-698 make_qx_quants, rmse_type 1 and no importance weights (the only
 * form quantize_row_q6_K_ref uses): symmetric scale fit with a 19-point search. */
static float make_qx_rmse1(int n, int nmax, const float *x, int8_t *L) {
    float mx = 0, amax = 0;
    for (int i = 0; i < n; ++i) {
        float ax = fabsf(x[i]);
        if (ax > amax) { amax = ax; mx = x[i]; }
    }
    if (amax < 1e-15f) {
        for (int i = 0; i < n; ++i) L[i] = 0;
        return 0.f;
    }
    float iscale = -nmax / mx;
    float sumlx = 0, suml2 = 0;
    for (int i = 0; i < n; ++i) {
        int l = nearest_int(iscale * x[i]);
        l = imax(-nmax, imin(nmax - 1, l));
        L[i] = (int8_t) (l + nmax);
        float w = x[i] * x[i];
        sumlx += w * x[i] * l;
        suml2 += w * l * l;
    }
    float scale = suml2 ? sumlx / suml2 : 0.0f;
    float best = scale * sumlx;
    for (int is = -9; is <= 9; ++is) {
        if (is == 0) continue;
        iscale = -(nmax + 0.1f * is) / mx;
        sumlx = suml2 = 0;
        for (int i = 0; i < n; ++i) {
            int l = nearest_int(iscale * x[i]);
            l = imax(-nmax, imin(nmax - 1, l));
            float w = x[i] * x[i];
            sumlx += w * x[i] * l;
            suml2 += w * l * l;
        }
        if (suml2 > 0 && sumlx * sumlx > best * suml2) {
            for (int i = 0; i < n; ++i) {
                int l = nearest_int(iscale * x[i]);
                L[i] = (int8_t) (nmax + imax(-nmax, imin(nmax - 1, l)));
            }
            scale = sumlx / suml2;
            best = scale * sumlx;
        }
    }
    return scale;
}

/* ggml-quants.c:1870-1936 quantize_row_q6_K_ref */
static void quantize_q6_K_row(const float *x, blk_q6_K *y, int64_t k) {
    const int64_t nb = k / QK_K;
    int8_t L[QK_K];
    float scales[QK_K / 16];
    for (int64_t i = 0; i < nb; ++i) {
        float max_scale = 0, max_abs_scale = 0;
        for (int ib = 0; ib < QK_K / 16; ++ib) {
            const float scale = make_qx_rmse1(16, 32, x + 16 * ib, L + 16 * ib);
            scales[ib] = scale;
            const float abs_scale = fabsf(scale);
            if (abs_scale > max_abs_scale) {
                max_abs_scale = abs_scale;
                max_scale = scale;
            }
        }
        if (max_abs_scale < 1e-15f) {
            memset(&y[i], 0, sizeof(blk_q6_K));
            y[i].d = qo_fp32_to_fp16(0.f);
            x += QK_K;
            continue;
        }
        float iscale = -128.f / max_scale;
        y[i].d = qo_fp32_to_fp16(1 / iscale);
        for (int ib = 0; ib < QK_K / 16; ++ib) y[i].scales[ib] = (int8_t) imin(127, nearest_int(iscale * scales[ib]));
        for (int j = 0; j < QK_K / 16; ++j) {
            float d = qo_fp16_to_fp32(y[i].d) * y[i].scales[j];
            if (!d) continue;
            for (int ii = 0; ii < 16; ++ii) {
                int l = nearest_int(x[16 * j + ii] / d);
                l = imax(-32, imin(31, l));
                L[16 * j + ii] = (int8_t) (l + 32);
            }
        }
        uint8_t *ql = y[i].ql, *qh = y[i].qh;
        for (int j = 0; j < QK_K; j += 128) {
            for (int l = 0; l < 32; ++l) {
                const uint8_t q1 = L[j + l + 0] & 0xF, q2 = L[j + l + 32] & 0xF;
                const uint8_t q3 = L[j + l + 64] & 0xF, q4 = L[j + l + 96] & 0xF;
                ql[l + 0] = (uint8_t) (q1 | (q3 << 4));
                ql[l + 32] = (uint8_t) (q2 | (q4 << 4));
                qh[l] = (uint8_t) ((L[j + l] >> 4) | ((L[j + l + 32] >> 4) << 2) |
                                   ((L[j + l + 64] >> 4) << 4) | ((L[j + l + 96] >> 4) << 6));
            }
            ql += 64;
            qh += 32;
        }
        x += QK_K;
    }
}

/* ggml-quants.c:276-300 quantize_row_q8_0_ref: d = amax/127, q = roundf(x * (1/d)) */
static void quantize_q8_0_ref_row(const float *x, blk_q8_0 *y, int64_t k) {
    const int64_t nb = k / QK8_0;
    for (int64_t i = 0; i < nb; ++i) {
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; ++j) {
            float a = fabsf(x[i * QK8_0 + j]);
            amax = amax > a ? amax : a;
        }
        const float d = amax / 127;
        const float id = d ? 1.0f / d : 0.0f;
        y[i].d = qo_fp32_to_fp16(d);
        for (int j = 0; j < QK8_0; ++j) y[i].qs[j] = (int8_t) roundf(x[i * QK8_0 + j] * id);
    }
}

int qo_quantize_weights(int type, const float *src, void *dst, int64_t nrow, int64_t n_per_row) {
    const size_t rs = qo_row_size(type, n_per_row);
    for (int64_t r = 0; r < nrow; ++r) {
        const float *x = src + r * n_per_row;
        char *y = (char *) dst + r * rs;
        switch (type) {
            case QO_TYPE_Q4_K: quantize_q4_K_row(x, (blk_q4_K *) y, n_per_row); break;
            case QO_TYPE_Q6_K: quantize_q6_K_row(x, (blk_q6_K *) y, n_per_row); break;
            case QO_TYPE_Q8_0: quantize_q8_0_ref_row(x, (blk_q8_0 *) y, n_per_row); break;
            default: return -1;
        }
    }
    return 0;
}

/* ------------------------------------------------------ activation quantizers */
/* ggml-quants.c:2769-2806 quantize_row_q8_K_ref (= the x86 CPU backend's quantize_row_q8_K,
 * arch/x86/quants.c:505): keep the signed value of the first max |x|, iscale = -127/max,
 * q = min(127, nearest_int(iscale*x)), 16 bsums, d = 1/iscale. */
void qo_quantize_row_q8_K(const float *x, void *vy, int64_t k) {
    blk_q8_K *y = (blk_q8_K *) vy;
    const int64_t nb = k / QK_K;
    for (int64_t i = 0; i < nb; ++i) {
        float mx = 0, amax = 0;
        for (int j = 0; j < QK_K; ++j) {
            float ax = fabsf(x[j]);
            if (ax > amax) { amax = ax; mx = x[j]; }
        }
        if (!amax) {
            y[i].d = 0;
            memset(y[i].qs, 0, QK_K);
            /* the reference leaves bsums untouched here; zero them so the output is defined */
            memset(y[i].bsums, 0, sizeof(y[i].bsums));
            x += QK_K;
            continue;
        }
        const float iscale = -127.f / mx;
        for (int j = 0; j < QK_K; ++j) {
            int v = nearest_int(iscale * x[j]);
            y[i].qs[j] = (int8_t) imin(127, v);
        }
        for (int j = 0; j < QK_K / 16; ++j) {
            int sum = 0;
            for (int ii = 0; ii < 16; ++ii) sum += y[i].qs[j * 16 + ii];
            y[i].bsums[j] = (int16_t) sum;
        }
        y[i].d = 1 / iscale;
        x += QK_K;
    }
}

/* Q8_0 activations.
 * QO_Q8_0_CPU: arch/x86/quants.c:302-360 (AVX path the CPU backend uses): d = max/127.f,
 *              id = 127.f/max, q = round-half-even(x*id).
 * QO_Q8_0_REF: ggml-quants.c:276-300. */
void qo_quantize_row_q8_0(const float *x, void *vy, int64_t k, int variant) {
    blk_q8_0 *y = (blk_q8_0 *) vy;
    if (variant == QO_Q8_0_REF) { quantize_q8_0_ref_row(x, y, k); return; }
    const int64_t nb = k / QK8_0;
    for (int64_t i = 0; i < nb; ++i) {
        float amax = 0.0f;
        for (int j = 0; j < QK8_0; ++j) {
            float a = fabsf(x[i * QK8_0 + j]);
            amax = a > amax ? a : amax;
        }
        const float d = amax / 127.f;
        y[i].d = qo_fp32_to_fp16(d);
        const float id = amax != 0.0f ? 127.f / amax : 0.0f;
        for (int j = 0; j < QK8_0; ++j) y[i].qs[j] = (int8_t) (int) rintf(x[i * QK8_0 + j] * id);
    }
}

/* ---------------------------------------------------------------- dequantize */
/* ggml-quants.c:1530-1552 dequantize_row_q4_K, :1940-1969 dequantize_row_q6_K,
 * :553 dequantize_row_q8_0 */
int qo_to_float(int type, const void *vx, float *y, int64_t nrow, int64_t k) {
    const size_t rs = qo_row_size(type, k);
    for (int64_t r = 0; r < nrow; ++r) {
        const char *row = (const char *) vx + r * rs;
        float *yr = y + r * k;
        switch (type) {
        case QO_TYPE_F32: memcpy(yr, row, (size_t) k * 4); break;
        case QO_TYPE_F16:
            for (int64_t j = 0; j < k; ++j) yr[j] = qo_fp16_to_fp32(((const uint16_t *) row)[j]);
            break;
        case QO_TYPE_Q8_0: {
            const blk_q8_0 *x = (const blk_q8_0 *) row;
            for (int64_t i = 0; i < k / QK8_0; ++i) {
                const float d = qo_fp16_to_fp32(x[i].d);
                for (int j = 0; j < QK8_0; ++j) yr[i * QK8_0 + j] = x[i].qs[j] * d;
            }
        } break;
        case QO_TYPE_Q4_K: {
            const blk_q4_K *x = (const blk_q4_K *) row;
            float *o = yr;
            for (int64_t i = 0; i < k / QK_K; ++i) {
                const uint8_t *q = x[i].qs;
                const float d = qo_fp16_to_fp32(x[i].d), mn = qo_fp16_to_fp32(x[i].dmin);
                int is = 0;
                for (int j = 0; j < QK_K; j += 64) {
                    uint8_t sc, m;
                    scale_min_k4(is + 0, x[i].scales, &sc, &m);
                    const float d1 = d * sc, m1 = mn * m;
                    scale_min_k4(is + 1, x[i].scales, &sc, &m);
                    const float d2 = d * sc, m2 = mn * m;
                    for (int l = 0; l < 32; ++l) *o++ = d1 * (q[l] & 0xF) - m1;
                    for (int l = 0; l < 32; ++l) *o++ = d2 * (q[l] >> 4) - m2;
                    q += 32;
                    is += 2;
                }
            }
        } break;
        case QO_TYPE_Q6_K: {
            const blk_q6_K *x = (const blk_q6_K *) row;
            float *o = yr;
            for (int64_t i = 0; i < k / QK_K; ++i) {
                const float d = qo_fp16_to_fp32(x[i].d);
                const uint8_t *ql = x[i].ql, *qh = x[i].qh;
                const int8_t *sc = x[i].scales;
                for (int n = 0; n < QK_K; n += 128) {
                    for (int l = 0; l < 32; ++l) {
                        int is = l / 16;
                        const int8_t q1 = (int8_t) ((ql[l + 0] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                        const int8_t q2 = (int8_t) ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                        const int8_t q3 = (int8_t) ((ql[l + 0] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                        const int8_t q4 = (int8_t) ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                        o[l + 0] = d * sc[is + 0] * q1;
                        o[l + 32] = d * sc[is + 2] * q2;
                        o[l + 64] = d * sc[is + 4] * q3;
                        o[l + 96] = d * sc[is + 6] * q4;
                    }
                    o += 128;
                    ql += 64;
                    qh += 32;
                    sc += 8;
                }
            }
        } break;
        default: return -1;
        }
    }
    return 0;
}

/* -------------------------------------------------------------- dot products */
/* ggml-cpu/quants.c:696-768 ggml_vec_dot_q4_K_q8_K: integer sub-block dots, then per
 * superblock d = fp16(x.d)*y.d times the scaled integer sum, minus dmin*y.d*sum(m*bsums). */
static float dot_q4_K_q8_K(int64_t n, const blk_q4_K *x, const blk_q8_K *y) {
    const int64_t nb = n / QK_K;
    float sumf = 0;
    for (int64_t i = 0; i < nb; ++i) {
        uint8_t sc[8], m[8];
        for (int j = 0; j < 8; ++j) scale_min_k4(j, x[i].scales, &sc[j], &m[j]);
        int32_t summ = 0;
        for (int j = 0; j < QK_K / 16; ++j) summ += y[i].bsums[j] * m[j / 2];
        int32_t sumi = 0;
        for (int g = 0; g < 4; ++g) {              /* 64-value groups: low nibbles, high nibbles */
            const uint8_t *q4 = x[i].qs + 32 * g;
            const int8_t *q8 = y[i].qs + 64 * g;
            int32_t s_lo = 0, s_hi = 0;
            for (int l = 0; l < 32; ++l) {
                s_lo += (q4[l] & 0xF) * q8[l];
                s_hi += (q4[l] >> 4) * q8[l + 32];
            }
            sumi += sc[2 * g] * s_lo + sc[2 * g + 1] * s_hi;
        }
        const float d = qo_fp16_to_fp32(x[i].d) * y[i].d;
        const float dmin = qo_fp16_to_fp32(x[i].dmin) * y[i].d;
        sumf += d * (float) sumi - dmin * (float) summ;
    }
    return sumf;
}

/* ggml-cpu/quants.c:851-915 ggml_vec_dot_q6_K_q8_K */
static float dot_q6_K_q8_K(int64_t n, const blk_q6_K *x, const blk_q8_K *y) {
    const int64_t nb = n / QK_K;
    float sumf = 0;
    for (int64_t i = 0; i < nb; ++i) {
        int8_t a[QK_K];
        const uint8_t *ql = x[i].ql, *qh = x[i].qh;
        for (int j = 0; j < QK_K; j += 128) {
            for (int l = 0; l < 32; ++l) {
                a[j + l + 0] = (int8_t) ((ql[l + 0] & 0xF) | (((qh[l] >> 0) & 3) << 4)) - 32;
                a[j + l + 32] = (int8_t) ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                a[j + l + 64] = (int8_t) ((ql[l + 0] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                a[j + l + 96] = (int8_t) ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
            }
            ql += 64;
            qh += 32;
        }
        int32_t sumi = 0;
        for (int j = 0; j < QK_K / 16; ++j) {
            int32_t s = 0;
            for (int l = 0; l < 16; ++l) s += a[16 * j + l] * y[i].qs[16 * j + l];
            sumi += x[i].scales[j] * s;
        }
        sumf += qo_fp16_to_fp32(x[i].d) * y[i].d * (float) sumi;
    }
    return sumf;
}

/* ggml-cpu/quants.c:451-480 ggml_vec_dot_q8_0_q8_0 */
static float dot_q8_0_q8_0(int64_t n, const blk_q8_0 *x, const blk_q8_0 *y) {
    const int64_t nb = n / QK8_0;
    float sumf = 0;
    for (int64_t i = 0; i < nb; ++i) {
        int32_t sumi = 0;
        for (int j = 0; j < QK8_0; ++j) sumi += x[i].qs[j] * y[i].qs[j];
        sumf += (float) sumi * (qo_fp16_to_fp32(x[i].d) * qo_fp16_to_fp32(y[i].d));
    }
    return sumf;
}

float qo_vec_dot(int type, int64_t k, const void *w, const void *a) {
    switch (type) {
        case QO_TYPE_Q4_K: return dot_q4_K_q8_K(k, (const blk_q4_K *) w, (const blk_q8_K *) a);
        case QO_TYPE_Q6_K: return dot_q6_K_q8_K(k, (const blk_q6_K *) w, (const blk_q8_K *) a);
        case QO_TYPE_Q8_0: return dot_q8_0_q8_0(k, (const blk_q8_0 *) w, (const blk_q8_0 *) a);
        default: return NAN;
    }
}

static int vec_dot_type(int type) { return type == QO_TYPE_Q8_0 ? QO_TYPE_Q8_0 : QO_TYPE_Q8_K; }

static void from_float(int vdt, const float *x, void *y, int64_t k, int q8_0_variant) {
    if (vdt == QO_TYPE_Q8_K) qo_quantize_row_q8_K(x, y, k);
    else qo_quantize_row_q8_0(x, y, k, q8_0_variant);
}

/* ggml-cpu/ggml-cpu.c:1554-1736 ggml_compute_forward_mul_mat_id: quantize every src1 row
 * with from_float (:1609-1644), then dst[:, slot, t] = as[:, :, ids[slot, t]] .
 * b[:, slot % n_b, t] via the type's vec_dot (:1483-1544).  Row grouping by expert is a
 * scheduling detail and does not change any value. */
int qo_mul_mat_id(int type, const void *as, int64_t K, int64_t M, int64_t n_as,
                  const float *b, int64_t n_b, int64_t T,
                  const int32_t *ids, int64_t n_used, int64_t ids_stride,
                  float *dst, int q8_0_variant) {
    const int vdt = vec_dot_type(type);
    const size_t ars = qo_row_size(vdt, K), wrs = qo_row_size(type, K);
    char *qa = (char *) malloc(ars * (size_t) (n_b * T));
    if (!qa) return -2;
    for (int64_t r = 0; r < n_b * T; ++r) from_float(vdt, b + r * K, qa + r * ars, K, q8_0_variant);
    int rc = 0;
    for (int64_t t = 0; t < T; ++t) {
        for (int64_t j = 0; j < n_used; ++j) {
            const int32_t e = ids[t * ids_stride + j];
            float *o = dst + (t * n_used + j) * M;
            if (e < 0 || e >= n_as) { rc = -1; for (int64_t m = 0; m < M; ++m) o[m] = 0; continue; }
            const char *w = (const char *) as + (size_t) e * M * wrs;
            const char *a = qa + (t * n_b + (j % n_b)) * ars;
            for (int64_t m = 0; m < M; ++m) o[m] = qo_vec_dot(type, K, w + m * wrs, a);
        }
    }
    free(qa);
    return rc;
}

/* ggml-cpu/ops.cpp:5204-5240 get_rows_q (dequantize_row of the indexed row) and
 * :5371 get_rows for F32 / F16 / I32 (plain copies). */
int qo_get_rows(int type, const void *src, int64_t ne0, int64_t nrows,
                const int32_t *idx, int64_t n, void *dst) {
    const size_t rs = qo_row_size(type, ne0);
    int rc = 0;
    for (int64_t i = 0; i < n; ++i) {
        const int32_t r = idx[i];
        if (r < 0 || r >= nrows) {
            rc = -1;
            memset((char *) dst + (size_t) i * ne0 * 4, 0, (size_t) ne0 * 4);
            continue;
        }
        const char *row = (const char *) src + (size_t) r * rs;
        if (type == QO_TYPE_I32) memcpy((char *) dst + (size_t) i * ne0 * 4, row, (size_t) ne0 * 4);
        else qo_to_float(type, row, (float *) dst + i * ne0, 1, ne0);
    }
    return rc;
}

/* core/runtime.cpp:2693-2734 route_experts on the CPU backend: soft_max_f32
 * (ops.cpp:5813: exp(x - max), sum in double, scale by 1/sum), argsort descending and the
 * top-k view (ggml.c:5462, ops.cpp:8717), get_rows of probs, sum_rows, clamp, div, scale. */
void qo_route(const float *logits, int64_t E, int64_t T, int64_t n_used, int norm, float scale,
              const float *mask, int32_t *selected, float *weights) {
    float *p = (float *) malloc(sizeof(float) * (size_t) E);
    for (int64_t t = 0; t < T; ++t) {
        const float *l = logits + t * E;
        float mx = -INFINITY;
        for (int64_t e = 0; e < E; ++e) {
            p[e] = l[e] + (mask ? mask[t * E + e] : 0.0f);
            if (p[e] > mx) mx = p[e];
        }
        double sum = 0;
        for (int64_t e = 0; e < E; ++e) { p[e] = expf(p[e] - mx); sum += p[e]; }
        const float inv = (float) (1.0 / sum);
        for (int64_t e = 0; e < E; ++e) p[e] *= inv;
        /* top-k by repeated selection: larger prob first, lower index on ties */
        int32_t *sel = selected + t * n_used;
        for (int64_t j = 0; j < n_used; ++j) {
            int64_t best = -1;
            for (int64_t e = 0; e < E; ++e) {
                int taken = 0;
                for (int64_t q = 0; q < j; ++q) if (sel[q] == e) { taken = 1; break; }
                if (taken) continue;
                if (best < 0 || p[e] > p[best]) best = e;
            }
            sel[j] = (int32_t) best;
        }
        float *w = weights + t * n_used;
        float ws = 0;
        for (int64_t j = 0; j < n_used; ++j) { w[j] = p[sel[j]]; ws += w[j]; }
        if (norm) {
            if (ws < 6.103515625e-5f) ws = 6.103515625e-5f;
            for (int64_t j = 0; j < n_used; ++j) w[j] = w[j] / ws;
        }
        if (scale != 0.0f && scale != 1.0f) for (int64_t j = 0; j < n_used; ++j) w[j] *= scale;
    }
    free(p);
}

/* ops.cpp:3331-3389 swiglu_f32 / vec.cpp:417-447 ggml_vec_swiglu_f32: silu(g)*u with
 * silu(g) = g / (1 + exp(-g)) (the reference evaluates exp with its own vector expf). */
void qo_swiglu(const float *g, const float *u, float *act, int64_t n) {
    for (int64_t i = 0; i < n; ++i) act[i] = g[i] / (1.0f + expf(-g[i])) * u[i];
}

/* core/runtime.cpp:2743-2816 build_moe (and :2769-2778 slot remap): see header. */
int qo_moe_layer(const float *x, int64_t H, int64_t T,
                 const float *router_w, int64_t E, int64_t n_used,
                 int type_gu, const void *gate, const void *up,
                 int type_d, const void *down, int64_t F, int64_t n_mat,
                 const int32_t *g2s, const float *mask,
                 float *out, int32_t *selected, float *weights, float *act_out) {
    float *logits = (float *) malloc(sizeof(float) * (size_t) (E * T));
    int32_t *sel = (int32_t *) malloc(sizeof(int32_t) * (size_t) (n_used * T));
    float *w = (float *) malloc(sizeof(float) * (size_t) (n_used * T));
    int32_t *ids[3];
    float *g = (float *) malloc(sizeof(float) * (size_t) (F * n_used * T));
    float *u = (float *) malloc(sizeof(float) * (size_t) (F * n_used * T));
    float *a = (float *) malloc(sizeof(float) * (size_t) (F * n_used * T));
    float *ex = (float *) malloc(sizeof(float) * (size_t) (H * n_used * T));
    int rc = 0;
    /* router: mul_mat f32 x f32 (dot of each router row with x) */
    for (int64_t t = 0; t < T; ++t)
        for (int64_t e = 0; e < E; ++e) {
            float s = 0;
            for (int64_t h = 0; h < H; ++h) s += router_w[e * H + h] * x[t * H + h];
            logits[t * E + e] = s;
        }
    qo_route(logits, E, T, n_used, 1, 0.0f, mask, sel, w);
    for (int r = 0; r < 3; ++r) {
        ids[r] = (int32_t *) malloc(sizeof(int32_t) * (size_t) (n_used * T));
        for (int64_t i = 0; i < n_used * T; ++i) ids[r][i] = g2s ? g2s[r * E + sel[i]] : sel[i];
    }
    rc |= qo_mul_mat_id(type_gu, up, H, F, n_mat, x, 1, T, ids[1], n_used, n_used, u, QO_Q8_0_CPU);
    rc |= qo_mul_mat_id(type_gu, gate, H, F, n_mat, x, 1, T, ids[0], n_used, n_used, g, QO_Q8_0_CPU);
    qo_swiglu(g, u, a, F * n_used * T);
    rc |= qo_mul_mat_id(type_d, down, F, H, n_mat, a, n_used, T, ids[2], n_used, n_used, ex, QO_Q8_0_CPU);
    for (int64_t t = 0; t < T; ++t)
        for (int64_t h = 0; h < H; ++h) {
            float s = 0;
            for (int64_t j = 0; j < n_used; ++j) s += ex[(t * n_used + j) * H + h] * w[t * n_used + j];
            out[t * H + h] = s;
        }
    if (selected) memcpy(selected, sel, sizeof(int32_t) * (size_t) (n_used * T));
    if (weights) memcpy(weights, w, sizeof(float) * (size_t) (n_used * T));
    if (act_out) memcpy(act_out, a, sizeof(float) * (size_t) (F * n_used * T));
    for (int r = 0; r < 3; ++r) free(ids[r]);
    free(logits); free(sel); free(w); free(g); free(u); free(a); free(ex);
    return rc;
}

/* ggml-cpu/ops.cpp:4107-4162 ggml_compute_forward_rms_norm_f32 fused with the following
 * MUL by the norm weight: sum of f32 squares accumulated in double, mean = (float)
 * (sum / H), scale = 1/sqrtf(mean + eps), y = x * scale * w. */
void qo_rms_norm_mul(const float *x, const float *w, float eps, int64_t T, int64_t H, float *y) {
    for (int64_t t = 0; t < T; ++t) {
        const float *xr = x + t * H;
        double sum = 0.0;
        for (int64_t i = 0; i < H; ++i) sum += (double) (xr[i] * xr[i]);
        const float mean = (float) (sum / (double) H);
        const float scale = 1.0f / sqrtf(mean + eps);
        for (int64_t i = 0; i < H; ++i) y[t * H + i] = xr[i] * scale * w[i];
    }
}

/* ------------------------------------------------------------ expert pool byte audit */

/* FNV-1a 64 over n bytes: core/expert_weight_audit.h:83-87 (offset basis, then per byte
 * xor and multiply by the FNV prime, modulo 2^64). */
uint64_t qo_fnv1a64(const uint8_t *p, size_t n) {
    uint64_t h = 14695981039346656037ull;
    for (size_t i = 0; i < n; ++i) {
        h ^= p[i];
        h *= 1099511628211ull;
    }
    return h;
}

/* ExpertWeightAudit::compare (core/expert_weight_audit.h:106-125): memcmp equality, the
 * first index where the bytes differ and the two bytes there, both checksums. */
void qo_slab_audit(const uint8_t *expected, const uint8_t *actual, size_t n, int32_t *equal,
                   uint64_t *first_difference, uint32_t *expected_byte, uint32_t *actual_byte,
                   uint64_t *expected_fnv, uint64_t *actual_fnv) {
    size_t first = 0;
    while (first < n && actual[first] == expected[first]) ++first;
    *equal = first == n;
    *first_difference = first;
    *expected_byte = first < n ? expected[first] : 0u;
    *actual_byte = first < n ? actual[first] : 0u;
    *expected_fnv = qo_fnv1a64(expected, n);
    *actual_fnv = qo_fnv1a64(actual, n);
}
