/*
 * cpq_oracle.c — scalar restatement of ggml-cpu mul_mat semantics.
 *
 * TEST INFRASTRUCTURE ONLY (parity checker + CPU baseline); see cpq_oracle.h.
 * Compiled with -ffp-contract=off: the quantizers' multiply-then-round steps
 * are separate fp32 roundings in the reference (ggml-base is built without
 * -mfma), so no FMA contraction may merge them here.
 *
 * The reference algorithm lives in ggml at llama.cpp b10423
 * (scripts/fetch-deps.sh:6-7), which is not present in the reference tree;
 * each function below names the ggml routine whose published behaviour it
 * restates. The code is this project's own.
 */
#include "cpq_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* Provided by cpq_oracle_avx2.c when built with -mavx2 (weak fallback). */
int oq_avx2_block_ints_q4_K(const oq_block_q4_K *x, const oq_block_q8_K *y, int32_t *sc, int32_t *mn)
    __attribute__((weak));
int oq_avx2_block_ints_q6_K(const oq_block_q6_K *x, const oq_block_q8_K *y, int32_t *sc)
    __attribute__((weak));
int oq_avx2_block_int_q8_0(const oq_block_q8_0 *x, const oq_block_q8_0 *y, int32_t *s)
    __attribute__((weak));
void oq_avx2_quantize_row_q8_0(const float *x, oq_block_q8_0 *y, int64_t k) __attribute__((weak));

int oq_has_avx2(void) { return oq_avx2_block_ints_q4_K != NULL; }

int oq_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

size_t oq_type_block(int type) {
    switch (type) {
    case OQ_TYPE_F32: return 1;
    case OQ_TYPE_F16: return 1;
    case OQ_TYPE_Q8_0: return OQ_QK8_0;
    case OQ_TYPE_Q4_K: return OQ_QK_K;
    case OQ_TYPE_Q6_K: return OQ_QK_K;
    case OQ_TYPE_Q8_K: return OQ_QK_K;
    default: return 0;
    }
}

size_t oq_type_size(int type) {
    switch (type) {
    case OQ_TYPE_F32: return 4;
    case OQ_TYPE_F16: return 2;
    case OQ_TYPE_Q8_0: return sizeof(oq_block_q8_0);
    case OQ_TYPE_Q4_K: return sizeof(oq_block_q4_K);
    case OQ_TYPE_Q6_K: return sizeof(oq_block_q6_K);
    case OQ_TYPE_Q8_K: return sizeof(oq_block_q8_K);
    default: return 0;
    }
}

size_t oq_row_size(int type, int64_t k) {
    size_t b = oq_type_block(type);
    if (b == 0 || k % (int64_t)b != 0) return 0;
    return (size_t)(k / (int64_t)b) * oq_type_size(type);
}

/* ---- IEEE binary16 conversions (round to nearest even) ------------------ */

float oq_fp16_to_fp32(oq_half h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu;
    uint32_t m = h & 0x3ffu;
    uint32_t bits;
    if (e == 0) {
        float v = (float)m * 5.9604644775390625e-08f; /* m * 2^-24, exact */
        return sign ? -v : v;
    } else if (e == 31) {
        bits = sign | 0x7f800000u | (m << 13);
    } else {
        bits = sign | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

oq_half oq_fp32_to_fp16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax > 0x7f800000u) return (oq_half)(sign | 0x7e00u);  /* NaN */
    if (ax >= 0x477ff000u) return (oq_half)(sign | 0x7c00u); /* >= 65520 -> inf */
    if (ax < 0x38800000u) {
        /* below 2^-14: half subnormal m * 2^-24; scaling by 2^24 is exact */
        float a;
        memcpy(&a, &ax, 4);
        uint32_t m = (uint32_t)rintf(a * 16777216.0f);
        return (oq_half)(sign | m);
    }
    uint32_t e = ax >> 23, mant = ax & 0x7fffffu;
    uint32_t h = ((e - 112u) << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h += 1u;
    return (oq_half)(sign | h);
}

/* ---- activation quantizers ---------------------------------------------- */

/* Round half to even for |v| < 2^22: ggml's nearest_int adds 1.5*2^23 and
 * reads the low mantissa bits, which is an fp32 RNE to integer. */
static inline int nearest_int(float v) {
    float t = v + 12582912.0f;
    int32_t i;
    memcpy(&i, &t, 4);
    return (i & 0x007fffff) - 0x00400000;
}

/* Restates ggml quantize_row_q8_K_ref (ggml-quants.c; x86 ggml-cpu uses it
 * unchanged): per 256-block, the element of largest magnitude (first one on
 * ties) is `max`; iscale = -127/max; q = min(127, rne(iscale*x));
 * d = 1/iscale; bsums = sums of 16. An all-zero block stores d = 0 and zero
 * quants; ggml leaves its bsums unwritten there, this restatement stores 0. */
void oq_quantize_row_q8_K(const float *x, oq_block_q8_K *y, int64_t k) {
    const int64_t nb = k / OQ_QK_K;
    for (int64_t i = 0; i < nb; i++, x += OQ_QK_K) {
        float max = 0.0f, amax = 0.0f;
        for (int j = 0; j < OQ_QK_K; j++) {
            float ax = fabsf(x[j]);
            if (ax > amax) {
                amax = ax;
                max = x[j];
            }
        }
        if (amax == 0.0f) {
            y[i].d = 0.0f;
            memset(y[i].qs, 0, sizeof y[i].qs);
            memset(y[i].bsums, 0, sizeof y[i].bsums);
            continue;
        }
        const float iscale = -127.0f / max;
        for (int j = 0; j < OQ_QK_K; j++) {
            float p = iscale * x[j];
            int v = nearest_int(p);
            y[i].qs[j] = (int8_t)(v < 127 ? v : 127);
        }
        for (int g = 0; g < OQ_QK_K / 16; g++) {
            int s = 0;
            for (int l = 0; l < 16; l++) s += y[i].qs[g * 16 + l];
            y[i].bsums[g] = (int16_t)s;
        }
        y[i].d = 1.0f / iscale;
    }
}

/* Restates the two ggml Q8_0 quantizers (see OQ_Q8_0_* in the header).
 * x86 AVX2 (ggml-cpu arch/x86 quantize_row_q8_0): d = amax/127 stored fp16,
 * id = 127/amax (0 if amax == 0), q = round-half-even(x*id).
 * portable (quantize_row_q8_0_ref): d = amax/127, id = 1/d, q = roundf(x*id). */
void oq_quantize_row_q8_0(const float *x, oq_block_q8_0 *y, int64_t k, int variant) {
    const int64_t nb = k / OQ_QK8_0;
    for (int64_t i = 0; i < nb; i++, x += OQ_QK8_0) {
        float amax = 0.0f;
        for (int j = 0; j < OQ_QK8_0; j++) {
            float a = fabsf(x[j]);
            amax = a > amax ? a : amax;
        }
        const float d = amax / 127.0f;
        y[i].d = oq_fp32_to_fp16(d);
        if (variant == OQ_Q8_0_PORTABLE) {
            const float id = d != 0.0f ? 1.0f / d : 0.0f;
            for (int j = 0; j < OQ_QK8_0; j++) {
                float p = x[j] * id;
                y[i].qs[j] = (int8_t)roundf(p);
            }
        } else {
            const float id = amax != 0.0f ? 127.0f / amax : 0.0f;
            for (int j = 0; j < OQ_QK8_0; j++) {
                float p = x[j] * id;
                y[i].qs[j] = (int8_t)nearest_int(p);
            }
        }
    }
}

/* ---- weight dequantizers ------------------------------------------------- */

/* Q4_K six-bit scale/min unpack: sub-blocks 0-3 use the low 6 bits of bytes
 * 0-3 (scale) and 4-7 (min); sub-blocks 4-7 combine a nibble of bytes 8-11
 * with the top 2 bits of bytes 0-7 (ggml get_scale_min_k4). */
static inline void q4k_scale_min(int j, const uint8_t *q, int *sc, int *mn) {
    if (j < 4) {
        *sc = q[j] & 63;
        *mn = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        *mn = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

void oq_dequantize_row_q8_0(const oq_block_q8_0 *x, float *y, int64_t k) {
    for (int64_t i = 0; i < k / OQ_QK8_0; i++) {
        const float d = oq_fp16_to_fp32(x[i].d);
        for (int j = 0; j < OQ_QK8_0; j++) y[i * OQ_QK8_0 + j] = x[i].qs[j] * d;
    }
}

/* ggml dequantize_row_q4_K: for each 64-element chunk j, sub-block 2j is the
 * low nibbles of qs[32j..32j+31] and sub-block 2j+1 the high nibbles;
 * w = (d*sc)*q - (dmin*m). */
void oq_dequantize_row_q4_K(const oq_block_q4_K *x, float *y, int64_t k) {
    for (int64_t i = 0; i < k / OQ_QK_K; i++) {
        const float d = oq_fp16_to_fp32(x[i].d);
        const float dmin = oq_fp16_to_fp32(x[i].dmin);
        const uint8_t *q = x[i].qs;
        for (int j = 0; j < 4; j++) {
            int sc0, m0, sc1, m1;
            q4k_scale_min(2 * j, x[i].scales, &sc0, &m0);
            q4k_scale_min(2 * j + 1, x[i].scales, &sc1, &m1);
            const float d0 = d * sc0, mm0 = dmin * m0, d1 = d * sc1, mm1 = dmin * m1;
            for (int l = 0; l < 32; l++) *y++ = d0 * (q[l] & 0x0f) - mm0;
            for (int l = 0; l < 32; l++) *y++ = d1 * (q[l] >> 4) - mm1;
            q += 32;
        }
    }
}

/* Q6_K element order (ggml dequantize_row_q6_K): in each 128-element half,
 * element l (0..31) takes ql[l] low nibble + qh[l] bits 0-1, element l+32
 * ql[l+32] low + bits 2-3, l+64 ql[l] high + bits 4-5, l+96 ql[l+32] high +
 * bits 6-7; the value is q-32 scaled by d*scales[l/16 + {0,2,4,6}]. */
static inline void q6k_unpack(const oq_block_q6_K *b, int8_t *q /* 256 */) {
    const uint8_t *ql = b->ql, *qh = b->qh;
    for (int half = 0; half < 2; half++) {
        for (int l = 0; l < 32; l++) {
            q[l + 0] = (int8_t)(((ql[l] & 0x0f) | (((qh[l] >> 0) & 3) << 4)) - 32);
            q[l + 32] = (int8_t)(((ql[l + 32] & 0x0f) | (((qh[l] >> 2) & 3) << 4)) - 32);
            q[l + 64] = (int8_t)(((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32);
            q[l + 96] = (int8_t)(((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32);
        }
        q += 128;
        ql += 64;
        qh += 32;
    }
}

void oq_dequantize_row_q6_K(const oq_block_q6_K *x, float *y, int64_t k) {
    int8_t q[OQ_QK_K];
    for (int64_t i = 0; i < k / OQ_QK_K; i++) {
        const float d = oq_fp16_to_fp32(x[i].d);
        q6k_unpack(&x[i], q);
        for (int e = 0; e < OQ_QK_K; e++) {
            /* scale index of element e: 16-element group e/16 */
            y[i * OQ_QK_K + e] = d * x[i].scales[e / 16] * q[e];
        }
    }
}

/* ---- integer block totals ------------------------------------------------ */

void oq_block_ints_q4_K(const oq_block_q4_K *x, const oq_block_q8_K *y, int32_t *sc_out, int32_t *mn_out) {
    int32_t s = 0, m = 0;
    const uint8_t *q = x->qs;
    const int8_t *a = y->qs;
    for (int j = 0; j < 4; j++) {
        int sc0, m0, sc1, m1;
        q4k_scale_min(2 * j, x->scales, &sc0, &m0);
        q4k_scale_min(2 * j + 1, x->scales, &sc1, &m1);
        int32_t lo = 0, hi = 0;
        for (int l = 0; l < 32; l++) {
            lo += (q[l] & 0x0f) * a[l];
            hi += (q[l] >> 4) * a[l + 32];
        }
        s += sc0 * lo + sc1 * hi;
        m += m0 * (y->bsums[4 * j + 0] + y->bsums[4 * j + 1]) + m1 * (y->bsums[4 * j + 2] + y->bsums[4 * j + 3]);
        q += 32;
        a += 64;
    }
    *sc_out = s;
    *mn_out = m;
}

void oq_block_ints_q6_K(const oq_block_q6_K *x, const oq_block_q8_K *y, int32_t *sc_out) {
    int8_t q[OQ_QK_K];
    q6k_unpack(x, q);
    int32_t s = 0;
    for (int g = 0; g < 16; g++) {
        int32_t t = 0;
        for (int l = 0; l < 16; l++) t += q[g * 16 + l] * y->qs[g * 16 + l];
        s += x->scales[g] * t;
    }
    *sc_out = s;
}

int32_t oq_block_int_q8_0(const oq_block_q8_0 *x, const oq_block_q8_0 *y) {
    int32_t s = 0;
    for (int j = 0; j < OQ_QK8_0; j++) s += x->qs[j] * y->qs[j];
    return s;
}

/* ---- block dots ---------------------------------------------------------- */

/* ggml_vec_dot_q4_K_q8_K: sum over superblocks of
 *   (d_w*d_x) * sum_j sc_j sum_i q*q8  -  (dmin_w*d_x) * sum_j m_j * bsum_j. */
static float dot_q4_K(int64_t n, const oq_block_q4_K *x, const oq_block_q8_K *y, int simd) {
    float sumf = 0.0f;
    for (int64_t i = 0; i < n / OQ_QK_K; i++) {
        int32_t s, m;
        if (simd) oq_avx2_block_ints_q4_K(&x[i], &y[i], &s, &m);
        else oq_block_ints_q4_K(&x[i], &y[i], &s, &m);
        const float d = oq_fp16_to_fp32(x[i].d) * y[i].d;
        const float dmin = oq_fp16_to_fp32(x[i].dmin) * y[i].d;
        sumf += d * (float)s;
        sumf -= dmin * (float)m;
    }
    return sumf;
}

/* ggml_vec_dot_q6_K_q8_K: sum over superblocks of (d_w*d_x) * sum_g s_g sum (q-32)*q8. */
static float dot_q6_K(int64_t n, const oq_block_q6_K *x, const oq_block_q8_K *y, int simd) {
    float sumf = 0.0f;
    for (int64_t i = 0; i < n / OQ_QK_K; i++) {
        int32_t s;
        if (simd) oq_avx2_block_ints_q6_K(&x[i], &y[i], &s);
        else oq_block_ints_q6_K(&x[i], &y[i], &s);
        const float d = oq_fp16_to_fp32(x[i].d) * y[i].d;
        sumf += d * (float)s;
    }
    return sumf;
}

/* ggml_vec_dot_q8_0_q8_0: sum over blocks of sumi * (d_w * d_x). */
static float dot_q8_0(int64_t n, const oq_block_q8_0 *x, const oq_block_q8_0 *y, int simd) {
    float sumf = 0.0f;
    for (int64_t i = 0; i < n / OQ_QK8_0; i++) {
        int32_t s;
        if (simd) oq_avx2_block_int_q8_0(&x[i], &y[i], &s);
        else s = oq_block_int_q8_0(&x[i], &y[i]);
        sumf += (float)s * (oq_fp16_to_fp32(x[i].d) * oq_fp16_to_fp32(y[i].d));
    }
    return sumf;
}

float oq_vec_dot_q4_K_q8_K(int64_t n, const oq_block_q4_K *x, const oq_block_q8_K *y) { return dot_q4_K(n, x, y, 0); }
float oq_vec_dot_q6_K_q8_K(int64_t n, const oq_block_q6_K *x, const oq_block_q8_K *y) { return dot_q6_K(n, x, y, 0); }
float oq_vec_dot_q8_0_q8_0(int64_t n, const oq_block_q8_0 *x, const oq_block_q8_0 *y) { return dot_q8_0(n, x, y, 0); }

/* ---- mul_mat -------------------------------------------------------------- */

static int vec_dot_type(int wtype) {
    switch (wtype) {
    case OQ_TYPE_Q4_K:
    case OQ_TYPE_Q6_K: return OQ_TYPE_Q8_K;
    case OQ_TYPE_Q8_0: return OQ_TYPE_Q8_0;
    default: return -1;
    }
}

int oq_quantize_act(int wtype, const float *x, int64_t k, int64_t m, void *out, int q8_0_variant) {
    const int vt = vec_dot_type(wtype);
    if (vt < 0 || k <= 0 || m < 0) return -1;
    const size_t rs = oq_row_size(vt, k);
    if (rs == 0) return -1;
    for (int64_t r = 0; r < m; r++) {
        char *dst = (char *)out + (size_t)r * rs;
        if (vt == OQ_TYPE_Q8_K) {
            oq_quantize_row_q8_K(x + r * k, (oq_block_q8_K *)dst, k);
        } else if (q8_0_variant == OQ_Q8_0_X86_AVX2 && oq_avx2_quantize_row_q8_0) {
            oq_avx2_quantize_row_q8_0(x + r * k, (oq_block_q8_0 *)dst, k);
        } else {
            oq_quantize_row_q8_0(x + r * k, (oq_block_q8_0 *)dst, k, q8_0_variant);
        }
    }
    return 0;
}

int oq_mul_mat_q(int wtype, const void *w, int64_t k, int64_t n, size_t row_stride,
                 const void *xq, int64_t m, float *y, int nthreads, int simd) {
    const int vt = vec_dot_type(wtype);
    if (vt < 0 || k <= 0 || n < 0 || m < 0) return -1;
    const size_t wrs = oq_row_size(wtype, k);
    const size_t xrs = oq_row_size(vt, k);
    if (wrs == 0 || xrs == 0 || row_stride < wrs) return -1;
    if (simd && !oq_has_avx2()) simd = 0;
#ifdef _OPENMP
    if (nthreads <= 0) nthreads = omp_get_max_threads();
#pragma omp parallel for num_threads(nthreads) schedule(static)
#endif
    for (int64_t r = 0; r < n; r++) {
        const char *wr = (const char *)w + (size_t)r * row_stride;
        for (int64_t c = 0; c < m; c++) {
            const char *xr = (const char *)xq + (size_t)c * xrs;
            float v;
            if (wtype == OQ_TYPE_Q4_K) v = dot_q4_K(k, (const oq_block_q4_K *)wr, (const oq_block_q8_K *)xr, simd);
            else if (wtype == OQ_TYPE_Q6_K) v = dot_q6_K(k, (const oq_block_q6_K *)wr, (const oq_block_q8_K *)xr, simd);
            else v = dot_q8_0(k, (const oq_block_q8_0 *)wr, (const oq_block_q8_0 *)xr, simd);
            y[c * n + r] = v;
        }
    }
    (void)nthreads;
    return 0;
}

int oq_mul_mat(int wtype, const void *w, int64_t k, int64_t n, size_t row_stride,
               const float *x, int64_t m, float *y, int nthreads, int simd, int q8_0_variant) {
    const int vt = vec_dot_type(wtype);
    if (vt < 0) return -1;
    const size_t xrs = oq_row_size(vt, k);
    if (xrs == 0) return -1;
    void *xq = malloc(xrs * (size_t)(m > 0 ? m : 1));
    if (!xq) return -1;
    int rc = oq_quantize_act(wtype, x, k, m, xq, q8_0_variant);
    if (rc == 0) rc = oq_mul_mat_q(wtype, w, k, n, row_stride, xq, m, y, nthreads, simd);
    free(xq);
    return rc;
}

void oq_mul_mat_f32(const float *w, int64_t k, int64_t n, const float *x, int64_t m, float *y) {
    for (int64_t c = 0; c < m; c++)
        for (int64_t r = 0; r < n; r++) {
            float s = 0.0f;
            for (int64_t i = 0; i < k; i++) s += w[r * k + i] * x[c * k + i];
            y[c * n + r] = s;
        }
}
