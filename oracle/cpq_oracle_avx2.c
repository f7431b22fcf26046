/*
 * cpq_oracle_avx2.c — AVX2 integer block totals for the CPU oracle.
 *
 * TEST INFRASTRUCTURE ONLY (timed CPU baseline); see cpq_oracle.h. The
 * reference builds ggml-cpu with AVX2/FMA/F16C (codpiece-ggml-sys/build.rs:
 * 59-63), so the baseline uses the same instruction set. The functions here
 * compute exactly the integers that the scalar routines in cpq_oracle.c
 * compute (integer arithmetic has no rounding), so the oracle's output is
 * bit-identical with or without them; tests check that.
 */
#include <immintrin.h>
#include <string.h>

#include "cpq_oracle.h"

static inline int32_t hsum_i32(__m256i v) {
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4e));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xb1));
    return _mm_cvtsi128_si32(s);
}

/* six-bit scales and mins of a Q4_K block as two 8-byte arrays */
static inline void q4k_unpack_scales(const uint8_t *s, uint8_t sc[8], uint8_t mn[8]) {
    uint32_t w0, w1, w2;
    memcpy(&w0, s + 0, 4);
    memcpy(&w1, s + 4, 4);
    memcpy(&w2, s + 8, 4);
    const uint32_t lo6 = 0x3f3f3f3fu, lo4 = 0x0f0f0f0fu, lo2 = 0x03030303u;
    uint32_t sc_lo = w0 & lo6;
    uint32_t mn_lo = w1 & lo6;
    uint32_t sc_hi = (w2 & lo4) | (((w0 >> 6) & lo2) << 4);
    uint32_t mn_hi = ((w2 >> 4) & lo4) | (((w1 >> 6) & lo2) << 4);
    memcpy(sc, &sc_lo, 4);
    memcpy(sc + 4, &sc_hi, 4);
    memcpy(mn, &mn_lo, 4);
    memcpy(mn + 4, &mn_hi, 4);
}

int oq_avx2_block_ints_q4_K(const oq_block_q4_K *x, const oq_block_q8_K *y, int32_t *sc_out, int32_t *mn_out) {
    uint8_t sc[8], mn[8];
    q4k_unpack_scales(x->scales, sc, mn);
    const __m256i lo4 = _mm256_set1_epi8(0x0f);
    __m256i acc = _mm256_setzero_si256();
    for (int j = 0; j < 4; j++) {
        __m256i q = _mm256_loadu_si256((const __m256i *)(x->qs + 32 * j));
        __m256i ql = _mm256_and_si256(q, lo4);
        __m256i qh = _mm256_and_si256(_mm256_srli_epi16(q, 4), lo4);
        __m256i al = _mm256_loadu_si256((const __m256i *)(y->qs + 64 * j));
        __m256i ah = _mm256_loadu_si256((const __m256i *)(y->qs + 64 * j + 32));
        /* u8 x s8 pair sums fit int16: 15*127*2 < 32767 */
        __m256i pl = _mm256_maddubs_epi16(ql, al);
        __m256i ph = _mm256_maddubs_epi16(qh, ah);
        pl = _mm256_madd_epi16(pl, _mm256_set1_epi16(sc[2 * j]));
        ph = _mm256_madd_epi16(ph, _mm256_set1_epi16(sc[2 * j + 1]));
        acc = _mm256_add_epi32(acc, _mm256_add_epi32(pl, ph));
    }
    int32_t m = 0;
    for (int g = 0; g < 16; g++) m += mn[g / 2] * y->bsums[g];
    *sc_out = hsum_i32(acc);
    *mn_out = m;
    return 0;
}

int oq_avx2_block_ints_q6_K(const oq_block_q6_K *x, const oq_block_q8_K *y, int32_t *sc_out) {
    const __m256i lo4 = _mm256_set1_epi8(0x0f);
    const __m256i lo2 = _mm256_set1_epi8(0x03);
    __m256i acc = _mm256_setzero_si256();
    for (int half = 0; half < 2; half++) {
        const uint8_t *ql = x->ql + 64 * half;
        const uint8_t *qh = x->qh + 32 * half;
        const int8_t *a = y->qs + 128 * half;
        const int8_t *s = x->scales + 8 * half;
        __m256i l0 = _mm256_loadu_si256((const __m256i *)ql);
        __m256i l1 = _mm256_loadu_si256((const __m256i *)(ql + 32));
        __m256i h = _mm256_loadu_si256((const __m256i *)qh);
        /* four 32-element runs, each q in 0..63 before the -32 offset */
        __m256i q[4];
        q[0] = _mm256_or_si256(_mm256_and_si256(l0, lo4), _mm256_slli_epi16(_mm256_and_si256(h, lo2), 4));
        q[1] = _mm256_or_si256(_mm256_and_si256(l1, lo4),
                               _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(h, 2), lo2), 4));
        q[2] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(l0, 4), lo4),
                               _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(h, 4), lo2), 4));
        q[3] = _mm256_or_si256(_mm256_and_si256(_mm256_srli_epi16(l1, 4), lo4),
                               _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(h, 6), lo2), 4));
        for (int r = 0; r < 4; r++) {
            __m256i av = _mm256_loadu_si256((const __m256i *)(a + 32 * r));
            /* (q-32)*a = q*a - 32*a; u8 x s8 pair sums: 63*127*2 < 32767 */
            __m256i p = _mm256_maddubs_epi16(q[r], av);
            __m256i o = _mm256_maddubs_epi16(_mm256_set1_epi8(32), av);
            p = _mm256_sub_epi16(p, o);
            /* 16-element groups of this run: scales s[2r] (low 16) and s[2r+1] */
            __m256i sv = _mm256_setr_epi16(s[2 * r], s[2 * r], s[2 * r], s[2 * r], s[2 * r], s[2 * r], s[2 * r],
                                           s[2 * r], s[2 * r + 1], s[2 * r + 1], s[2 * r + 1], s[2 * r + 1],
                                           s[2 * r + 1], s[2 * r + 1], s[2 * r + 1], s[2 * r + 1]);
            acc = _mm256_add_epi32(acc, _mm256_madd_epi16(p, sv));
        }
    }
    *sc_out = hsum_i32(acc);
    return 0;
}

int oq_avx2_block_int_q8_0(const oq_block_q8_0 *x, const oq_block_q8_0 *y, int32_t *s) {
    __m256i a = _mm256_loadu_si256((const __m256i *)x->qs);
    __m256i b = _mm256_loadu_si256((const __m256i *)y->qs);
    /* s8 x s8: widen both to int16 and pair-sum into int32 (exact for -128 too) */
    __m256i lo = _mm256_madd_epi16(_mm256_cvtepi8_epi16(_mm256_castsi256_si128(a)),
                                   _mm256_cvtepi8_epi16(_mm256_castsi256_si128(b)));
    __m256i hi = _mm256_madd_epi16(_mm256_cvtepi8_epi16(_mm256_extracti128_si256(a, 1)),
                                   _mm256_cvtepi8_epi16(_mm256_extracti128_si256(b, 1)));
    *s = hsum_i32(_mm256_add_epi32(lo, hi));
    return 0;
}

/* Q8_0 quantizer with the x86 AVX2 semantics (d = amax/127 as fp16,
 * q = round-half-even(x * (127/amax))), vectorized 8 lanes at a time. */
void oq_avx2_quantize_row_q8_0(const float *x, oq_block_q8_0 *y, int64_t k) {
    const __m256 absmask = _mm256_castsi256_ps(_mm256_set1_epi32(0x7fffffff));
    for (int64_t i = 0; i < k / OQ_QK8_0; i++, x += OQ_QK8_0) {
        __m256 v[4], m = _mm256_setzero_ps();
        for (int r = 0; r < 4; r++) {
            v[r] = _mm256_loadu_ps(x + 8 * r);
            m = _mm256_max_ps(m, _mm256_and_ps(v[r], absmask));
        }
        __m128 m4 = _mm_max_ps(_mm256_castps256_ps128(m), _mm256_extractf128_ps(m, 1));
        m4 = _mm_max_ps(m4, _mm_movehl_ps(m4, m4));
        m4 = _mm_max_ss(m4, _mm_movehdup_ps(m4));
        const float amax = _mm_cvtss_f32(m4);
        y[i].d = oq_fp32_to_fp16(amax / 127.0f);
        const __m256 mul = _mm256_set1_ps(amax != 0.0f ? 127.0f / amax : 0.0f);
        int32_t q[32];
        for (int r = 0; r < 4; r++) {
            __m256 p = _mm256_round_ps(_mm256_mul_ps(v[r], mul), _MM_FROUND_TO_NEAREST_INT | _MM_FROUND_NO_EXC);
            _mm256_storeu_si256((__m256i *)(q + 8 * r), _mm256_cvtps_epi32(p));
        }
        for (int j = 0; j < 32; j++) y[i].qs[j] = (int8_t)q[j];
    }
}
