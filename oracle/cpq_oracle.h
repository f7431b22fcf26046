/*
 * cpq_oracle.h — CPU restatement of ggml-cpu's quantized mul_mat semantics.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker and the timed
 * CPU baseline ("restated ggml CPU semantics", not ggml itself). The product
 * path (codpiece_b200, libcpq.so) never links, loads or calls it; only tests/,
 * __graft_entry__.smoke() and bench.py's CPU legs do.
 *
 * What it restates. codpiece computes every projection with
 * ggml_mul_mat(ctx, W, X) (codpiece-model/src/qwen35.rs:2779-2782, 2797, 3029,
 * 3047, 3051, 3197) and executes it in ggml at llama.cpp tag b10423
 * (scripts/fetch-deps.sh:6-7). That ggml source is not vendored in the
 * reference tree, so this file restates ggml-cpu's published algorithm for an
 * F32 src1:
 *   1. every X row is re-quantized to W's vec_dot_type: Q8_K for Q4_K/Q6_K,
 *      Q8_0 for Q8_0;
 *   2. each output is the integer-block dot of one W row with one quantized X
 *      row, integer inside a superblock, fp32 across superblocks.
 * Block geometry follows codpiece-gguf/src/lib.rs:179-186 (Q8_0 32/34,
 * Q4_K 256/144, Q6_K 256/210, Q8_K 256/292) and the ggml layout convention of
 * codpiece-ggml-sys/tests/smoke.rs:29-54: W ne=[K,N], X ne=[K,M],
 * Y ne=[N,M] with Y[m*N+n] = dot(W row n, X row m).
 *
 * Parity status: dequantization of Q8_0/Q4_K/Q6_K and the portable Q8_0
 * quantizer are pinned against gguf-py 0.19.0 (llama.cpp's own Python
 * implementation of the formats) by tests/golden; Q8_K quantization and the
 * block dots are restatements with no reference golden vector available.
 */
#ifndef CPQ_ORACLE_H
#define CPQ_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type ids as serialized in GGUF (codpiece-gguf/src/lib.rs:172-205). */
enum {
    OQ_TYPE_F32 = 0,
    OQ_TYPE_F16 = 1,
    OQ_TYPE_Q8_0 = 8,
    OQ_TYPE_Q4_K = 12,
    OQ_TYPE_Q6_K = 14,
    OQ_TYPE_Q8_K = 15,
};

#define OQ_QK_K 256
#define OQ_QK8_0 32

typedef uint16_t oq_half;

typedef struct {
    oq_half d;
    int8_t qs[OQ_QK8_0];
} oq_block_q8_0; /* 34 bytes */

typedef struct {
    oq_half d;
    oq_half dmin;
    uint8_t scales[12]; /* 8 six-bit scales + 8 six-bit mins */
    uint8_t qs[OQ_QK_K / 2];
} oq_block_q4_K; /* 144 bytes */

typedef struct {
    uint8_t ql[OQ_QK_K / 2]; /* low 4 bits */
    uint8_t qh[OQ_QK_K / 4]; /* high 2 bits */
    int8_t scales[OQ_QK_K / 16];
    oq_half d;
} oq_block_q6_K; /* 210 bytes */

typedef struct {
    float d;
    int8_t qs[OQ_QK_K];
    int16_t bsums[OQ_QK_K / 16]; /* sum of each group of 16 qs */
} oq_block_q8_K; /* 292 bytes */

/* Q8_0 activation quantizer variants. The reference builds ggml-cpu with
 * GGML_AVX2=ON (codpiece-ggml-sys/build.rs:59-63), whose Q8_0 quantizer
 * multiplies by 127/amax and rounds half to even; the portable scalar
 * quantizer divides by d=amax/127 and rounds half away from zero. */
enum {
    OQ_Q8_0_X86_AVX2 = 0, /* default: what the reference binary runs */
    OQ_Q8_0_PORTABLE = 1, /* quantize_row_q8_0_ref semantics (gguf-py agrees) */
};

/* Sizes. */
size_t oq_type_block(int type);      /* elements per block, 0 if unknown */
size_t oq_type_size(int type);       /* bytes per block, 0 if unknown */
size_t oq_row_size(int type, int64_t k);

/* fp16 <-> fp32, IEEE binary16, round to nearest even. */
float oq_fp16_to_fp32(oq_half h);
oq_half oq_fp32_to_fp16(float f);

/* Activation quantizers (k must be a multiple of the block). */
void oq_quantize_row_q8_K(const float *x, oq_block_q8_K *y, int64_t k);
void oq_quantize_row_q8_0(const float *x, oq_block_q8_0 *y, int64_t k, int variant);

/* Weight dequantizers. */
void oq_dequantize_row_q8_0(const oq_block_q8_0 *x, float *y, int64_t k);
void oq_dequantize_row_q4_K(const oq_block_q4_K *x, float *y, int64_t k);
void oq_dequantize_row_q6_K(const oq_block_q6_K *x, float *y, int64_t k);

/* Block dots: integer inside a superblock/block, fp32 across. */
float oq_vec_dot_q4_K_q8_K(int64_t n, const oq_block_q4_K *x, const oq_block_q8_K *y);
float oq_vec_dot_q6_K_q8_K(int64_t n, const oq_block_q6_K *x, const oq_block_q8_K *y);
float oq_vec_dot_q8_0_q8_0(int64_t n, const oq_block_q8_0 *x, const oq_block_q8_0 *y);

/* Per-superblock integer totals (exposed for tests and the SIMD build).
 * q4_K: *sc = sum_j sc_j * sum_i q*q8, *mn = sum_g m_{g/2} * bsums[g].
 * q6_K: *sc = sum_j s_j * sum_i (q-32)*q8.  q8_0: *sc = sum_i q*q8. */
void oq_block_ints_q4_K(const oq_block_q4_K *x, const oq_block_q8_K *y, int32_t *sc, int32_t *mn);
void oq_block_ints_q6_K(const oq_block_q6_K *x, const oq_block_q8_K *y, int32_t *sc);
int32_t oq_block_int_q8_0(const oq_block_q8_0 *x, const oq_block_q8_0 *y);

/* Quantize M rows of X (fp32, row stride K) into the vec_dot_type of wtype.
 * out must hold M * oq_row_size(vec_dot_type, K) bytes. Returns 0 or -1. */
int oq_quantize_act(int wtype, const float *x, int64_t k, int64_t m, void *out, int q8_0_variant);

/* Y[m*N+n] = dot(W row n, quantize(X row m)).
 * W: N rows of row_stride bytes (>= oq_row_size(wtype, K)).
 * simd: 0 = scalar integer totals, 1 = AVX2 integer totals (identical output).
 * nthreads: OpenMP threads over output rows (<=0: library default).
 * Returns 0 on success, -1 on an unsupported type or shape. */
int oq_mul_mat(int wtype, const void *w, int64_t k, int64_t n, size_t row_stride,
               const float *x, int64_t m, float *y, int nthreads, int simd, int q8_0_variant);

/* Same, with X already quantized (xq as produced by oq_quantize_act). */
int oq_mul_mat_q(int wtype, const void *w, int64_t k, int64_t n, size_t row_stride,
                 const void *xq, int64_t m, float *y, int nthreads, int simd);

/* Plain fp32 row-dot mul_mat for F32 weights (the smoke.rs layout pin). */
void oq_mul_mat_f32(const float *w, int64_t k, int64_t n, const float *x, int64_t m, float *y);

/* ggml_gated_delta_net (ggml-cuda gated_delta_net.cu:4-167), contiguous fp32:
 * q, k [n_seqs_qk][T][H_qk][S_v]; v [n_seqs][T][H][S_v]; g [n_seqs][T][H] (or
 * [..][H][S_v] when kda); beta [n_seqs][T][H]; state [n_seqs][H][col][i].
 * attn [n_seqs][T][H][S_v]; state_out: K <= 1 the final state, else slot j
 * (j < min(K, T)) at state_out + j * slot_stride holds the state j tokens
 * before the last. In cpq_oracle_gdn.c. Returns 0 or -1. */
int oq_gated_delta_net(const float *q, const float *k, const float *v, const float *g, const float *beta,
                       const float *state, float *attn, float *state_out, int64_t sv, int64_t H, int64_t H_qk,
                       int64_t T, int64_t n_seqs, int64_t n_seqs_qk, int kda, int K, int64_t slot_stride);

/* 1 when the AVX2 build is compiled in. */
int oq_has_avx2(void);
int oq_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
