// act_prep.cuh — produce the quantized activation image the decode GEMV reads.
//
// The row GEMV (gemv_row.cuh) pulls its activations into shared memory with
// one bulk copy of this image:
//   qs  [m][K]        int8 Q8_K quants, natural element order
//   d   [m][nbk]      f32 Q8_K scales (padded to 16 bytes)
//   bs  [m][nbk][16]  32-element sums split into low bytes (0-7) and high
//                     bytes (8-15), the operands of the min-term dp4a
// (row_act_bytes() gives the size, a multiple of 128).
//
// One warp per (token, 256-block), all blocks in one round across the GPU.
// The input transform before quantization is one of the fused prologues of
// codpiece's layer (qwen35.rs:2534-2537, 2777-2783):
//   PLAIN   v = x
//   RMS     v = rms_norm(x + r) * g   (r, g optional; x + r is also written
//                                      out when h_out is given: the residual add)
//   SWIGLU  v = silu(x) * r           (x = gate, r = up)
// rms_norm follows ggml-cpu: sum of (x*x rounded to fp32) in double,
// mean = sum/K as fp32, scale = 1/sqrt(mean + eps). Every CTA of a row
// recomputes the row's sum itself (the row is a few KB), so no second pass
// or grid-wide reduction is needed.
#pragma once

#include "q8k_block.cuh"

namespace cpq {

enum ActMode : int { kActPlain = 0, kActRms = 1, kActSwiglu = 2 };

__host__ __device__ constexpr int row_act_bytes(int64_t k, int m) {
    return int(align_up(align_up(size_t(m) * size_t(k), 16) + align_up(size_t(m) * size_t(k / kQK_K) * 4, 16) +
                            size_t(m) * size_t(k / kQK_K) * 16,
                        128));
}

struct ActPrepArgs {
    int mode;
    const float *x;    // [m][x_stride]
    const float *r;    // residual (RMS) or up (SWIGLU); may be null for RMS
    const float *g;    // RMS weight or null
    float *h_out;      // RMS: x + r written here when non-null (must not alias x or r)
    int64_t x_stride;  // floats between rows of x, r and h_out
    int64_t k;
    int m;
    float eps;
    uint8_t *out;      // the image (row_act_bytes(k, m) bytes)
    ArIn ar;           // RMS: r = the all-reduced residual of this channel (r must be null)
    // the fragment-order image of the int8-MMA GEMV instead (act_prep_kernel<false, true>):
    // quants [nbk][mp][4][8][8], split 32-sums [nbk][mp][16], scales [nbk][mp]; tokens m..mp-1 zero
    int8_t *fq;
    uint8_t *fb;
    float *fd;
    int mp;
};

template <bool L2>
__device__ __forceinline__ float4 act_ld4(const float *p) {
    return L2 ? __ldcg(reinterpret_cast<const float4 *>(p)) : *reinterpret_cast<const float4 *>(p);
}

// This lane's 8 elements of block b before scaling: x (PLAIN), x + r (RMS;
// x when r is null) or silu(x) * r (SWIGLU). With ar (RMS), r is the sum of
// the ranks' partial rows in rank order (the fused allreduce). L2: read
// through L2 only (the inputs were written by other SMs in the same launch).
template <bool L2>
__device__ __forceinline__ void act_load_v(int mode, const float *xr, const float *rr, int b, float (&v)[8],
                                           const ArRows *ar = nullptr) {
    const int lane = threadIdx.x & 31;
    const int64_t e0 = int64_t(b) * kQK_K + lane * 8;
    const float4 x0 = act_ld4<L2>(xr + e0), x1 = act_ld4<L2>(xr + e0 + 4);
    v[0] = x0.x; v[1] = x0.y; v[2] = x0.z; v[3] = x0.w;
    v[4] = x1.x; v[5] = x1.y; v[6] = x1.z; v[7] = x1.w;
    if (mode == kActRms) {
        if (ar) {
            float rv[8];
            ar_sum8(ar->p0 + e0, ar->stride, ar->n, ar->seq, rv);
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = __fadd_rn(v[e], rv[e]);
        } else if (rr) {
            const float4 r0 = act_ld4<L2>(rr + e0), r1 = act_ld4<L2>(rr + e0 + 4);
            const float rv[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = __fadd_rn(v[e], rv[e]);
        }
    } else if (mode == kActSwiglu) {
        const float4 u0 = act_ld4<L2>(rr + e0), u1 = act_ld4<L2>(rr + e0 + 4);
        const float uv[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const float s = __fdiv_rn(v[e], __fadd_rn(1.0f, expf(-v[e])));
            v[e] = __fmul_rn(s, uv[e]);
        }
    }
}

// Block b of token row t from its loaded values v: RMS scaling (and weight
// g), the Q8_K quantizer, and the three parts of the activation image of m
// rows (layout above). One warp.
__device__ __forceinline__ void act_scale(int mode, float (&v)[8], float scale, const float *g, int b) {
    if (mode != kActRms) return;
    const int64_t e0 = int64_t(b) * kQK_K + (threadIdx.x & 31) * 8;
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = __fmul_rn(v[e], scale);
    if (g) {
#pragma unroll
        for (int e = 0; e < 8; e++) v[e] = __fmul_rn(v[e], g[e0 + e]);
    }
}

__device__ __forceinline__ void act_quantize_store(int mode, float (&v)[8], float scale, const float *g, int b, int t,
                                                   int64_t k, int m, uint8_t *img) {
    const int lane = threadIdx.x & 31;
    const int nbk = int(k / kQK_K);
    const int64_t e0 = int64_t(b) * kQK_K + lane * 8;
    act_scale(mode, v, scale, g, b);
    int q[8];
    const float d = q8k_quantize_block(v, lane, q);
    uint32_t lo, hi;
    pack8(q, lo, hi);
    uint8_t *qs = img;
    float *dd = reinterpret_cast<float *>(img + align_up(size_t(m) * size_t(k), 16));
    uint8_t *bs = reinterpret_cast<uint8_t *>(dd) + align_up(size_t(m) * nbk * 4, 16);
    *reinterpret_cast<uint2 *>(qs + t * k + e0) = make_uint2(lo, hi);
    int s8 = 0;
#pragma unroll
    for (int e = 0; e < 8; e++) s8 += q[e];
    int s32 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
    s32 += __shfl_xor_sync(0xffffffffu, s32, 2);
    if ((lane & 3) == 0) {
        uint8_t *bb = bs + (size_t(t) * nbk + b) * 16;
        bb[lane >> 2] = uint8_t(s32 & 0xff);
        bb[8 + (lane >> 2)] = uint8_t(int8_t(s32 >> 8));
    }
    if (lane == 0) dd[t * nbk + b] = d;
}

// The same for the fragment-order image (ActPrepArgs::fq/fb/fd): lane l's
// elements 8l..8l+7 are sub-block l/4 at position 8(l%4), stored at
// [b][t][l%4][l/4][8]; the 32-sum of sub-block s as its low byte at 16bt + s
// and its high byte at 16bt + 8 + s; d at bt (bt = b * mp + t).
__device__ __forceinline__ void act_quantize_store_frag(int mode, float (&v)[8], float scale, const float *g, int b,
                                                        int t, const ActPrepArgs &a) {
    const int lane = threadIdx.x & 31;
    act_scale(mode, v, scale, g, b);
    int q[8];
    const float d = q8k_quantize_block(v, lane, q);
    uint32_t lo, hi;
    pack8(q, lo, hi);
    const size_t bt = size_t(b) * a.mp + t;
    *reinterpret_cast<uint2 *>(a.fq + bt * kQK_K + (lane & 3) * 64 + (lane >> 2) * 8) = make_uint2(lo, hi);
    int s8 = 0;
#pragma unroll
    for (int e = 0; e < 8; e++) s8 += q[e];
    int s32 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
    s32 += __shfl_xor_sync(0xffffffffu, s32, 2);
    if ((lane & 3) == 0) {
        a.fb[bt * 16 + (lane >> 2)] = uint8_t(s32 & 0xff);
        a.fb[bt * 16 + 8 + (lane >> 2)] = uint8_t(int8_t(s32 >> 8));
    }
    if (lane == 0) a.fd[bt] = d;
}

__device__ __forceinline__ void store8(float *p, const float (&v)[8]) {
    *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4 *>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// Blocks a warp handles when a CTA of 8 warps covers a whole row: w, w+8, ...
constexpr int kActBatch = 5;  // blocks whose loads are in flight together

// RMS scale of one token row, 1/sqrt(mean((x + r)^2) + eps) with ggml-cpu's
// arithmetic (fp32 squares summed in double), computed by a whole CTA of 256
// threads. Summation order (fixed, so every caller gets the same bits):
// lane l of warp w adds, for its blocks b = w, w+8, ... in turn, elements
// 8l..8l+7 of b; then a butterfly over the warp; then warps 0..7 in order.
// `part` is 8 doubles of shared scratch. When every warp has at most
// kActBatch blocks, their values are left in vk (block j of the warp in
// vk[j]) and the function returns true.
template <bool L2>
__device__ __forceinline__ bool act_rms_row(const float *xr, const float *rr, int64_t k, float eps, double *part,
                                            float &scale, float (&vk)[kActBatch][8], const ArRows *ar = nullptr) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nbk = int(k / kQK_K);
    const int nbw = nbk > warp ? (nbk - warp + 7) / 8 : 0;
    double s = 0.0;
    for (int j0 = 0; j0 < nbw; j0 += kActBatch) {
#pragma unroll
        for (int jj = 0; jj < kActBatch; jj++)
            if (j0 + jj < nbw) act_load_v<L2>(kActRms, xr, rr, warp + 8 * (j0 + jj), vk[jj], ar);
#pragma unroll
        for (int jj = 0; jj < kActBatch; jj++)
            if (j0 + jj < nbw) {
#pragma unroll
                for (int e = 0; e < 8; e++) s += double(__fmul_rn(vk[jj][e], vk[jj][e]));
            }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    __syncthreads();  // part may still be read by a previous call
    if (lane == 0) part[warp] = s;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < 8; w++) tot += part[w];
    const float mean = float(tot / double(k));
    scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    return (nbk + 7) / 8 <= kActBatch;
}

// grid: (ceil(nbk / 8), m); block 256 = 8 warps, warp w quantizes block 8*blockIdx.x + w of token blockIdx.y
// AR: the input's residual comes from an all-reduce channel (a.ar); the
// instance without it carries none of that code. Both stay small enough
// (256 threads x at most 104 registers) to share an SM with a row-GEMV CTA
// while they wait under programmatic dependent launch.
// FRAG: the fragment-order image of the int8-MMA GEMV (verify, M = 4..16);
// grid (ceil(nbk / 8), mp), the CTAs of tokens m..mp-1 store zero blocks.
#ifndef CPQ_ACT_AR_MAXNREG
#define CPQ_ACT_AR_MAXNREG 104
#endif
template <bool AR, bool FRAG = false>
__global__ void __launch_bounds__(256, 1) __maxnreg__(AR ? CPQ_ACT_AR_MAXNREG : 104) act_prep_kernel(const ActPrepArgs a) {
    static_assert(!(AR && FRAG), "the fragment image is built without the all-reduce input");
    // Dependents (the row GEMV) may launch before this kernel even starts
    // waiting: they only prefetch weights until their own griddepcontrol.wait,
    // which still orders them after this kernel, and so they take each SM as
    // soon as the GEMV before this kernel leaves it.
    pdl_launch_dependents();
    pdl_wait();
    __shared__ double part[8];
    __shared__ unsigned ar_seq;
    const int warp = threadIdx.x >> 5;
    const int t = blockIdx.y;
    const int nbk = int(a.k / kQK_K);
    if (FRAG && t >= a.m) {  // padding token (uniform over the CTA: no barrier is skipped by part of it)
        const int bz = blockIdx.x * 8 + warp;
        if (bz < nbk) {
            float z[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
            act_quantize_store_frag(kActPlain, z, 1.0f, nullptr, bz, t, a);
        }
        return;
    }
    const float *xr = a.x + t * a.x_stride;
    const float *rr = a.r ? a.r + t * a.x_stride : nullptr;
    ArRows rows;
    const ArRows *arp = nullptr;
    unsigned ticket = 0;
    if (AR) {
        // r = the sum over ranks of the all-reduced output (LL words, waited for one by one)
        if (threadIdx.x == 0) ar_seq = ar_consumer_begin(a.ar, ticket);
        __syncthreads();
        const int par = int(ar_seq % kArSlots);
        rows.n = a.ar.world;
        rows.seq = ar_seq;
        rows.p0 = a.ar.base + int64_t(par) * a.ar.world * a.ar.n_max + int64_t(t) * a.ar.n;
        rows.stride = a.ar.n_max;
        arp = &rows;
    }
    float scale = 1.0f;
    float vk[kActBatch][8];
    bool have = false;
    if (a.mode == kActRms) have = act_rms_row<false>(xr, rr, a.k, a.eps, part, scale, vk, arp);
    const int b = blockIdx.x * 8 + warp;
    if (b >= nbk) return;
    float v[8];
    if (have) {  // block b is this warp's block number blockIdx.x of the row pass: reuse its values
#pragma unroll
        for (int jj = 0; jj < kActBatch; jj++)
            if (jj == int(blockIdx.x)) {
#pragma unroll
                for (int e = 0; e < 8; e++) v[e] = vk[jj][e];
            }
    } else {
        act_load_v<false>(a.mode, xr, rr, b, v, arp);
    }
    if (a.mode == kActRms && (rr || arp) && a.h_out)
        store8(a.h_out + t * a.x_stride + int64_t(b) * kQK_K + (threadIdx.x & 31) * 8, v);
    if (FRAG) act_quantize_store_frag(a.mode, v, scale, a.g, b, t, a);
    else act_quantize_store(a.mode, v, scale, a.g, b, t, a.k, a.m, a.out);
    if (AR && threadIdx.x == 0) ar_consumer_end(a.ar, ticket, ar_seq);  // thread 0's block is always < nbk
}

}  // namespace cpq
