// elementwise.cuh — the small ops around the projections of a decode layer:
// rms norm (qwen35.rs:2534-2537, ggml_rms_norm + ggml_mul), SwiGLU
// (qwen35.rs:2781, ggml_silu + ggml_mul), residual add (qwen35.rs:2777, 2783)
// and the greedy argmax after the LM head (qwen35.rs:2800-2818).
#pragma once

#include "common.cuh"

namespace cpq {

// ggml-cpu rms_norm: sum of x*x (each product rounded to fp32, summed in
// double), mean = sum/k as fp32, scale = 1/sqrt(mean + eps), y = x*scale;
// then the weight multiply of rms(). One CTA per row.
__global__ void __launch_bounds__(256) rms_norm_kernel(const float *__restrict__ x, const float *__restrict__ g,
                                                       float *__restrict__ out, int64_t k, float eps) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ double part[8];
    const int64_t row = blockIdx.x;
    const float *xr = x + row * k;
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
        const float v = xr[i];
        s += double(__fmul_rn(v, v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    double tot = 0.0;
    for (int w = 0; w < int(blockDim.x >> 5); w++) tot += part[w];
    const float mean = float(tot / double(k));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    float *orow = out + row * k;
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
        const float v = __fmul_rn(xr[i], scale);
        orow[i] = g ? __fmul_rn(v, g[i]) : v;
    }
}

// The fp32 form of the fused prologues (act_prep.cuh) for paths that
// quantize separately: RMS  out = rms_norm(x + r) * g  (h_out = x + r when
// given);  SWIGLU  out = silu(x) * r. One CTA per row; out is [m][k] dense.
__global__ void __launch_bounds__(256) prologue_f32_kernel(int mode, const float *__restrict__ x,
                                                           const float *__restrict__ r, const float *__restrict__ g,
                                                           float *__restrict__ h_out, int64_t x_stride, int64_t k,
                                                           float eps, float *__restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t row = blockIdx.x;
    const float *xr = x + row * x_stride;
    const float *rr = r ? r + row * x_stride : nullptr;
    float *orow = out + row * k;
    if (mode == 2) {  // SWIGLU
        for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
            const float gv = xr[i];
            const float s = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
            orow[i] = __fmul_rn(s, rr[i]);
        }
        return;
    }
    __shared__ double part[8];
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
        const float v = rr ? __fadd_rn(xr[i], rr[i]) : xr[i];
        if (h_out) h_out[row * x_stride + i] = v;
        s += double(__fmul_rn(v, v));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    double tot = 0.0;
    for (int w = 0; w < int(blockDim.x >> 5); w++) tot += part[w];
    const float mean = float(tot / double(k));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
        const float v0 = rr ? __fadd_rn(xr[i], rr[i]) : xr[i];
        const float v = __fmul_rn(v0, scale);
        orow[i] = g ? __fmul_rn(v, g[i]) : v;
    }
}

// The RMS prologue for rows of k <= kRmsFastMaxK (k % 4 == 0, 16-byte aligned
// rows): one CTA of 512 threads per row, every load of the row issued at once
// and kept in registers (thread t holds float4s t, t + 512, ...), so the row
// costs one memory round trip instead of one per loop step. Same arithmetic
// as prologue_f32_kernel (fp32 add and square, double sum, fp32 scale),
// summed per thread, then per warp, then over warps in order.
constexpr int kRmsFastThreads = 512, kRmsFastVec = 8;
constexpr int64_t kRmsFastMaxK = int64_t(kRmsFastThreads) * kRmsFastVec * 4;
__global__ void __launch_bounds__(kRmsFastThreads) prologue_rms_fast_kernel(
    const float *__restrict__ x, const float *__restrict__ r, const float *__restrict__ g, float *__restrict__ h_out,
    int64_t x_stride, int64_t k, float eps, float *__restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    const int64_t row = blockIdx.x;
    const int64_t n4 = k / 4;
    const float4 *xr = reinterpret_cast<const float4 *>(x + row * x_stride);
    const float4 *rr = r ? reinterpret_cast<const float4 *>(r + row * x_stride) : nullptr;
    float4 v[kRmsFastVec];
#pragma unroll
    for (int u = 0; u < kRmsFastVec; u++) {
        const int64_t i = threadIdx.x + int64_t(u) * kRmsFastThreads;
        v[u] = i < n4 ? xr[i] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (rr && i < n4) {
            const float4 b = rr[i];
            v[u] = make_float4(__fadd_rn(v[u].x, b.x), __fadd_rn(v[u].y, b.y), __fadd_rn(v[u].z, b.z),
                               __fadd_rn(v[u].w, b.w));
        }
    }
    double s = 0.0;
#pragma unroll
    for (int u = 0; u < kRmsFastVec; u++) {
        const int64_t i = threadIdx.x + int64_t(u) * kRmsFastThreads;
        if (i < n4) {
            if (h_out) reinterpret_cast<float4 *>(h_out + row * x_stride)[i] = v[u];
            s += double(__fmul_rn(v[u].x, v[u].x));
            s += double(__fmul_rn(v[u].y, v[u].y));
            s += double(__fmul_rn(v[u].z, v[u].z));
            s += double(__fmul_rn(v[u].w, v[u].w));
        }
    }
    __shared__ double part[kRmsFastThreads / 32];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    double tot = 0.0;
#pragma unroll
    for (int w = 0; w < kRmsFastThreads / 32; w++) tot += part[w];
    const float mean = float(tot / double(k));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, eps)));
    float4 *orow = reinterpret_cast<float4 *>(out + row * k);
    const float4 *g4 = reinterpret_cast<const float4 *>(g);
#pragma unroll
    for (int u = 0; u < kRmsFastVec; u++) {
        const int64_t i = threadIdx.x + int64_t(u) * kRmsFastThreads;
        if (i < n4) {
            float4 o = make_float4(__fmul_rn(v[u].x, scale), __fmul_rn(v[u].y, scale), __fmul_rn(v[u].z, scale),
                                   __fmul_rn(v[u].w, scale));
            if (g) {
                const float4 gg = g4[i];
                o = make_float4(__fmul_rn(o.x, gg.x), __fmul_rn(o.y, gg.y), __fmul_rn(o.z, gg.z), __fmul_rn(o.w, gg.w));
            }
            orow[i] = o;
        }
    }
}

// ggml silu(x) = x / (1 + exp(-x)); act = silu(gate) * up.
__global__ void swiglu_kernel(const float *__restrict__ gate, const float *__restrict__ up, float *__restrict__ act,
                              int64_t n) {
    pdl_wait();
    pdl_launch_dependents();
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const float gv = gate[i];
        const float s = __fdiv_rn(gv, __fadd_rn(1.0f, expf(-gv)));
        act[i] = __fmul_rn(s, up[i]);
    }
}

__global__ void add_inplace_kernel(float *__restrict__ y, const float *__restrict__ x, int64_t n) {
    pdl_wait();
    pdl_launch_dependents();
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x)
        y[i] = __fadd_rn(y[i], x[i]);
}

// First index of the maximum of each row (NaN-free input assumed). Grid
// (nchunk, m): each CTA reduces one chunk of a row to (max, first index),
// publishes it, and the last CTA of the row (counter, acq_rel) reduces the
// chunk results in chunk order and resets the counter for the next call.
__device__ __forceinline__ void argmax_merge(float &best, int32_t &bi, float ov, int32_t oi) {
    if (ov > best || (ov == best && oi < bi)) {
        best = ov;
        bi = oi;
    }
}

__global__ void __launch_bounds__(256) argmax_kernel(const float *__restrict__ x, int64_t n, int64_t chunk,
                                                    float *__restrict__ pval, int32_t *__restrict__ pidx,
                                                    int *__restrict__ counters, int32_t *__restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ float sv[8];
    __shared__ int32_t si[8];
    __shared__ int last;
    const int64_t row = blockIdx.y;
    const int nchunk = gridDim.x;
    const float *xr = x + row * n;
    const int64_t lo = int64_t(blockIdx.x) * chunk, hi = min(n, lo + chunk);
    float best = -INFINITY;
    int32_t bi = 0x7fffffff;
    for (int64_t i = lo + threadIdx.x; i < hi; i += 256) argmax_merge(best, bi, xr[i], int32_t(i));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        argmax_merge(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = best;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < 8; w++) argmax_merge(best, bi, sv[w], si[w]);
        pval[row * nchunk + blockIdx.x] = best;
        pidx[row * nchunk + blockIdx.x] = bi;
        int old;
        asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(old) : "l"(counters + row) : "memory");
        last = (old == nchunk - 1);
    }
    __syncthreads();
    if (!last) return;
    if (threadIdx.x == 0) {
        float b = -INFINITY;
        int32_t ix = 0x7fffffff;
        for (int c = 0; c < nchunk; c++) argmax_merge(b, ix, __ldcg(pval + row * nchunk + c), __ldcg(pidx + row * nchunk + c));
        out[row] = ix == 0x7fffffff ? 0 : ix;
        counters[row] = 0;
    }
}

// out = x + sum over ranks of the channel's last all-reduced value (rank
// order, the same additions as act_load_v). grid: (ceil(k / 2048), m), 256
// threads x 8 elements.
__global__ void __launch_bounds__(256, 1) ar_add_kernel(const ArIn ar, const float *__restrict__ x,
                                                     float *__restrict__ out, int64_t k) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ unsigned seq;
    unsigned ticket = 0;
    if (threadIdx.x == 0) seq = ar_consumer_begin(ar, ticket);
    __syncthreads();
    const int t = blockIdx.y;
    const int64_t e0 = (int64_t(blockIdx.x) * 256 + threadIdx.x) * 8;
    if (e0 >= k) return;
    const uint64_t *base = ar.base + int64_t(seq % kArSlots) * ar.world * ar.n_max + int64_t(t) * ar.n + e0;
    float v[8];
    ar_sum8(base, ar.n_max, ar.world, seq, v);
    const float4 x0 = *reinterpret_cast<const float4 *>(x + int64_t(t) * k + e0);
    const float4 x1 = *reinterpret_cast<const float4 *>(x + int64_t(t) * k + e0 + 4);
    const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int e = 0; e < 8; e++) v[e] = __fadd_rn(xv[e], v[e]);
    float *o = out + int64_t(t) * k + e0;
    *reinterpret_cast<float4 *>(o) = make_float4(v[0], v[1], v[2], v[3]);
    *reinterpret_cast<float4 *>(o + 4) = make_float4(v[4], v[5], v[6], v[7]);
    if (threadIdx.x == 0) ar_consumer_end(ar, ticket, seq);  // thread 0's e0 is always < k
}

// Greedy token over a vocabulary split across ranks (the LM head's N split):
// each CTA takes one token row, reduces this rank's logits [n] to (max, first
// index), publishes it as two LL words (value bits, row0 + index) to every
// rank's buffer (the producer side of the channel), then reads every rank's
// pair and keeps the largest value, the lowest global index on ties (the
// argmax of the unsplit row). grid m, 1024 threads.
__global__ void __launch_bounds__(1024) ar_argmax_kernel(const ArIn in, const ArOut out, const float *__restrict__ x,
                                                        int64_t n, int64_t ld, int64_t row0, int32_t *__restrict__ res) {
    pdl_wait();
    pdl_launch_dependents();
    __shared__ unsigned seq;
    __shared__ float sv[32];
    __shared__ int32_t si[32];
    unsigned ticket = 0;
    if (threadIdx.x == 0) seq = ar_consumer_begin(in, ticket);  // = the producers' sequence number
    const int t = blockIdx.x;
    const float *xr = x + int64_t(t) * ld;
    float best = -INFINITY;
    int32_t bi = 0x7fffffff;
    for (int64_t i = threadIdx.x; i < n; i += blockDim.x) argmax_merge(best, bi, xr[i], int32_t(i));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
        argmax_merge(best, bi, __shfl_xor_sync(0xffffffffu, best, o), __shfl_xor_sync(0xffffffffu, bi, o));
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = best;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x != 0) return;
    for (int w = 1; w < int(blockDim.x >> 5); w++) argmax_merge(best, bi, sv[w], si[w]);
    const unsigned e = seq;
    const int64_t slot = int64_t(e % kArSlots) * out.world;
    const uint64_t wv = (uint64_t(e) << 32) | __float_as_uint(best);
    const uint64_t wi = (uint64_t(e) << 32) | uint32_t(int32_t(row0) + (bi == 0x7fffffff ? 0 : bi));
    for (int d = 0; d < out.world; d++) {
        uint64_t *dst = out.peer[d] + (slot + out.rank) * out.n_max + 2 * t;
        st_relaxed_sys_u64(dst, wv);
        st_relaxed_sys_u64(dst + 1, wi);
    }
    float gb = -INFINITY;
    int32_t gi = 0x7fffffff;
    for (int r = 0; r < in.world; r++) {
        const uint64_t *src = in.base + (slot + r) * in.n_max + 2 * t;
        const float v = ar_word(src, e);
        const int32_t ix = int32_t(__float_as_uint(ar_word(src + 1, e)));
        argmax_merge(gb, gi, v, ix);
    }
    res[t] = gi == 0x7fffffff ? 0 : gi;
    ar_consumer_end(in, ticket, seq);
}

// A zero contribution to the next all-reduce (this rank's slot of every
// rank's buffer): the producer side of row_block_out with all values 0.
__global__ void __launch_bounds__(256) ar_zero_kernel(const ArOut ar, int64_t total) {
    pdl_wait();
    pdl_launch_dependents();
    const unsigned e = *ar.seq + 1u;
    const int64_t slot = (int64_t(e % kArSlots) * ar.world + ar.rank) * ar.n_max;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x)
        for (int d = 0; d < ar.world; d++) st_relaxed_sys_u64(ar.peer[d] + slot + i, uint64_t(e) << 32);
}

}  // namespace cpq
