// quantize.cuh — activation re-quantization kernels (fp32 -> Q8_K / Q8_0).
//
// ggml-cpu quantizes every src1 row to the weight's vec_dot_type before its
// integer dots. These kernels reproduce those quantizers bit for bit:
//
// Q8_K (ggml quantize_row_q8_K_ref, used unchanged by x86 ggml-cpu): per
//   256-block, `max` is the element of largest magnitude (first on ties),
//   iscale = -127/max, q = min(127, round-half-even(iscale*x)), d = 1/iscale,
//   bsums = sums of 16 quants. An all-zero block gives d = 0, q = 0, bsums = 0.
// Q8_0 (ggml-cpu x86 AVX2 quantize_row_q8_0, the reference's build,
//   codpiece-ggml-sys/build.rs:59-63): d = amax/127 stored as fp16,
//   q = round-half-even(x * (127/amax)), 0 when amax = 0.
//
// Every product, quotient and rounding is spelled with an _rn intrinsic so no
// FMA contraction or fast-math can change a bit.
#pragma once

#include "common.cuh"

namespace cpq {

// One warp per 256-element block; lane l owns elements 8l..8l+7.
// soa_* may be null (AoS only); aos may be null (SoA only).
__global__ void __launch_bounds__(256) quantize_q8K_kernel(const float *__restrict__ x, int64_t k, int64_t m,
                                                           int64_t x_stride, int8_t *__restrict__ soa_qs,
                                                           float *__restrict__ soa_d,
                                                           int16_t *__restrict__ soa_bs, uint8_t *__restrict__ aos) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t nb = k / kQK_K;
    const int64_t total = m * nb;
    const int64_t nwarps = int64_t(gridDim.x) * (blockDim.x >> 5);
    for (int64_t blk = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; blk < total; blk += nwarps) {
        const int64_t row = blk / nb, b = blk - row * nb;
        const float *xb = x + row * x_stride + b * kQK_K + lane * 8;
        const float4 v0 = *reinterpret_cast<const float4 *>(xb);
        const float4 v1 = *reinterpret_cast<const float4 *>(xb + 4);
        const float v[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};

        float amax = 0.0f, mx = 0.0f;
        int idx = 0x7fffffff;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            const float ax = fabsf(v[e]);
            if (ax > amax) {
                amax = ax;
                mx = v[e];
                idx = lane * 8 + e;
            }
        }
        // largest magnitude, first index on ties: same pick as the sequential scan
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float oa = __shfl_xor_sync(0xffffffffu, amax, o);
            const float om = __shfl_xor_sync(0xffffffffu, mx, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (oa > amax || (oa == amax && oi < idx)) {
                amax = oa;
                mx = om;
                idx = oi;
            }
        }

        int q[8];
        float d = 0.0f;
        if (amax == 0.0f) {
#pragma unroll
            for (int e = 0; e < 8; e++) q[e] = 0;
        } else {
            const float iscale = __fdiv_rn(-127.0f, mx);
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const int t = __float2int_rn(__fmul_rn(iscale, v[e]));
                q[e] = t < 127 ? t : 127;
            }
            d = __fdiv_rn(1.0f, iscale);
        }
        uint32_t lo = 0, hi = 0;
        int s8 = 0;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            lo |= (uint32_t(q[e]) & 0xffu) << (8 * e);
            hi |= (uint32_t(q[e + 4]) & 0xffu) << (8 * e);
        }
#pragma unroll
        for (int e = 0; e < 8; e++) s8 += q[e];
        const int s16 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);

        if (soa_qs) {
            *reinterpret_cast<uint2 *>(soa_qs + row * k + b * kQK_K + lane * 8) = make_uint2(lo, hi);
            if (lane == 0) soa_d[row * nb + b] = d;
            if ((lane & 1) == 0) soa_bs[row * (k / 16) + b * 16 + (lane >> 1)] = int16_t(s16);
        }
        if (aos) {
            uint8_t *ob = aos + (row * nb + b) * kQ8K_Bytes;
            if (lane == 0) *reinterpret_cast<float *>(ob) = d;
            uint32_t *oq = reinterpret_cast<uint32_t *>(ob + 4 + lane * 8);
            oq[0] = lo;
            oq[1] = hi;
            if ((lane & 1) == 0) reinterpret_cast<int16_t *>(ob + 4 + kQK_K)[lane >> 1] = int16_t(s16);
        }
    }
}

// Four lanes per 32-element block (8 elements each); 8 blocks per warp.
__global__ void __launch_bounds__(256) quantize_q8_0_kernel(const float *__restrict__ x, int64_t k, int64_t m,
                                                            int64_t x_stride, int8_t *__restrict__ soa_qs,
                                                            float *__restrict__ soa_d, uint8_t *__restrict__ aos) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int sub = lane & 3;
    const int64_t nb = k / kQK8_0;
    const int64_t total = m * nb;
    const int64_t nthreads = int64_t(gridDim.x) * blockDim.x;
    // a group of 4 lanes handles one block; iterate whole warps so shuffles stay converged
    const int64_t groups_per_iter = nthreads / 4;
    const int64_t first = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) / 4;
    for (int64_t base = first - (lane >> 2); base < total; base += groups_per_iter) {
        const int64_t blk = base + (lane >> 2);
        const bool valid = blk < total;
        float v[8];
        int64_t row = 0, b = 0;
        if (valid) {
            row = blk / nb;
            b = blk - row * nb;
            const float *xb = x + row * x_stride + b * kQK8_0 + sub * 8;
            const float4 v0 = *reinterpret_cast<const float4 *>(xb);
            const float4 v1 = *reinterpret_cast<const float4 *>(xb + 4);
            v[0] = v0.x; v[1] = v0.y; v[2] = v0.z; v[3] = v0.w;
            v[4] = v1.x; v[5] = v1.y; v[6] = v1.z; v[7] = v1.w;
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = 0.0f;
        }
        float amax = 0.0f;
#pragma unroll
        for (int e = 0; e < 8; e++) amax = fmaxf(amax, fabsf(v[e]));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        if (!valid) continue;
        const __half hd = __float2half_rn(__fdiv_rn(amax, 127.0f));
        const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        uint32_t lo = 0, hi = 0;
#pragma unroll
        for (int e = 0; e < 8; e++) {
            int t = __float2int_rn(__fmul_rn(v[e], id));
            t = t < -128 ? -128 : (t > 127 ? 127 : t);
            if (e < 4) lo |= (uint32_t(t) & 0xffu) << (8 * e);
            else hi |= (uint32_t(t) & 0xffu) << (8 * (e - 4));
        }
        if (soa_qs) {
            *reinterpret_cast<uint2 *>(soa_qs + row * k + b * kQK8_0 + sub * 8) = make_uint2(lo, hi);
            if (sub == 0) soa_d[row * nb + b] = __half2float(hd);
        }
        if (aos) {
            uint8_t *ob = aos + (row * nb + b) * kQ8_0_Bytes;
            if (sub == 0) *reinterpret_cast<__half *>(ob) = hd;
            uint16_t *oq = reinterpret_cast<uint16_t *>(ob + 2 + sub * 8);
            oq[0] = uint16_t(lo & 0xffffu);
            oq[1] = uint16_t(lo >> 16);
            oq[2] = uint16_t(hi & 0xffffu);
            oq[3] = uint16_t(hi >> 16);
        }
    }
}

}  // namespace cpq
