// q8k_block.cuh — the Q8_K block quantizer as a warp-level device function.
//
// ggml quantize_row_q8_K_ref (used unchanged by x86 ggml-cpu): per 256-block,
// `max` is the element of largest magnitude (first on ties),
// iscale = -127/max, q = min(127, round-half-even(iscale*x)), d = 1/iscale;
// an all-zero block gives d = 0 and zero quants. Every product, quotient and
// rounding is an _rn intrinsic so no FMA contraction can change a bit. All
// Q8_K quantizers in this library (the standalone kernels and the GEMV
// prologues) call this one function, so they agree bit for bit.
#pragma once

#include "common.cuh"

namespace cpq {

// Lane l holds elements 8l..8l+7 of the block in v; on return q holds their
// quants and the function returns d (the same value in every lane).
//
// The element of largest magnitude, first index on ties (the pick of the
// sequential scan), in two warp reductions: the largest |x| as fp32 bits
// (monotone for non-negative values), then the smallest index among the
// lanes that hold it; that lane's signed value comes back by one shuffle.
__device__ __forceinline__ float q8k_quantize_block(const float (&v)[8], int lane, int (&q)[8]) {
    float amax = 0.0f, mx = 0.0f;
    unsigned idx = 0xffffffffu;
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const float ax = fabsf(v[e]);
        if (ax > amax) {
            amax = ax;
            mx = v[e];
            idx = unsigned(lane * 8 + e);
        }
    }
    const unsigned abits = __float_as_uint(amax);
    const unsigned m = __reduce_max_sync(0xffffffffu, abits);
    if (m == 0u) {
#pragma unroll
        for (int e = 0; e < 8; e++) q[e] = 0;
        return 0.0f;
    }
    const unsigned first = __reduce_min_sync(0xffffffffu, abits == m ? idx : 0xffffffffu);
    mx = __shfl_sync(0xffffffffu, mx, int(first >> 3));
    const float iscale = __fdiv_rn(-127.0f, mx);
#pragma unroll
    for (int e = 0; e < 8; e++) {
        const int t = __float2int_rn(__fmul_rn(iscale, v[e]));
        q[e] = t < 127 ? t : 127;
    }
    return __fdiv_rn(1.0f, iscale);
}

__device__ __forceinline__ void pack8(const int (&q)[8], uint32_t &lo, uint32_t &hi) {
    lo = hi = 0;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        lo |= (uint32_t(q[e]) & 0xffu) << (8 * e);
        hi |= (uint32_t(q[e + 4]) & 0xffu) << (8 * e);
    }
}

}  // namespace cpq
