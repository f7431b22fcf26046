// synth.cuh — seeded synthetic quantized weights, generated on the device.
//
// The benchmark configs fix value distributions, not files: fp16 scales
// |N(0, 0.01)| (Q4_K d and dmin, Q6_K d) or |N(0, 0.02)|/127 (Q8_0 d),
// uniform six-bit Q4_K scales/mins, uniform quant bits, uniform int8 Q6_K
// scales, Q8_0 quants uniform in [-127, 127]. Every byte is a pure function of
// (seed, global row, global block, position), so a tensor-parallel shard
// generated on its own device equals the same slice of the whole tensor.
#pragma once

#include "common.cuh"

namespace cpq {

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    // splitmix64 finalizer (Steele, Lea, Flood: "Fast splittable PRNGs", 2014)
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t synth_hash(uint64_t seed, int64_t row, int64_t blk, uint32_t slot) {
    uint64_t h = mix64(seed + 0x9e3779b97f4a7c15ull);
    h = mix64(h ^ uint64_t(row) * 0xd1b54a32d192ed03ull);
    h = mix64(h ^ uint64_t(blk) * 0x8cb92ba72f3d8dd7ull);
    return mix64(h ^ (uint64_t(slot) + 1) * 0x9e3779b97f4a7c15ull);
}

// |N(0, sigma)| by Box-Muller from one 64-bit hash.
__device__ __forceinline__ float half_normal(uint64_t h, float sigma) {
    const float u1 = float((h >> 40) + 1) * (1.0f / 16777216.0f);  // (0, 1]
    const float u2 = float(h & 0xffffffull) * (1.0f / 16777216.0f);
    return fabsf(sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2)) * sigma;
}

__device__ __forceinline__ uint16_t f16_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

// Writes one block of `type` for (row, blk) to dst (byte-addressed, any alignment).
__device__ void synth_block(int32_t type, uint64_t seed, int64_t row, int64_t blk, uint8_t *dst) {
    if (type == CPQ_TYPE_Q4_K) {
        const uint16_t d = f16_bits(half_normal(synth_hash(seed, row, blk, 0), 0.01f));
        const uint16_t dm = f16_bits(half_normal(synth_hash(seed, row, blk, 1), 0.01f));
        dst[0] = uint8_t(d);
        dst[1] = uint8_t(d >> 8);
        dst[2] = uint8_t(dm);
        dst[3] = uint8_t(dm >> 8);
        const uint64_t hs = synth_hash(seed, row, blk, 2), hm = synth_hash(seed, row, blk, 3);
        uint8_t sc[8], mn[8];
        for (int j = 0; j < 8; j++) {
            sc[j] = uint8_t((hs >> (6 * j)) & 63);
            mn[j] = uint8_t((hm >> (6 * j)) & 63);
        }
        // pack: bytes 0-3 sc[0..3] | top bits of sc[4..7]; 4-7 mn likewise; 8-11 low nibbles
        for (int j = 0; j < 4; j++) {
            dst[4 + j] = uint8_t(sc[j] | ((sc[j + 4] >> 4) << 6));
            dst[8 + j] = uint8_t(mn[j] | ((mn[j + 4] >> 4) << 6));
            dst[12 + j] = uint8_t((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
        }
        for (int w = 0; w < 16; w++) {
            const uint64_t h = synth_hash(seed, row, blk, 4 + w);
            for (int b = 0; b < 8; b++) dst[16 + 8 * w + b] = uint8_t(h >> (8 * b));
        }
    } else if (type == CPQ_TYPE_Q6_K) {
        for (int w = 0; w < 26; w++) {  // ql 128 + qh 64 + scales 16 = 208 bytes
            const uint64_t h = synth_hash(seed, row, blk, 4 + w);
            for (int b = 0; b < 8; b++) dst[8 * w + b] = uint8_t(h >> (8 * b));
        }
        const uint16_t d = f16_bits(half_normal(synth_hash(seed, row, blk, 0), 0.01f));
        dst[208] = uint8_t(d);
        dst[209] = uint8_t(d >> 8);
    } else if (type == CPQ_TYPE_Q8_0) {
        const uint16_t d = f16_bits(half_normal(synth_hash(seed, row, blk, 0), 0.02f) / 127.0f);
        dst[0] = uint8_t(d);
        dst[1] = uint8_t(d >> 8);
        for (int w = 0; w < 8; w++) {
            const uint64_t h = synth_hash(seed, row, blk, 4 + w);
            for (int b = 0; b < 4; b++) {
                const int q = int((h >> (16 * b)) & 0xffffu) % 255 - 127;
                dst[2 + 4 * w + b] = uint8_t(int8_t(q));
            }
        }
    }
}

// One CTA per row; blocks are generated into shared memory in groups of
// blockDim.x and written out with coalesced 2-byte stores (every format has
// an even block size, rows start 2-byte aligned).
__global__ void __launch_bounds__(128) synth_kernel(int32_t type, uint8_t *__restrict__ dst, int64_t n_blk,
                                                    size_t row_stride, int blk_bytes, uint64_t seed, int64_t row0,
                                                    int64_t blk0) {
    extern __shared__ __align__(16) uint8_t buf[];
    pdl_wait();  // the destination may still be read by the previous kernel
    const int64_t r = blockIdx.x;
    uint8_t *out = dst + size_t(r) * row_stride;
    for (int64_t g = 0; g < n_blk; g += blockDim.x) {
        const int cnt = int(n_blk - g < int64_t(blockDim.x) ? n_blk - g : int64_t(blockDim.x));
        if (int(threadIdx.x) < cnt) synth_block(type, seed, row0 + r, blk0 + g + threadIdx.x, buf + threadIdx.x * blk_bytes);
        __syncthreads();
        const int nh = cnt * blk_bytes / 2;
        uint16_t *o16 = reinterpret_cast<uint16_t *>(out + size_t(g) * blk_bytes);
        const uint16_t *b16 = reinterpret_cast<const uint16_t *>(buf);
        for (int i = threadIdx.x; i < nh; i += blockDim.x) o16[i] = b16[i];
        __syncthreads();
    }
}

}  // namespace cpq
