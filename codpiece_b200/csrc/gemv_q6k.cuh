// gemv_q6k.cuh — Q6_K x Q8_K small-M GEMV for whole row pairs (the LM head).
//
// Same arithmetic as ggml_vec_dot_q6_K_q8_K: for each 16-element group g of a
// superblock, the integer dot of (q6 - 32) with the Q8_K quants (computed as
// dot(q6, q8) - 32 * bsum_g), times the int8 group scale, summed exactly in
// integers over the superblock, then d_w * d_x in fp32 per superblock.
//
// Why a second Q6_K kernel. The generic dp4a GEMV (gemv.cuh) walks a row in
// 8-block chunks with per-chunk address arithmetic and reads the activations
// from global memory per token; on the head [151936 x 5120] it is issue-bound
// at M = 1 (2.5 TB/s) and load-latency-bound at M = 8 (0.6 TB/s). Here:
//   * a stage is two whole consecutive rows, 2 * K/256 * 210 bytes, which is
//     a multiple of 16 whenever K is a multiple of 1024 — one bulk copy per
//     stage (cp.async.bulk, no tensor map: a Q6_K row is not a 16-byte
//     multiple, so no 2-D tensor map can describe the matrix), one mbarrier;
//   * the Q8_K activations of all MT tokens (quants, scales, 16-sums) are
//     copied into shared memory once per CTA, so the per-token loads are
//     shared-memory loads. The quants are stored with 16-byte slot s at
//     s ^ 2*((s >> 3) & 3): the 8 lanes of a quarter warp (quarters (h, c)
//     of two consecutive superblocks) then read 8 different bank groups,
//     where the plain layout put 4 of them on each group;
//   * lane l takes the work items l, l+32, ... of a stage, an item being one
//     quarter (64 elements) of one superblock of one of the two rows; a row's
//     sum is one warp reduction per stage.
// Rows are split over the warps of the grid in contiguous ranges of row pairs.
#pragma once

#include "common.cuh"

namespace cpq {

constexpr int kQ6rWarps = 8;
constexpr int kQ6rMaxTokens = 8;
// ring depth per warp: 3 stages when the activations are small, else 2
__host__ __device__ constexpr int q6r_stages(int mt) { return mt <= 2 ? 3 : 2; }

// shared-memory 16-byte slot of activation-quant slot s (see above)
__device__ __forceinline__ int q6r_swz(int s) { return s ^ (((s >> 3) & 3) << 1); }

struct Q6RowArgs {
    const uint8_t *w;      // [n rows][nbk * 210 B], dense, 16-byte aligned
    float *y;              // [m][y_stride]
    int64_t y_stride;
    int64_t n;             // rows (even)
    int nbk;               // superblocks per row (a multiple of 4)
    int m;                 // tokens (1..8)
    const int8_t *qs;      // Q8_K quants   [m][K]
    const float *d;        // Q8_K scales   [m][nbk]
    const int16_t *bsums;  // Q8_K 16-sums  [m][K/16]
};

__host__ __device__ constexpr int q6r_stage_bytes(int nbk) { return 2 * nbk * kQ6K_Bytes; }
__host__ __device__ constexpr int q6r_bar_bytes() { return 128 * ((kQ6rWarps * 3 * 8 + 8 + 127) / 128); }
__host__ __device__ constexpr int q6r_act_bytes(int nbk, int m) {
    return int(align_up(size_t(m) * nbk * kQK_K, 16) + align_up(size_t(m) * nbk * 4, 16) +
               align_up(size_t(m) * nbk * 32, 16));
}
// + 16 bytes: the scale words of a stage's last block are read with aligned
// 4-byte loads that may reach 2 bytes past the block
__host__ __device__ constexpr int q6r_smem_bytes(int nbk, int m) {
    return q6r_bar_bytes() + q6r_act_bytes(nbk, m) + kQ6rWarps * q6r_stages(m) * q6r_stage_bytes(nbk) + 16;
}

// One item: quarter p (h = p >> 1 picks the 128-element half, c = p & 1 the
// 16-element column pair) of superblock blk, against MT tokens' activations
// in shared memory (xq/xd/xb: quants, scales, 16-sums of token 0; tokens are
// k, nbk and k/16 apart). Adds d_w * d_x * (integer dot) to acc[t].
template <int MT>
__device__ __forceinline__ void q6r_item(const uint8_t *blk, int p, int b, const int8_t *xq, const float *xd,
                                         const int16_t *xb, int64_t k, int nbk, int m, float (&acc)[MT]) {
    const int h = p >> 1, c = p & 1;
    const uint4 qa = lds16_a2(blk + 64 * h + 16 * c);
    const uint4 qb = lds16_a2(blk + 64 * h + 32 + 16 * c);
    const uint4 qh = lds16_a2(blk + 128 + 32 * h + 16 * c);
    // scales of this item's four 16-element groups: bytes c, c+2, c+4, c+6 of scales[8h..8h+7]
    const uint8_t *sp = blk + 192 + 8 * h;
    const uintptr_t sa = reinterpret_cast<uintptr_t>(sp);
    const uint32_t *sw = reinterpret_cast<const uint32_t *>(sa & ~uintptr_t(3));
    const uint32_t ssh = uint32_t(sa & 3u) * 8u;
    const uint32_t s_lo = __funnelshift_r(sw[0], sw[1], ssh), s_hi = __funnelshift_r(sw[1], sw[2], ssh);
    const int sc0 = int(int8_t((s_lo >> (8 * c)) & 0xff));
    const int sc1 = int(int8_t((s_lo >> (8 * (c + 2))) & 0xff));
    const int sc2 = int(int8_t((s_hi >> (8 * c)) & 0xff));
    const int sc3 = int(int8_t((s_hi >> (8 * (c + 2))) & 0xff));
    const uint16_t dbits = uint16_t(blk[208]) | uint16_t(uint16_t(blk[209]) << 8);
    const float dw = half_bits_to_float(dbits);
    const uint32_t qa_[4] = {qa.x, qa.y, qa.z, qa.w}, qb_[4] = {qb.x, qb.y, qb.z, qb.w},
                   qh_[4] = {qh.x, qh.y, qh.z, qh.w};
    uint32_t r0[4], r1[4], r2[4], r3[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        r0[i] = (qa_[i] & 0x0f0f0f0fu) | ((qh_[i] << 4) & 0x30303030u);
        r1[i] = (qb_[i] & 0x0f0f0f0fu) | ((qh_[i] << 2) & 0x30303030u);
        r2[i] = ((qa_[i] >> 4) & 0x0f0f0f0fu) | (qh_[i] & 0x30303030u);
        r3[i] = ((qb_[i] >> 4) & 0x0f0f0f0fu) | ((qh_[i] >> 2) & 0x30303030u);
    }
    const int e0 = b * kQK_K + 128 * h + 16 * c;
    const int g0 = b * 16 + 8 * h + c;
    // elements e0, e0+32, e0+64, e0+96 of token 0 sit in slots s0, s0+2, s0+4, s0+6; token t is k/16 slots
    // (a multiple of 64, which the swizzle leaves alone) further on
    const int s0 = e0 >> 4;
    const int4 *xp0 = reinterpret_cast<const int4 *>(xq) + q6r_swz(s0);
    const int4 *xp1 = reinterpret_cast<const int4 *>(xq) + q6r_swz(s0 + 2);
    const int4 *xp2 = reinterpret_cast<const int4 *>(xq) + q6r_swz(s0 + 4);
    const int4 *xp3 = reinterpret_cast<const int4 *>(xq) + q6r_swz(s0 + 6);
    const int tstride = int(k >> 4);
#pragma unroll
    for (int t = 0; t < MT; t++) {
        if (t >= m) break;
        const int4 x0 = xp0[t * tstride], x1 = xp1[t * tstride], x2 = xp2[t * tstride], x3 = xp3[t * tstride];
        const int16_t *bs = xb + t * (k / 16) + g0;
        const int d0 = dp4a_us(r0[3], x0.w, dp4a_us(r0[2], x0.z, dp4a_us(r0[1], x0.y, dp4a_us(r0[0], x0.x, 0))));
        const int d1 = dp4a_us(r1[3], x1.w, dp4a_us(r1[2], x1.z, dp4a_us(r1[1], x1.y, dp4a_us(r1[0], x1.x, 0))));
        const int d2 = dp4a_us(r2[3], x2.w, dp4a_us(r2[2], x2.z, dp4a_us(r2[1], x2.y, dp4a_us(r2[0], x2.x, 0))));
        const int d3 = dp4a_us(r3[3], x3.w, dp4a_us(r3[2], x3.z, dp4a_us(r3[1], x3.y, dp4a_us(r3[0], x3.x, 0))));
        const int tot = sc0 * (d0 - 32 * int(bs[0])) + sc1 * (d1 - 32 * int(bs[2])) + sc2 * (d2 - 32 * int(bs[4])) +
                        sc3 * (d3 - 32 * int(bs[6]));
        acc[t] += (dw * xd[t * nbk + b]) * float(tot);
    }
}

template <int MT>
__global__ void __launch_bounds__(kQ6rWarps * 32, 1) gemv_q6k_rows_kernel(const __grid_constant__ Q6RowArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int kQ6rStages = q6r_stages(MT);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nbk = a.nbk;
    const int64_t k = int64_t(nbk) * kQK_K;
    const int sb = q6r_stage_bytes(nbk);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * kQ6rStages;
    uint64_t *act_bar = reinterpret_cast<uint64_t *>(smem) + kQ6rWarps * 3;
    int8_t *xq = reinterpret_cast<int8_t *>(smem + q6r_bar_bytes());
    const uint32_t qs_bytes = uint32_t(align_up(size_t(a.m) * k, 16));
    const uint32_t d_bytes = uint32_t(align_up(size_t(a.m) * nbk * 4, 16));
    const uint32_t bs_bytes = uint32_t(align_up(size_t(a.m) * nbk * 32, 16));
    float *xd = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(xq) + align_up(size_t(MT) * k, 16));
    int16_t *xb = reinterpret_cast<int16_t *>(reinterpret_cast<uint8_t *>(xd) + align_up(size_t(MT) * nbk * 4, 16));
    uint8_t *ring = smem + q6r_bar_bytes() + q6r_act_bytes(nbk, MT) + warp * kQ6rStages * sb;
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < kQ6rStages; s++) mbar_init(&bars[s], 1);
        if (warp == 0) mbar_init(act_bar, 1);
        fence_mbar_init();
    }
    __syncthreads();

    // this warp's row pairs: a contiguous range
    const int64_t npairs = a.n / 2;
    const int64_t G = int64_t(gridDim.x) * kQ6rWarps;
    const int64_t g = int64_t(blockIdx.x) * kQ6rWarps + warp;
    const int64_t p_begin = g * npairs / G, p_end = (g + 1) * npairs / G;
    const uint64_t policy = l2_policy_evict_first();
    int64_t p_issue = p_begin;
    auto issue = [&](int slot) {
        if (lane == 0) {
            mbar_arrive_expect_tx(&bars[slot], uint32_t(sb));
            bulk_g2s_stream(ring + slot * sb, a.w + size_t(p_issue) * sb, uint32_t(sb), &bars[slot], policy);
        }
        p_issue++;
    };
    for (int s = 0; s < kQ6rStages && p_issue < p_end; s++) issue(s);

    // ---- activations (written by the quantizer before this kernel) ----
    // scales and 16-sums: two bulk copies; quants: 16-byte loads stored at swizzled slots
    pdl_wait();
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(act_bar, d_bytes + bs_bytes);
        bulk_g2s(xd, a.d, d_bytes, act_bar);
        bulk_g2s(xb, a.bsums, bs_bytes, act_bar);
    }
    {
        const int4 *src = reinterpret_cast<const int4 *>(a.qs);
        int4 *dst = reinterpret_cast<int4 *>(xq);
        const int nslots = int(qs_bytes >> 4);
        for (int s = threadIdx.x; s < nslots; s += blockDim.x) dst[q6r_swz(s)] = __ldcg(src + s);
    }
    __syncthreads();
    const int64_t pre = p_issue - p_begin;
    if (!mbar_wait_bounded(act_bar, 0)) {
        // error recorded in the device word: wait (bounded) for this warp's copies, then leave
        for (int64_t j = 0; j < pre; j++) mbar_wait_bounded(&bars[j], 0);
        return;
    }
    pdl_launch_dependents();

    const int items = 8 * nbk;  // 2 rows x nbk superblocks x 4 quarters, a multiple of 32
    int slot = 0;
    uint32_t phase = 0;
    for (int64_t pr = p_begin; pr < p_end; pr++) {
        if (!mbar_wait_bounded(&bars[slot], phase)) {
            for (int k2 = 1; k2 < kQ6rStages && p_issue > pr + k2; k2++)
                mbar_wait_bounded(&bars[(slot + k2) % kQ6rStages], phase ^ uint32_t(slot + k2 >= kQ6rStages));
            return;
        }
        const uint8_t *st = ring + slot * sb;
        float acc0[MT], acc1[MT];
#pragma unroll
        for (int t = 0; t < MT; t++) acc0[t] = acc1[t] = 0.0f;
        for (int it = lane; it < items; it += 32) {
            const int row = it >= 4 * nbk;
            const int rem = it - row * 4 * nbk;
            const int b = rem >> 2;
            const uint8_t *blk = st + row * (nbk * kQ6K_Bytes) + b * kQ6K_Bytes;
            if (row) q6r_item<MT>(blk, rem & 3, b, xq, xd, xb, k, nbk, a.m, acc1);
            else q6r_item<MT>(blk, rem & 3, b, xq, xd, xb, k, nbk, a.m, acc0);
        }
        __syncwarp();
        if (p_issue < p_end) issue(slot);  // every lane is done with the stage
#pragma unroll
        for (int t = 0; t < MT; t++) {
            if (t >= a.m) break;
            const float v0 = warp_sum(acc0[t]), v1 = warp_sum(acc1[t]);
            if (lane == 0) {
                a.y[size_t(t) * a.y_stride + 2 * pr] = v0;
                a.y[size_t(t) * a.y_stride + 2 * pr + 1] = v1;
            }
        }
        if (++slot == kQ6rStages) {
            slot = 0;
            phase ^= 1u;
        }
    }
}


// ---- Q8_0 over whole row pairs -------------------------------------------
//
// The same structure for Q8_0 (ggml_vec_dot_q8_0_q8_0: 32-element blocks,
// integer dot of the quants, times d_w * d_x in fp32 per block): a stage is
// two whole rows, 2 * K/32 * 34 bytes (a multiple of 16 when K is a multiple
// of 128), one bulk copy; an item is one block of one row; the Q8_0
// activations (quants and scales) of all MT tokens are in shared memory, the
// quants at 16-byte slot s ^ ((s >> 3) & 1), which puts the two 16-byte loads
// of the 8 lanes of a quarter warp (8 consecutive blocks) on 8 different bank
// groups.

constexpr int kQ8rWarps = 8;

struct Q8RowArgs {
    const uint8_t *w;      // [n rows][nb * 34 B], dense, 16-byte aligned
    float *y;
    int64_t y_stride;
    int64_t n;             // rows (even)
    int nb;                // 32-element blocks per row (a multiple of 8: token rows are then
                           // 16-slot multiples, which the swizzle leaves alone)
    int m;
    const int8_t *qs;      // Q8_0 quants [m][K]
    const float *d;        // Q8_0 scales [m][nb] (fp16 widened)
    const float *x;        // or (quantize inside): the fp32 activations [m][x_stride], 16-byte aligned rows
    int64_t x_stride;
};

__host__ __device__ constexpr int q8r_stage_bytes(int nb) { return 2 * nb * kQ8_0_Bytes; }
__host__ __device__ constexpr int q8r_bar_bytes() { return 128 * ((kQ8rWarps * 3 * 8 + 8 + 127) / 128); }
__host__ __device__ constexpr int q8r_act_bytes(int nb, int m) {
    return int(align_up(size_t(m) * nb * kQK8_0, 16) + align_up(size_t(m) * nb * 4, 16));
}
// + 16 bytes: the last block's quants are read with aligned 4-byte loads that reach 2 bytes past it
// (w warps of s stages; the barrier area holds up to kQ8rWarps * 3 stage barriers)
__host__ __device__ constexpr int q8r_smem_bytes(int nb, int m, int w = kQ8rWarps, int s = 2) {
    return q8r_bar_bytes() + q8r_act_bytes(nb, m) + w * s * q8r_stage_bytes(nb) + 16;
}
__device__ __forceinline__ int q8r_swz(int s) { return s ^ ((s >> 3) & 1); }

// Q8_0 quantization of the activations straight into this CTA's shared
// image, with quantize_q8_0_kernel's arithmetic (x86 AVX2 semantics: d =
// fp16(amax / 127), q = round-half-even(x * 127 / amax)): four lanes per
// 32-element block, 8 elements each.
__device__ __forceinline__ void q8r_quantize_into(const Q8RowArgs &a, int8_t *xq, float *xd) {
    const int lane = threadIdx.x & 31, sub = lane & 3;
    const int nb = a.nb;
    const int tstride = nb * 2;  // 16-byte slots per token row
    const int total = a.m * nb;
    for (int base = int(threadIdx.x >> 2) - (lane >> 2); base < total; base += int(blockDim.x >> 2)) {
        const int blk = base + (lane >> 2);
        const bool valid = blk < total;
        const int t = valid ? blk / nb : 0, b = valid ? blk - t * nb : 0;
        float v[8];
        if (valid) {
            const float *xb = a.x + t * a.x_stride + b * kQK8_0 + sub * 8;
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
            int q = __float2int_rn(__fmul_rn(v[e], id));
            q = q < -128 ? -128 : (q > 127 ? 127 : q);
            if (e < 4) lo |= (uint32_t(q) & 0xffu) << (8 * e);
            else hi |= (uint32_t(q) & 0xffu) << (8 * (e - 4));
        }
        // bytes 8 sub .. 8 sub + 7 of the block: half (sub & 1) of 16-byte slot 2b + sub / 2
        uint8_t *slot = reinterpret_cast<uint8_t *>(xq) + 16 * (t * tstride + q8r_swz(2 * b + (sub >> 1)));
        *reinterpret_cast<uint2 *>(slot + 8 * (sub & 1)) = make_uint2(lo, hi);
        if (sub == 0) xd[t * nb + b] = __half2float(hd);
    }
}

// QX: the activations arrive as fp32 and are quantized here (a.x) instead of
// by a separate quantizer launch (a.qs, a.d). W warps of S ring stages.
template <int MT, bool QX = false, int W = kQ8rWarps, int S = 2>
__global__ void __launch_bounds__(W * 32, 1) gemv_q8_0_rows_kernel(const __grid_constant__ Q8RowArgs a) {
    static_assert(W * S <= kQ8rWarps * 3, "stage barriers");
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nb = a.nb;
    const int64_t k = int64_t(nb) * kQK8_0;
    const int sb = q8r_stage_bytes(nb);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * S;
    uint64_t *act_bar = reinterpret_cast<uint64_t *>(smem) + kQ8rWarps * 3;
    int8_t *xq = reinterpret_cast<int8_t *>(smem + q8r_bar_bytes());
    float *xd = reinterpret_cast<float *>(reinterpret_cast<uint8_t *>(xq) + align_up(size_t(MT) * k, 16));
    uint8_t *ring = smem + q8r_bar_bytes() + q8r_act_bytes(nb, MT) + warp * S * sb;
    const uint32_t qs_bytes = uint32_t(align_up(size_t(a.m) * k, 16));
    const uint32_t d_bytes = uint32_t(align_up(size_t(a.m) * nb * 4, 16));
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < S; s++) mbar_init(&bars[s], 1);
        if (warp == 0) mbar_init(act_bar, 1);
        fence_mbar_init();
    }
    __syncthreads();

    const int64_t npairs = a.n / 2;
    const int64_t G = int64_t(gridDim.x) * W;
    const int64_t g = int64_t(blockIdx.x) * W + warp;
    const int64_t p_begin = g * npairs / G, p_end = (g + 1) * npairs / G;
    const uint64_t policy = l2_policy_evict_first();
    int64_t p_issue = p_begin;
    auto issue = [&](int slot) {
        if (lane == 0) {
            mbar_arrive_expect_tx(&bars[slot], uint32_t(sb));
            bulk_g2s_stream(ring + slot * sb, a.w + size_t(p_issue) * sb, uint32_t(sb), &bars[slot], policy);
        }
        p_issue++;
    };
    for (int s = 0; s < S && p_issue < p_end; s++) issue(s);

    pdl_wait();
    if (QX) {
        q8r_quantize_into(a, xq, xd);
    } else {
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(act_bar, d_bytes);
            bulk_g2s(xd, a.d, d_bytes, act_bar);
        }
        const int4 *src = reinterpret_cast<const int4 *>(a.qs);
        int4 *dst = reinterpret_cast<int4 *>(xq);
        const int nslots = int(qs_bytes >> 4);
        for (int s = threadIdx.x; s < nslots; s += blockDim.x) dst[q8r_swz(s)] = __ldcg(src + s);
    }
    __syncthreads();
    const int64_t pre = p_issue - p_begin;
    if (!QX && !mbar_wait_bounded(act_bar, 0)) {
        for (int64_t j = 0; j < pre; j++) mbar_wait_bounded(&bars[j], 0);
        return;
    }
    pdl_launch_dependents();

    const int items = 2 * nb;
    const int tstride = int(k >> 4);  // slots per token row (a multiple of 8: the swizzle leaves it alone)
    int slot = 0;
    uint32_t phase = 0;
    for (int64_t pr = p_begin; pr < p_end; pr++) {
        if (!mbar_wait_bounded(&bars[slot], phase)) {
            for (int k2 = 1; k2 < S && p_issue > pr + k2; k2++)
                mbar_wait_bounded(&bars[(slot + k2) % S], phase ^ uint32_t(slot + k2 >= S));
            return;
        }
        const uint8_t *st = ring + slot * sb;
        float acc0[MT], acc1[MT];
#pragma unroll
        for (int t = 0; t < MT; t++) acc0[t] = acc1[t] = 0.0f;
        for (int it = lane; it < items; it += 32) {
            const int row = it >= nb;
            const int b = it - row * nb;
            const uint8_t *blk = st + row * (nb * kQ8_0_Bytes) + b * kQ8_0_Bytes;
            const uint16_t dbits = uint16_t(blk[0]) | uint16_t(uint16_t(blk[1]) << 8);
            const float dw = half_bits_to_float(dbits);
            const uint4 q0 = lds16_a2(blk + 2), q1 = lds16_a2(blk + 18);
            const int4 *x0p = reinterpret_cast<const int4 *>(xq) + q8r_swz(2 * b);
            const int4 *x1p = reinterpret_cast<const int4 *>(xq) + q8r_swz(2 * b + 1);
#pragma unroll
            for (int t = 0; t < MT; t++) {
                if (t >= a.m) break;
                const int4 x0 = x0p[t * tstride], x1 = x1p[t * tstride];
                int dot = __dp4a(int(q0.x), x0.x, __dp4a(int(q0.y), x0.y, __dp4a(int(q0.z), x0.z, __dp4a(int(q0.w), x0.w, 0))));
                dot = __dp4a(int(q1.x), x1.x, __dp4a(int(q1.y), x1.y, __dp4a(int(q1.z), x1.z, __dp4a(int(q1.w), x1.w, dot))));
                const float v = float(dot) * (dw * xd[t * nb + b]);
                if (row) acc1[t] += v;
                else acc0[t] += v;
            }
        }
        __syncwarp();
        if (p_issue < p_end) issue(slot);
#pragma unroll
        for (int t = 0; t < MT; t++) {
            if (t >= a.m) break;
            const float v0 = warp_sum(acc0[t]), v1 = warp_sum(acc1[t]);
            if (lane == 0) {
                a.y[size_t(t) * a.y_stride + 2 * pr] = v0;
                a.y[size_t(t) * a.y_stride + 2 * pr + 1] = v1;
            }
        }
        if (++slot == S) {
            slot = 0;
            phase ^= 1u;
        }
    }
}

}  // namespace cpq
