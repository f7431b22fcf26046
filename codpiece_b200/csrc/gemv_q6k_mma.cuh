// gemv_q6k_mma.cuh — Q6_K x Q8_K for M = 1..16 tokens on int8 tensor-core tiles.
//
// Same arithmetic as ggml_vec_dot_q6_K_q8_K: per 16-element group g of a
// superblock the integer dot of the 6-bit quants q with the Q8_K quants, minus
// 32 * bsum_g (the -32 offset), times the int8 group scale s_g, summed exactly
// in integers over the superblock; then d_w * d_x in fp32 per superblock.
//
// Roles. mma.sync m16n8k16 with A = activations (16 tokens x 16 k, s8) and
// B = weights (16 k x 8 rows, the 6-bit quants as u8), one MMA per scale
// group: the instruction count per weight byte is the same for any M <= 16,
// so a verify batch streams the weights once. The -32 * sum_g s_g * bsum_g
// term is two more MMAs per superblock: A = the bytes of bsum (low as u8,
// high as s8; 16 groups = the k of one MMA) against B = the scales.
//
// Tiles. A tile is 8 consecutive weight rows over the whole K: 8 * K/256 *
// 210 bytes, a multiple of 16 whatever the row alignment, fetched by one bulk
// copy into a ring of q6m_stages() tile slots shared by the CTA. For M <= 8
// the CTA has two teams of W = 10 warps taking alternate tiles (fewer warps
// per scheduler are too few to hide the latency of this kernel's long
// dependent chains); the ring then has an even number of slots, so the
// previous tile in a slot always belongs to the same team, whose warps have
// waited for it: a wait on a slot's barrier is never two phases behind. For
// M <= 16 the larger activations leave room for three slots and one team of
// W = 10. In a team, warp w takes superblocks [w*nbk/W, (w+1)*nbk/W) of the
// tile (two each at K = 5120; with 8 warps some took three, which set the
// tile's time: head at M = 4 / 8 / 16 232 / 234 / 330 -> 204 / 207 / 312 us)
// and leaves its fp32 partial [16 tokens][8 rows] in a per-slot buffer; the
// last warp to arrive (shared-memory counter) adds the W partials in warp
// order, stores the rows and refills the slot with the tile q6m_stages()
// ahead. CTAs take contiguous ranges of tiles. The M <= 8 instance runs 640
// threads (at most 102 registers: a few bytes spill, measured cheaper than 8
// warps without spills).
//
// Activations in shared memory (copied once per CTA from the quantizer's
// image): quants per token row (row stride K + 64 bytes), inside each
// superblock in fragment order: lane quarter tig owns 64 bytes holding, for
// groups g = 0..15, elements 16g + 4tig .. 16g + 4tig + 3; its four 16-byte
// chunks (groups 4c..4c+3) are stored at position c ^ tig. With the 64-byte
// row padding, the 8 lanes of a quarter warp read 8 different bank groups.
// bsums split into a low-byte and a high-byte plane [token][K/16], d [token][nbk].
#pragma once

#include "gemv_mma.cuh"

namespace cpq {

#ifndef CPQ_Q6M_WARPS8
#define CPQ_Q6M_WARPS8 10
#endif
#ifndef CPQ_Q6M_WARPS16
#define CPQ_Q6M_WARPS16 10
#endif
// warps of a team (one tile): CPQ_Q6M_WARPS8 for M <= 8 (two teams), CPQ_Q6M_WARPS16 for M <= 16 (one team)
__host__ __device__ constexpr int q6m_warps(int mt) { return mt <= 8 ? CPQ_Q6M_WARPS8 : CPQ_Q6M_WARPS16; }
__host__ __device__ constexpr int q6m_teams(int mt) { return mt <= 8 ? 2 : 1; }
__host__ __device__ constexpr int q6m_threads(int mt) { return q6m_warps(mt) * q6m_teams(mt) * 32; }
constexpr int kQ6mMaxK = 30 * kQK_K;  // 8 rows x 30 superblocks = 50,400 B per tile
__host__ __device__ constexpr int q6m_stages(int mt) { return mt <= 8 ? 4 : 3; }
static_assert(q6m_stages(8) % 2 == 0, "two teams need an even ring");
__host__ __device__ constexpr int q6m_tile_bytes(int nbk) { return 8 * nbk * kQ6K_Bytes; }
__host__ __device__ constexpr int q6m_qs_stride(int nbk) { return nbk * kQK_K + 64; }
__host__ __device__ constexpr int q6m_act_bytes(int nbk, int mt) {
    return int(align_up(size_t(mt) * q6m_qs_stride(nbk), 16) + 2 * align_up(size_t(mt) * nbk * 16, 16) +
               align_up(size_t(mt) * nbk * 4, 16));
}
// one slot of partials: [warp][16 tokens][8 rows] fp32
__host__ __device__ constexpr int q6m_red_bytes(int mt) { return q6m_warps(mt) * 16 * 8 * 4; }
__host__ __device__ constexpr int q6m_smem_bytes(int nbk, int mt) {
    return 256 + q6m_act_bytes(nbk, mt) + q6m_stages(mt) * (q6m_tile_bytes(nbk) + q6m_red_bytes(mt)) + 16;
}

struct Q6MmaArgs {
    const uint8_t *w;      // [n rows][nbk * 210 B], dense
    float *y;              // [m][y_stride]
    int64_t y_stride;
    int64_t n;             // rows (a multiple of 8)
    int nbk;               // superblocks per row (<= 30)
    int m;                 // tokens (1..16)
    const int8_t *qs;      // Q8_K quants   [m][K]
    const float *d;        // Q8_K scales   [m][nbk]
    const int16_t *bsums;  // Q8_K 16-sums  [m][K/16]
};

__device__ __forceinline__ void mma_k16(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0, bool a_unsigned) {
    if (a_unsigned)
        asm("mma.sync.aligned.m16n8k16.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
                     : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
                     : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
    else
        asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
                     : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
                     : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}

// A = activations (s8), B = 6-bit quants (u8).
__device__ __forceinline__ void mma_k16_s8u8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t b0) {
    asm("mma.sync.aligned.m16n8k16.row.col.s32.s8.u8.s32 {%0,%1,%2,%3}, {%4,%5}, {%6}, {%7,%8,%9,%10};"
                 : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
                 : "r"(a0), "r"(a1), "r"(b0), "r"(0), "r"(0), "r"(0), "r"(0));
}

// 4 bytes from shared memory at a 2-byte aligned address.
__device__ __forceinline__ uint32_t lds4_a2(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    return __funnelshift_r(w[0], w[1], uint32_t(a & 3u) * 8u);
}

__device__ __forceinline__ int sbyte(uint32_t w, int i) { return int(int8_t(uint8_t(w >> (8 * i)))); }

__device__ __forceinline__ uint32_t u4_word(const uint4 &v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// Copies the quantizer's Q8_K image of m tokens into shared memory in the
// layout described at the top (tokens m..MT-1 zero). All threads.
template <int MT>
__device__ __forceinline__ void q6m_load_act(const Q6MmaArgs &a, int8_t *xq, uint8_t *blo, uint8_t *bhi, float *xd) {
    const int nbk = a.nbk;
    const int64_t k = int64_t(nbk) * kQK_K;
    const int qstride = q6m_qs_stride(nbk);
    // quants: one 16-byte group (16 elements: words tig' = 0..3) per thread and step
    const int ngroups = MT * nbk * 16;
    for (int u = threadIdx.x; u < ngroups; u += blockDim.x) {
        const int t = u / (nbk * 16), r = u - t * (nbk * 16), b = r >> 4, g = r & 15;
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (t < a.m) v = __ldcg(reinterpret_cast<const uint4 *>(a.qs + int64_t(t) * k + b * kQK_K + 16 * g));
        int8_t *dst = xq + t * qstride + b * kQK_K + 4 * (g & 3);
#pragma unroll
        for (int tg = 0; tg < 4; tg++)
            *reinterpret_cast<uint32_t *>(dst + 64 * tg + 16 * ((g >> 2) ^ tg)) = u4_word(v, tg);
    }
    // 16-sums as low and high byte planes, scales
    for (int u = threadIdx.x; u < MT * nbk * 16; u += blockDim.x) {
        const int t = u / (nbk * 16);
        const int bs = t < a.m ? int(a.bsums[int64_t(t) * (k / 16) + (u - t * nbk * 16)]) : 0;
        blo[u] = uint8_t(bs & 0xff);
        bhi[u] = uint8_t(int8_t(bs >> 8));
    }
    for (int u = threadIdx.x; u < MT * nbk; u += blockDim.x) {
        const int t = u / nbk;
        xd[u] = t < a.m ? a.d[int64_t(t) * nbk + (u - t * nbk)] : 0.0f;
    }
}

// One superblock b of the 8-row tile against the tokens: this lane's four
// outputs (tokens gid, gid+8 x rows 2tig, 2tig+1) in acc.
template <int MT>
__device__ __forceinline__ void q6m_superblock(const uint8_t *tile, int rowb, int b, const int8_t *xq, int qstride,
                                               const uint8_t *blo, const uint8_t *bhi, const float *xd, int nbk,
                                               float (&acc)[4]) {
    const int lane = threadIdx.x & 31, gid = lane >> 2, tig = lane & 3;
    // B operand: row gid, k = 4tig..4tig+3 of each 16-element group
    const uint8_t *blk = tile + gid * rowb + b * kQ6K_Bytes;
    uint32_t qlw[2][2][2], qhw[2][2];
#pragma unroll
    for (int n = 0; n < 2; n++)
#pragma unroll
        for (int hh = 0; hh < 2; hh++) {
#pragma unroll
            for (int jb = 0; jb < 2; jb++) qlw[n][jb][hh] = lds4_a2(blk + 64 * n + 32 * jb + 16 * hh + 4 * tig);
            qhw[n][hh] = lds4_a2(blk + 128 + 32 * n + 16 * hh + 4 * tig);
        }
    const uint32_t scb = lds4_a2(blk + 192 + 4 * tig);
    // the scales and d of rows 2tig, 2tig+1 (the rows of this lane's outputs)
    const uint8_t *ba = tile + (2 * tig) * rowb + b * kQ6K_Bytes, *bb = ba + rowb;
    const uint4 sca = lds16_a2(ba + 192), scbb = lds16_a2(bb + 192);
    const float dwa = __half2float(*reinterpret_cast<const __half *>(ba + 208));
    const float dwb = __half2float(*reinterpret_cast<const __half *>(bb + 208));
    // A operand: tokens gid (and gid+8), four 16-byte chunks (stored at c ^ tig)
    const int8_t *xa = xq + gid * qstride + b * kQK_K + 64 * tig;
    uint4 A0[4], A1[4];
#pragma unroll
    for (int c = 0; c < 4; c++) {
        A0[c] = *reinterpret_cast<const uint4 *>(xa + 16 * (c ^ tig));
        A1[c] = MT > 8 ? *reinterpret_cast<const uint4 *>(xa + 8 * qstride + 16 * (c ^ tig)) : make_uint4(0u, 0u, 0u, 0u);
    }
    int isum[4] = {0, 0, 0, 0};
#pragma unroll
    for (int g = 0; g < 16; g++) {
        const int n = g >> 3, gp = g & 7, j = gp >> 1, hh = gp & 1;
        const uint32_t bw = ((qlw[n][j & 1][hh] >> (4 * (j >> 1))) & 0x0f0f0f0fu) |
                            (((qhw[n][hh] >> (2 * j)) & 0x03030303u) << 4);
        int cc[4];
        mma_k16_s8u8(cc, u4_word(A0[g >> 2], g & 3), u4_word(A1[g >> 2], g & 3), bw);
        const int s0 = sbyte(u4_word(sca, g >> 2), g & 3), s1 = sbyte(u4_word(scbb, g >> 2), g & 3);
        isum[0] += s0 * cc[0];
        isum[1] += s1 * cc[1];
        if (MT > 8) {  // tokens gid + 8 (zero rows of A for M <= 8)
            isum[2] += s0 * cc[2];
            isum[3] += s1 * cc[3];
        }
    }
    // sum_g s_g * bsum_g for the -32 offset: bsum bytes (16 groups = k) x scales
    const int bo = b * 16 + 4 * tig;
    const uint32_t l0 = *reinterpret_cast<const uint32_t *>(blo + gid * nbk * 16 + bo);
    const uint32_t h0 = *reinterpret_cast<const uint32_t *>(bhi + gid * nbk * 16 + bo);
    const uint32_t l1 = MT > 8 ? *reinterpret_cast<const uint32_t *>(blo + (gid + 8) * nbk * 16 + bo) : 0u;
    const uint32_t h1 = MT > 8 ? *reinterpret_cast<const uint32_t *>(bhi + (gid + 8) * nbk * 16 + bo) : 0u;
    int cl[4], ch[4];
    mma_k16(cl, l0, l1, scb, true);
    mma_k16(ch, h0, h1, scb, false);
    const float dx0 = xd[gid * nbk + b], dx1 = MT > 8 ? xd[(gid + 8) * nbk + b] : 0.0f;
    acc[0] += (dwa * dx0) * float(isum[0] - 32 * (cl[0] + 256 * ch[0]));
    acc[1] += (dwb * dx0) * float(isum[1] - 32 * (cl[1] + 256 * ch[1]));
    if (MT > 8) {
        acc[2] += (dwa * dx1) * float(isum[2] - 32 * (cl[2] + 256 * ch[2]));
        acc[3] += (dwb * dx1) * float(isum[3] - 32 * (cl[3] + 256 * ch[3]));
    }
}

template <int MT>
__global__ void __launch_bounds__(q6m_threads(MT), 1) gemv_q6k_mma_kernel(const __grid_constant__ Q6MmaArgs a) {
    constexpr int S = q6m_stages(MT);
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int kQ6mWarps = q6m_warps(MT);
    const int lane = threadIdx.x & 31, team = int(threadIdx.x >> 5) / kQ6mWarps, warp = int(threadIdx.x >> 5) % kQ6mWarps;
    const int gid = lane >> 2, tig = lane & 3;
    const int nbk = a.nbk;
    const int rowb = nbk * kQ6K_Bytes;
    const int tb = q6m_tile_bytes(nbk);
    const int qstride = q6m_qs_stride(nbk);
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);   // [S]: the tile landed
    int *tcnt = reinterpret_cast<int *>(smem + 64);       // [S]: warps done with the tile
    int *issued = reinterpret_cast<int *>(smem + 128);    // [S]: copies issued into the slot
    int8_t *xq = reinterpret_cast<int8_t *>(smem + 256);
    uint8_t *blo = smem + 256 + align_up(size_t(MT) * qstride, 16);
    uint8_t *bhi = blo + align_up(size_t(MT) * nbk * 16, 16);
    float *xd = reinterpret_cast<float *>(bhi + align_up(size_t(MT) * nbk * 16, 16));
    uint8_t *tiles = smem + 256 + q6m_act_bytes(nbk, MT);
    float *red = reinterpret_cast<float *>(tiles + size_t(S) * tb);  // [S][warp][16 tokens][8 rows]

    const int64_t T = a.n / 8;
    const int64_t t0 = int64_t(blockIdx.x) * T / gridDim.x, t1 = int64_t(blockIdx.x + 1) * T / gridDim.x;
    const uint64_t policy = l2_policy_evict_first();
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            tcnt[s] = 0;
            issued[s] = 0;
        }
        fence_mbar_init();
        // the weight tiles do not depend on the previous kernel: issue them before griddepcontrol.wait
        for (int s = 0; s < S && t0 + s < t1; s++) {
            mbar_arrive_expect_tx(&full[s], uint32_t(tb));
            bulk_g2s_stream(tiles + size_t(s) * tb, a.w + size_t(t0 + s) * tb, uint32_t(tb), &full[s], policy);
            issued[s] = 1;
        }
    }
    pdl_wait();
    q6m_load_act<MT>(a, xq, blo, bhi, xd);
    __syncthreads();
    pdl_launch_dependents();

    const int sb0 = warp * nbk / kQ6mWarps, sb1 = (warp + 1) * nbk / kQ6mWarps;
    for (int64_t t = t0 + team; t < t1; t += q6m_teams(MT)) {
        const int64_t i = t - t0;
        const int s = int(i % S);
        if (!mbar_wait_bounded(&full[s], uint32_t(i / S) & 1u)) break;  // error recorded in the device word
        const uint8_t *tile = tiles + size_t(s) * tb;
        float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        for (int b = sb0; b < sb1; b++) q6m_superblock<MT>(tile, rowb, b, xq, qstride, blo, bhi, xd, nbk, acc);
        float *rw = red + (size_t(s) * kQ6mWarps + warp) * 128;
        rw[gid * 8 + 2 * tig] = acc[0];
        rw[gid * 8 + 2 * tig + 1] = acc[1];
        rw[(gid + 8) * 8 + 2 * tig] = acc[2];
        rw[(gid + 8) * 8 + 2 * tig + 1] = acc[3];
        __syncwarp();
        int old = 0;
        if (lane == 0) {
            __threadfence_block();
            old = atomicAdd(&tcnt[s], 1);
        }
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old != kQ6mWarps - 1) continue;
        // the last warp with this tile: partials in warp order, then the slot takes tile t + S
        __threadfence_block();
        const float *rs = red + size_t(s) * kQ6mWarps * 128;
        for (int e = lane; e < 128; e += 32) {
            const int tok = e >> 3;
            float v = 0.0f;
#pragma unroll
            for (int w = 0; w < kQ6mWarps; w++) v += rs[w * 128 + e];
            if (tok < a.m) a.y[size_t(tok) * a.y_stride + t * 8 + (e & 7)] = v;
        }
        __syncwarp();
        if (lane == 0) {
            tcnt[s] = 0;
            if (t + S < t1) {
                fence_proxy_async_smem();  // the generic reads of the slot come before the copy's writes
                mbar_arrive_expect_tx(&full[s], uint32_t(tb));
                bulk_g2s_stream(tiles + size_t(s) * tb, a.w + size_t(t + S) * tb, uint32_t(tb), &full[s], policy);
                issued[s]++;
            }
        }
    }
    // copies still in flight (only after an error) land before the CTA leaves
    __syncthreads();
    if (threadIdx.x == 0)
        for (int s = 0; s < S; s++)
            if (issued[s] > 0) mbar_wait_bounded(&full[s], uint32_t(issued[s] - 1) & 1u);
}

}  // namespace cpq
