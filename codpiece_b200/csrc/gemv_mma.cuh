// gemv_mma.cuh — Q4_K x Q8_K mat-vec / small-M mat-mat on int8 tensor-core tiles.
//
// Same arithmetic as ggml_vec_dot_q4_K_q8_K (exact integer sub-block dots,
// six-bit scales and mins applied as integers, fp32 per superblock):
//   y[t][n] += d_w*d_x * sum_s sc_s * dot_s  -  dmin_w*d_x * sum_s m_s * bsum_s
// with dot_s = sum over the 32 elements of sub-block s of q4 * q8.
//
// Tiles. One warp multiplies 16 weight rows by up to 16 tokens with
// mma.sync m16n8k32 (A = weights, s8/u8; B = activations, s8; C = s32): one
// MMA per sub-block and token group of 8, so the instruction count per weight
// byte is the same for M = 1 and M = 8. Inside a sub-block the k index is
// permuted (k-label 4*tig+i <-> element 8*tig+i, 16+4*tig+i <-> 8*tig+4+i):
// each lane's A operand is then 8 contiguous quant bytes (one 8-byte shared
// load yields the low nibbles of sub-block 2j and the high nibbles of
// sub-block 2j+1) and its B operand is contiguous in the activation buffer,
// which the quantizer writes in this order. The min term sum_s m_s*bsum_s is
// two more MMAs per superblock (mins x low and high bytes of the sums).
//
// Memory path. Each warp streams its rows through a private ring of
// kMmaStages shared-memory stages; a stage is one 2-D TMA tensor copy (the
// weight seen as [N rows][row bytes], box = 16 rows x kMmaSB superblocks,
// no multicast) completing on one mbarrier. With two superblocks per stage
// the dense 288-byte row pitch puts four consecutive rows in distinct bank
// groups, so the 8-byte fragment loads are conflict-free.
//
// Work split (stream-K). The iteration space is (16-row block, superblock);
// every warp of the persistent grid takes an equal contiguous share, so all
// warps stream the same number of bytes. A row block cut between warps is
// finished by whichever warp arrives last on its counter: it sums the
// partials in K order (deterministic) and resets the counter for the next
// call.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace cpq {

#ifndef CPQ_MMA_WARPS
#define CPQ_MMA_WARPS 8
#endif
#ifndef CPQ_MMA_STAGES
#define CPQ_MMA_STAGES 4
#endif

constexpr int kMmaWarps = CPQ_MMA_WARPS;
constexpr int kMmaSB = 2;  // superblocks per stage (row pitch 288 B = 32 mod 128)
constexpr int kMmaStages = CPQ_MMA_STAGES;
constexpr int kMmaRows = 16;
constexpr int kMmaPitch = kMmaSB * kQ4K_Bytes;
constexpr int kMmaStageBytes = kMmaRows * kMmaPitch;
__host__ __device__ constexpr int mma_bar_bytes(int w, int st) { return 128 * ((w * st * 8 + 8 + 127) / 128); }  // + the activation barrier
__host__ __device__ constexpr int mma_smem(int w, int st) { return mma_bar_bytes(w, st) + w * st * kMmaStageBytes; }
constexpr int kMmaSmem = mma_smem(kMmaWarps, kMmaStages);
// Per instance: for M <= 8 (one token group) more warps with shallower rings
// keep more rows in flight per SM (FFN shapes at M = 8: 51.3 vs 58.2 us);
// for M <= 16 the register-heavier two-group tiles keep 8 warps x 4 stages.
template <int NG> struct MmaCfg {
    static constexpr int kWarps = NG == 1 ? 16 : kMmaWarps;
    static constexpr int kStages = NG == 1 ? 2 : kMmaStages;
};
static_assert(mma_smem(16, 2) == kMmaSmem, "every instance has the same ring bytes");
constexpr int kMmaMaxTokens = 16;
static_assert(kMmaPitch % 128 == 32, "fragment loads of rows gid..gid+3 must hit distinct bank groups");

// Activations in fragment order, per superblock b and padded token t < mp
// (tokens >= M are zero):
//   qs: [nbk][mp][tig 0..3][sub-block 0..7][8 bytes], element 32*s + 8*tig + i
//   bs: [nbk][mp][16 bytes]: bytes 0-7 = bsum_s & 255, bytes 8-15 = bsum_s >> 8
//       (bsum_s = sum of the 32 quants of sub-block s)
//   d:  [nbk][mp] f32
struct ActFrag {
    const int8_t *qs;
    const uint8_t *bs;
    const float *d;
    int mp;
};

struct alignas(64) MmaArgs {
    CUtensorMap tmap[4];     // weight i as [n rows][row bytes / 8] u64, box 16 x (kMmaSB * 18)
    float *y[4];
    int64_t n[4];            // rows of each weight
    int64_t y_stride[4];     // floats between tokens
    int64_t mb_start[5];     // prefix sums of 16-row blocks per weight
    int n_w;
    int nbk;                 // superblocks per row
    int m;                   // tokens (1..16)
    ActFrag act;
    int64_t n_warps;         // G: warps taking part (<= iterations, so none is idle)
    int act_smem;            // > 0: bytes of the activation image, copied into shared memory after the ring
    float *partials;         // [warp][2 segments][16 rows][16 tokens]
    int *counters;           // [row block], zero between calls
    ArOut ar;                // on: weight 0's rows go as LL words to every rank (the fused all-reduce)
};

__device__ __forceinline__ void mma_s8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void mma_u8u8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.u8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%11,%12,%13};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0), "r"(0), "r"(0), "r"(0));
}

__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar,
                                            uint64_t policy) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
        "%3}], [%4], %5;" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ int byte_of(uint32_t w, int k) { return int((w >> (8 * k)) & 0xffu); }

// Counter increment with release (publishes this warp's partials, which the
// preceding __syncwarp ordered before it) and acquire (the last arriver then
// sees every other warp's partials).
__device__ __forceinline__ int atom_add_acq_rel_gpu(int *p, int v) {
    int old;
    asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// The warp holding iteration i of the stream-K split: largest g with g*T/G <= i.
__device__ __forceinline__ int64_t owner_warp(int64_t i, int64_t G, int64_t T) { return ((i + 1) * G - 1) / T; }

// Activation operands of one superblock held in registers.
template <int NG>
struct ActRegs {
    uint32_t bw[NG][16];        // B fragments, token ng*8+gid
    uint32_t blo[NG], bhi[NG];  // bsum bytes for the min MMA (lanes tig 0/1), else 0
    float2 dx[NG];              // Q8_K scales of output tokens ng*8+2*tig, +1
};

// SM: the image is in shared memory (plain loads) rather than global (read-only path).
template <int NG, bool SM>
__device__ __forceinline__ void load_act(const ActFrag &act, int kb, int m, int gid, int tig, ActRegs<NG> &r) {
#pragma unroll
    for (int ng = 0; ng < NG; ng++) {
        const size_t bt = size_t(kb) * act.mp + ng * 8 + gid;
        const bool live = ng * 8 + gid < m;  // padded tokens are zero: skip their loads
        const int4 *p = reinterpret_cast<const int4 *>(act.qs + bt * 256 + tig * 64);
#pragma unroll
        for (int v = 0; v < 4; v++) {
            const int4 q = live ? (SM ? p[v] : ldg_nc_v4(p + v)) : make_int4(0, 0, 0, 0);
            r.bw[ng][4 * v + 0] = q.x;
            r.bw[ng][4 * v + 1] = q.y;
            r.bw[ng][4 * v + 2] = q.z;
            r.bw[ng][4 * v + 3] = q.w;
        }
        const int4 b = (live && tig < 2)
                           ? (SM ? *reinterpret_cast<const int4 *>(act.bs + bt * 16) : ldg_nc_v4(act.bs + bt * 16))
                           : make_int4(0, 0, 0, 0);
        r.blo[ng] = tig == 0 ? uint32_t(b.x) : (tig == 1 ? uint32_t(b.y) : 0u);
        r.bhi[ng] = tig == 0 ? uint32_t(b.z) : (tig == 1 ? uint32_t(b.w) : 0u);
        const float2 *dp = reinterpret_cast<const float2 *>(act.d + size_t(kb) * act.mp + ng * 8 + 2 * tig);
        r.dx[ng] = SM ? *dp : __ldg(dp);
    }
}

// One superblock of 16 rows (row gid at p0, row gid+8 at p1) against the
// activation operands in ar; adds to acc[ng][row pair][token pair].
template <int NG>
__device__ __forceinline__ void q4k_superblock(const uint8_t *p0, const uint8_t *p1, const ActRegs<NG> &ar, int tig,
                                               float (&acc)[NG][4]) {
    const uint4 h0 = *reinterpret_cast<const uint4 *>(p0);
    const uint4 h1 = *reinterpret_cast<const uint4 *>(p1);
    // six-bit scales (sub-blocks 0-3 | 4-7) and mins of both rows
    const uint32_t sc0a = h0.y & 0x3f3f3f3fu, sc0b = (h0.w & 0x0f0f0f0fu) | (((h0.y >> 6) & 0x03030303u) << 4);
    const uint32_t mn0a = h0.z & 0x3f3f3f3fu, mn0b = ((h0.w >> 4) & 0x0f0f0f0fu) | (((h0.z >> 6) & 0x03030303u) << 4);
    const uint32_t sc1a = h1.y & 0x3f3f3f3fu, sc1b = (h1.w & 0x0f0f0f0fu) | (((h1.y >> 6) & 0x03030303u) << 4);
    const uint32_t mn1a = h1.z & 0x3f3f3f3fu, mn1b = ((h1.w >> 4) & 0x0f0f0f0fu) | (((h1.z >> 6) & 0x03030303u) << 4);

    int ilo[NG][4], ihi[NG][4];
#pragma unroll
    for (int ng = 0; ng < NG; ng++)
#pragma unroll
        for (int i = 0; i < 4; i++) ilo[ng][i] = ihi[ng][i] = 0;
    // the superblock's quant fragments of both rows first (M = 16: 90.4 -> 87.6 us for the FFN set)
    uint2 qq0[4], qq1[4];
#pragma unroll
    for (int jj = 0; jj < 4; jj++) {
        qq0[jj] = *reinterpret_cast<const uint2 *>(p0 + 16 + 32 * jj + 8 * tig);
        qq1[jj] = *reinterpret_cast<const uint2 *>(p1 + 16 + 32 * jj + 8 * tig);
    }
#pragma unroll
    for (int jj = 0; jj < 4; jj++) {
        const uint2 q0 = qq0[jj];
        const uint2 q1 = qq1[jj];
        constexpr uint32_t M4 = 0x0f0f0f0fu, H4 = 0xf0f0f0f0u;
        const uint32_t sw0 = jj < 2 ? sc0a : sc0b, sw1 = jj < 2 ? sc1a : sc1b;
        const int sl0 = byte_of(sw0, (2 * jj) & 3), sh0 = byte_of(sw0, (2 * jj + 1) & 3);
        const int sl1 = byte_of(sw1, (2 * jj) & 3), sh1 = byte_of(sw1, (2 * jj + 1) & 3);
#pragma unroll
        for (int ng = 0; ng < NG; ng++) {
            int c[4];
            mma_s8s8(c, q0.x & M4, q1.x & M4, q0.y & M4, q1.y & M4, ar.bw[ng][4 * jj], ar.bw[ng][4 * jj + 1]);
            ilo[ng][0] += sl0 * c[0];
            ilo[ng][1] += sl0 * c[1];
            ilo[ng][2] += sl1 * c[2];
            ilo[ng][3] += sl1 * c[3];
            mma_u8s8(c, q0.x & H4, q1.x & H4, q0.y & H4, q1.y & H4, ar.bw[ng][4 * jj + 2], ar.bw[ng][4 * jj + 3]);
            ihi[ng][0] += sh0 * c[0];
            ihi[ng][1] += sh0 * c[1];
            ihi[ng][2] += sh1 * c[2];
            ihi[ng][3] += sh1 * c[3];
        }
    }
    // min term: A = mins of rows gid / gid+8 in k-labels 0..7 (lanes tig 0/1)
    const uint32_t am0 = tig == 0 ? mn0a : (tig == 1 ? mn0b : 0u);
    const uint32_t am1 = tig == 0 ? mn1a : (tig == 1 ? mn1b : 0u);
    const float dw0 = half_bits_to_float(h0.x), dm0 = half_bits_to_float(h0.x >> 16);
    const float dw1 = half_bits_to_float(h1.x), dm1 = half_bits_to_float(h1.x >> 16);
#pragma unroll
    for (int ng = 0; ng < NG; ng++) {
        int cl[4], ch[4];
        mma_u8u8(cl, am0, am1, 0u, 0u, ar.blo[ng], 0u);
        mma_u8s8(ch, am0, am1, 0u, 0u, ar.bhi[ng], 0u);
        const float dx0 = ar.dx[ng].x, dx1 = ar.dx[ng].y;
        const float dw[4] = {dw0 * dx0, dw0 * dx1, dw1 * dx0, dw1 * dx1};
        const float dm[4] = {dm0 * dx0, dm0 * dx1, dm1 * dx0, dm1 * dx1};
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int is = ilo[ng][i] + (ihi[ng][i] >> 4);  // high nibbles were fed as 16*q
            const int mn = 256 * ch[i] + cl[i];
            acc[ng][i] += dw[i] * float(is) - dm[i] * float(mn);
        }
    }
}

// SM: the activation image is copied into shared memory (a.act_smem bytes,
// after the ring) once per CTA, so the per-superblock fragment loads do not
// wait on L2.
// W warps of S ring stages each (W * S stages per CTA in all instances).
template <int NG, bool SM, int W = MmaCfg<NG>::kWarps, int S = MmaCfg<NG>::kStages>  // token groups of 8 (1: M <= 8, 2: M <= 16)
__global__ void __launch_bounds__(W * 32) gemv_q4k_mma_kernel(const __grid_constant__ MmaArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gid = lane >> 2, tig = lane & 3;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * S;
    uint64_t *act_bar = reinterpret_cast<uint64_t *>(smem) + W * S;
    uint8_t *ring = smem + mma_bar_bytes(W, S) + warp * S * kMmaStageBytes;
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < S; s++) mbar_init(&bars[s], 1);
        if (SM && warp == 0) mbar_init(act_bar, 1);
        fence_mbar_init();
    }
    __syncthreads();

    const int nbk = a.nbk;
    const int64_t T = a.mb_start[a.n_w] * nbk;
    const int64_t G = a.n_warps;
    const int64_t g = int64_t(blockIdx.x) * W + warp;
    if (g >= G) return;  // the grid is rounded up to whole CTAs
    const int64_t it_begin = g * T / G, it_end = (g + 1) * T / G;
    const uint64_t policy = l2_policy_evict_first();

    auto weight_of = [&](int64_t mb) {
        int wi = 0;
#pragma unroll
        for (int q = 1; q < 4; q++)
            if (q < a.n_w && mb >= a.mb_start[q]) wi = q;
        return wi;
    };

    // producer cursor
    int64_t p_it = it_begin, p_mb = it_begin / nbk;
    int p_kb = int(it_begin - p_mb * nbk);
    int n_issued = 0;  // stages issued before the activation wait
    auto issue = [&](int slot) {
        n_issued++;
        const int n = int(min(int64_t(min(kMmaSB, nbk - p_kb)), it_end - p_it));
        if (lane == 0) {
            const int wi = weight_of(p_mb);
            const int row0 = int((p_mb - a.mb_start[wi]) * kMmaRows);
            mbar_arrive_expect_tx(&bars[slot], kMmaStageBytes);
            tma_load_2d(ring + slot * kMmaStageBytes, &a.tmap[wi], p_kb * (kQ4K_Bytes / 8), row0, &bars[slot],
                        policy);
        }
        p_it += n;
        p_kb += n;
        if (p_kb == nbk) {
            p_kb = 0;
            p_mb++;
        }
    };
    for (int j = 0; j < S && p_it < it_end; j++) issue(j);

    pdl_wait();
    pdl_launch_dependents();
    // the all-reduce's sequence number (advanced by the consumer of the previous one)
    const unsigned ar_e = a.ar.on ? *reinterpret_cast<const volatile unsigned *>(a.ar.seq) + 1u : 0u;
    // a finished output: to Y, or (fused all-reduce) as an LL word (ar_e << 32 | value) into
    // slot (ar_e % kArSlots, this rank) of every rank's receive buffer
    auto out_row = [&](int wi, int t, int64_t row, float v) {
        if (!a.ar.on) {
            a.y[wi][size_t(t) * a.y_stride[wi] + row] = v;
            return;
        }
        const int64_t off = (int64_t(ar_e % kArSlots) * a.ar.world + a.ar.rank) * a.ar.n_max + int64_t(t) * a.ar.n + row;
        const uint64_t w = (uint64_t(ar_e) << 32) | __float_as_uint(v);
        for (int d = 0; d < a.ar.world; d++) st_relaxed_sys_u64(a.ar.peer[d] + off, w);
    };
    ActFrag act = a.act;
    if (SM) {
        // the activation image (quants, split 32-sums, scales) into shared memory after the ring
        uint8_t *as = smem + mma_smem(W, S);
        const uint32_t qb = uint32_t(nbk) * uint32_t(act.mp) * 256u, bb = uint32_t(nbk) * uint32_t(act.mp) * 16u;
        const uint32_t db = uint32_t(align_up(size_t(nbk) * act.mp * 4, 16));
        if (threadIdx.x == 0) {
            mbar_arrive_expect_tx(act_bar, qb + bb + db);
            bulk_g2s(as, a.act.qs, qb, act_bar);
            bulk_g2s(as + qb, a.act.bs, bb, act_bar);
            bulk_g2s(as + qb + bb, a.act.d, db, act_bar);
        }
        if (!mbar_wait_bounded(act_bar, 0)) {
            // error recorded in the device word: wait (bounded) for this warp's weight copies, then leave
            for (int k2 = 0; k2 < n_issued; k2++) mbar_wait_bounded(&bars[k2], 0);
            return;
        }
        act.qs = reinterpret_cast<const int8_t *>(as);
        act.bs = as + qb;
        act.d = reinterpret_cast<const float *>(as + qb + bb);
    }

    float acc[NG][4];
#pragma unroll
    for (int ng = 0; ng < NG; ng++)
#pragma unroll
        for (int i = 0; i < 4; i++) acc[ng][i] = 0.0f;

    int64_t c_it = it_begin, c_mb = it_begin / nbk;
    int c_kb = int(it_begin - c_mb * nbk);
    int64_t seg_start = it_begin;
    ActRegs<NG> ra, rb;
    load_act<NG, SM>(act, c_kb, a.m, gid, tig, ra);
    int slot = 0;
    uint32_t phase = 0;
    while (c_it < it_end) {
        const int n = int(min(int64_t(min(kMmaSB, nbk - c_kb)), it_end - c_it));
        if (!mbar_wait_bounded(&bars[slot], phase)) {
            // error recorded in the device word: wait (bounded) for the other copies
            // this warp still has in flight into its ring, then leave
            const int64_t pending = (p_it - c_it) > 0 ? 1 : 0;
            for (int k2 = 1; k2 < S && pending; k2++) {
                const int sl = (slot + k2) % S;
                mbar_wait_bounded(&bars[sl], phase ^ uint32_t(slot + k2 >= S));
            }
            return;
        }
        __syncwarp();
        const uint8_t *st = ring + slot * kMmaStageBytes;
        const uint8_t *p0 = st + gid * kMmaPitch;
        const uint8_t *p1 = st + (gid + 8) * kMmaPitch;
        // first superblock of the stage with ra while rb is loaded, then the second with rb
        {
            int kn = c_kb + 1;
            if (kn == nbk) kn = 0;
            load_act<NG, SM>(act, kn, a.m, gid, tig, rb);
            q4k_superblock<NG>(p0, p1, ra, tig, acc);
        }
        if (n == 2) {
            int kn = c_kb + 2;
            if (kn >= nbk) kn -= nbk;
            load_act<NG, SM>(act, kn, a.m, gid, tig, ra);
            q4k_superblock<NG>(p0 + kQ4K_Bytes, p1 + kQ4K_Bytes, rb, tig, acc);
        } else {
            ra = rb;
        }
        __syncwarp();
        if (p_it < it_end) issue(slot);
        c_it += n;
        c_kb += n;
        if (++slot == S) {
            slot = 0;
            phase ^= 1u;
        }

        // end of a row-block segment: write or hand over the partial sums
        if (c_kb == nbk || c_it == it_end) {
            const int wi = weight_of(c_mb);
            const int64_t row0 = (c_mb - a.mb_start[wi]) * kMmaRows;
            const int64_t rows_here = a.n[wi] - row0;
            const bool whole = (seg_start == c_mb * nbk) && (c_kb == nbk);
            if (whole) {
#pragma unroll
                for (int ng = 0; ng < NG; ng++)
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int t = ng * 8 + 2 * tig + (i & 1);
                        const int r = gid + 8 * (i >> 1);
                        if (t < a.m && r < rows_here) out_row(wi, t, row0 + r, acc[ng][i]);
                    }
            } else {
                const int64_t first = owner_warp(c_mb * nbk, G, T);
                const int64_t last = owner_warp(c_mb * nbk + nbk - 1, G, T);
                const int npieces = int(last - first + 1);
                // a warp writes at most two partial segments: the row block it starts
                // in (slot 0) and the one it ends in (slot 1)
                const int my_slot = (c_mb == it_begin / nbk) ? 0 : 1;
                float *pp = a.partials + (size_t(g) * 2 + my_slot) * (kMmaRows * kMmaMaxTokens);
#pragma unroll
                for (int ng = 0; ng < NG; ng++)
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const int t = ng * 8 + 2 * tig + (i & 1);
                        const int r = gid + 8 * (i >> 1);
                        pp[r * kMmaMaxTokens + t] = acc[ng][i];
                    }
                __syncwarp();
                int old = 0;
                if (lane == 0) old = atom_add_acq_rel_gpu(&a.counters[c_mb], 1);
                old = __shfl_sync(0xffffffffu, old, 0);
                __syncwarp();  // orders lane 0's acquire before every lane's reads below
                if (old == npieces - 1) {
                    float sum[NG][4];
#pragma unroll
                    for (int ng = 0; ng < NG; ng++)
#pragma unroll
                        for (int i = 0; i < 4; i++) sum[ng][i] = 0.0f;
                    // piece p > 0 starts inside this row block (slot 0); piece 0 uses slot 1 when
                    // its share began earlier. Loads of a batch of pieces go out together, then
                    // are added in piece order.
                    const int first_slot = (first * T / G < c_mb * nbk) ? 1 : 0;
                    constexpr int kBatch = 4;
                    for (int p0 = 0; p0 < npieces; p0 += kBatch) {
                        float pv[kBatch][NG][4];
#pragma unroll
                        for (int j = 0; j < kBatch; j++) {
                            if (p0 + j < npieces) {
                                const int sl = (p0 + j == 0) ? first_slot : 0;
                                const float *q =
                                    a.partials + (size_t(first + p0 + j) * 2 + sl) * (kMmaRows * kMmaMaxTokens);
#pragma unroll
                                for (int ng = 0; ng < NG; ng++)
#pragma unroll
                                    for (int i = 0; i < 4; i++) {
                                        const int t = ng * 8 + 2 * tig + (i & 1);
                                        const int r = gid + 8 * (i >> 1);
                                        pv[j][ng][i] = __ldcg(q + r * kMmaMaxTokens + t);
                                    }
                            }
                        }
#pragma unroll
                        for (int j = 0; j < kBatch; j++) {
                            if (p0 + j < npieces) {
#pragma unroll
                                for (int ng = 0; ng < NG; ng++)
#pragma unroll
                                    for (int i = 0; i < 4; i++) sum[ng][i] += pv[j][ng][i];
                            }
                        }
                    }
#pragma unroll
                    for (int ng = 0; ng < NG; ng++)
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const int t = ng * 8 + 2 * tig + (i & 1);
                            const int r = gid + 8 * (i >> 1);
                            if (t < a.m && r < rows_here) out_row(wi, t, row0 + r, sum[ng][i]);
                        }
                    if (lane == 0) a.counters[c_mb] = 0;  // ready for the next call
                }
            }
#pragma unroll
            for (int ng = 0; ng < NG; ng++)
#pragma unroll
                for (int i = 0; i < 4; i++) acc[ng][i] = 0.0f;
            seg_start = c_it;
            if (c_kb == nbk) {
                c_kb = 0;
                c_mb++;
            }
        }
    }
}

// Quantize fp32 rows to Q8_K in fragment order (see ActFrag), padding the
// token dimension to mp with zeros. One warp per (superblock, token), the
// same arithmetic as quantize_q8K_kernel.
// up != NULL: the quantized row is silu(x) * up (the SwiGLU before ffn_down,
// ggml's silu x / (1 + exp(-x)) then the product), up with x's row stride.
__global__ void __launch_bounds__(256) quantize_q8K_frag_kernel(const float *__restrict__ x, int64_t k, int m, int mp,
                                                                int64_t x_stride, int8_t *__restrict__ qs,
                                                                uint8_t *__restrict__ bs, float *__restrict__ dout,
                                                                const float *__restrict__ up) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31;
    const int64_t nb = k / kQK_K;
    const int64_t total = nb * mp;
    const int64_t nwarps = int64_t(gridDim.x) * (blockDim.x >> 5);
    for (int64_t w = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; w < total; w += nwarps) {
        const int64_t b = w / mp;
        const int t = int(w - b * mp);
        float v[8];
        if (t < m) {
            const float *xb = x + t * x_stride + b * kQK_K + lane * 8;
            const float4 v0 = *reinterpret_cast<const float4 *>(xb);
            const float4 v1 = *reinterpret_cast<const float4 *>(xb + 4);
            v[0] = v0.x; v[1] = v0.y; v[2] = v0.z; v[3] = v0.w;
            v[4] = v1.x; v[5] = v1.y; v[6] = v1.z; v[7] = v1.w;
            if (up) {
                const float *ub = up + t * x_stride + b * kQK_K + lane * 8;
                const float4 u0 = *reinterpret_cast<const float4 *>(ub);
                const float4 u1 = *reinterpret_cast<const float4 *>(ub + 4);
                const float u[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
                for (int e = 0; e < 8; e++) v[e] = __fmul_rn(__fdiv_rn(v[e], __fadd_rn(1.0f, expf(-v[e]))), u[e]);
            }
        } else {
#pragma unroll
            for (int e = 0; e < 8; e++) v[e] = 0.0f;
        }
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
                const int tq = __float2int_rn(__fmul_rn(iscale, v[e]));
                q[e] = tq < 127 ? tq : 127;
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
        // lane owns elements 8*lane..+7: sub-block s = lane/4, position 8*tig within it
        const int s = lane >> 2, t4 = lane & 3;
        const size_t bt = size_t(b) * mp + t;
        *reinterpret_cast<uint2 *>(qs + bt * kQK_K + t4 * 64 + s * 8) = make_uint2(lo, hi);
        int s32 = s8 + __shfl_xor_sync(0xffffffffu, s8, 1);
        s32 += __shfl_xor_sync(0xffffffffu, s32, 2);
        if (t4 == 0) {
            bs[bt * 16 + s] = uint8_t(s32 & 0xff);
            bs[bt * 16 + 8 + s] = uint8_t(int8_t(s32 >> 8));
        }
        if (lane == 0) dout[bt] = d;
    }
}

}  // namespace cpq
