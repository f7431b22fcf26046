// gemm_tc.cuh — chunked-prefill GEMM on 5th-generation tensor cores (tcgen05)
// for Q4_K, Q8_0 and Q6_K weights. Written out below for Q4_K; Q8_0 and Q6_K
// differ only in how a slot of raw weights arrives and how a stage is
// dequantized (TcW and dq_*_stage), and Q8_0 activations are Q8_0- rather
// than Q8_K-quantized (act_f16_q8_0_kernel).
//
// Y[t][n] = sum_k W[n][k] * X~[t][k] for M > 16 tokens, where
//   W[n][k] = d*sc_j*q - dmin*m_j     (Q4_K, dequant_row_q4_K in ggml-quants.c)
//   X~[t][k] = d_x * q_x              (the Q8_K re-quantization ggml-cpu dots
//                                      against; act_f16_kernel below)
// Both operands enter the tensor core as fp16 and the products accumulate in
// fp32 in tensor memory (TMEM). Relative to the integer-exact CPU dot this
// adds two fp16 roundings: W as fp16(fp16(d*sc)*q - fp16(dmin*m)) (one HFMA2)
// and X~ as fp16(d_x*q_x). At the benchmark's value distributions that is a
// max |dy| / max |y| of about 4e-4 (the parity bound is 1e-3).
//
// K order. Both operands store K permuted inside every group of 8 elements
// as (0,2,1,3,4,6,5,7): a 32-bit word of Q4_K nibbles then yields two fp16
// pairs with one mask each (bits 0-3|16-19 and, shifted by 8, 8-11|24-27).
// The dot product is unchanged because A and B use the same order.
//
// A cluster of two CTAs (one per SM) computes a 256-row x tile_n-token tile
// of Y (tile_n a multiple of 32, at most 256) over the whole K, in stages of
// 128 K elements (half a superblock; 8 MMAs per stage, which keeps the
// tensor pipe busy across the per-stage barrier round trip), with 2-SM MMAs (tcgen05.mma.cta_group::2, M = 256): CTA
// rank r owns weight rows 128r..128r+127 of the pair and tokens
// tile_n/2*r.. of the activation tile; the pair's tensor cores share both
// halves of the activation operand, so each SM stores and reads only half
// of it. The dequantized weights (operand A) never touch shared memory: each
// CTA writes its rows into its own tensor memory with tcgen05.st and the MMA
// reads A from there.
// TMEM per CTA: 512 columns = the fp32 accumulator (columns 0-255, lane =
// the CTA's tile row, column = token) + kTcAStages A stages of 64 columns.
//   warp 0      (rank 0 only) one lane issues the MMAs, 8 x K=16 per stage, and
//               commits each stage to the "emptyA"/"emptyB" barriers of both
//               CTAs (multicast commit)
//   warp 1      one lane TMA-loads this CTA's half of the activation stage (two
//               boxes of 64 x tile_n/2 fp16, one per 128-byte swizzle atom,
//               SWIZZLE_128B K-major, 2-SM form, no multicast); both CTAs'
//               loads complete on rank 0's "fullB"
//   warp 2      one lane TMA-loads this CTA's raw Q4_K superblocks (box 128
//               rows x 144 bytes) into its raw ring ("rawFull"/"rawEmpty")
//   warps 4-15  dequantize, in kTcDqGroups = 3 groups of 4: warp w owns TMEM
//               lanes (rows) 32*(w%4)..+31, group g = (w-4)/4 the stages s
//               with s % 3 == g (a stage is half a superblock, s % 2 says
//               which); a thread turns its row's 64 bytes of nibbles into
//               128 fp16 and stores them as 64 columns with tcgen05.st; each
//               warp arrives on rank 0's "fullA" (8 arrivals per stage, 4
//               per CTA; a plain remote arrive: the operand lives in tensor
//               memory, ordered by the tcgen05 fences, so no cluster-scope
//               memory fence is needed). Three groups instead of two: the
//               Q4_K FFN shapes at M = 512 and 2048, FLOP-weighted, 0.571
//               -> 0.587 of the bf16 peak, Q6_K at M = 512 +9-10 % (the
//               dequantization is latency-bound per warp).
//               After the K loop they read the CTA's accumulator
//               (tcgen05.ld 32x32b), group g a third of the token columns,
//               and store Y.
// Waits are bounded (wait_limit_ns()); a timeout sets g_dev_error and a CTA-wide
// abort flag, every role skips to the end, the TMA lanes wait (bounded) for
// their copies in flight, the MMA lane for its last commit, and the TMEM is
// released after a cluster barrier. CTAs that start after any wait of the
// device has timed out skip their work (the result is then reported through
// cpq_device_status).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "q8k_block.cuh"

namespace cpq {

constexpr int kTcRows = 128;      // weight rows per CTA (the pair's MMA has M = 256)
constexpr int kTcMaxTok = 256;    // tokens per pair tile at most (MMA N)
constexpr int kTcK = 128;         // K elements per stage (two 64-element swizzle atoms)
constexpr int kTcAtomK = 64;      // K elements per 128-byte swizzle atom
constexpr int kTcMinTokens = 16;  // Q8_0 / Q6_K products above this many tokens run here
#ifndef CPQ_TC_A_STAGES
#define CPQ_TC_A_STAGES 4
#endif
#ifndef CPQ_TC_B_STAGES
#define CPQ_TC_B_STAGES 4
#endif
#ifndef CPQ_TC_RAW_SLOTS
#define CPQ_TC_RAW_SLOTS 4
#endif
constexpr int kTcAStages = CPQ_TC_A_STAGES;    // dequantized weight stages in TMEM (64 columns each)
constexpr int kTcBStages = CPQ_TC_B_STAGES;    // activation half-stages in shared memory (32 KB each)
constexpr uint32_t kTcAccCols = 256;           // accumulator columns (tile_n <= 256)
constexpr uint32_t kTcTmemCols = 512;
constexpr uint32_t kTcAStageCols = kTcK / 2;  // two fp16 per 32-bit column
static_assert(kTcAccCols + kTcAStageCols * kTcAStages <= kTcTmemCols, "TMEM columns");
// Dequantizing warps come in groups of 4 (one per TMEM lane quarter); group g
// takes the stages s with s % kTcDqGroups == g.
#ifndef CPQ_TC_DQ_GROUPS
#define CPQ_TC_DQ_GROUPS 3
#endif
constexpr int kTcDqGroups = CPQ_TC_DQ_GROUPS;
static_assert(kTcDqGroups >= 2 && kTcDqGroups <= 3, "dequant groups (512 threads at most: 128 registers)");
constexpr int kTcThreads = 128 + 128 * kTcDqGroups;  // 4 role warps + the dequantizing warps
constexpr int kTcDqWarps = 8;                        // arrivals per A stage: one group of 4 warps in each CTA
constexpr int kTcBAtomBytes = kTcMaxTok / 2 * 128;  // one swizzle atom column of the CTA's half
constexpr int kTcBBytes = kTcBAtomBytes * (kTcK / kTcAtomK);

// The raw weight ring: one slot holds 256 K elements (a Q4_K / Q6_K superblock,
// eight Q8_0 blocks) of the CTA's 128 rows.
//   Q4_K  TMA box 128 rows x 144 bytes
//   Q8_0  TMA box 128 rows x 272 bytes (K a multiple of 256 keeps rows and boxes 16-byte aligned)
//   Q6_K  210-byte superblocks are only 2-byte aligned and rows rs bytes apart, so the
//         tensor map's rows are groups of L rows (L * rs the smallest multiple of 16): one
//         box per member j of the group, 128 / L groups x 240 bytes from the superblock's
//         start (j * rs + kb * 210 in the group) rounded down to 16. Every row of box j
//         then has its superblock at the same offset (0..14) inside its 240 bytes, and
//         bytes past the matrix arrive as zeros. Slot row p holds tile row
//         L * (p % (128 / L)) + p / (128 / L).
template <int WT> struct TcW;
template <> struct TcW<CPQ_TYPE_Q4_K> {
    static constexpr int kRowBytes = kQ4K_Bytes;
    static constexpr int kSlots = CPQ_TC_RAW_SLOTS;
};
template <> struct TcW<CPQ_TYPE_Q8_0> {
    static constexpr int kRowBytes = 8 * kQ8_0_Bytes;
    static constexpr int kSlots = 2;
};
template <> struct TcW<CPQ_TYPE_Q6_K> {
    static constexpr int kRowBytes = 240;
    static constexpr int kSlots = 3;
};
template <int WT> __host__ __device__ constexpr int tc_raw_bytes() { return kTcRows * TcW<WT>::kRowBytes; }
template <int WT> __host__ __device__ constexpr int tc_bar_offset() { return kTcBStages * kTcBBytes + TcW<WT>::kSlots * tc_raw_bytes<WT>(); }
template <int WT> constexpr int tc_bar_bytes() {
    return int(align_up((2 * (kTcAStages + kTcBStages + TcW<WT>::kSlots) + 2) * 8 + 8, 128));
}
// barriers, TMEM slot and abort flag after the rings, plus alignment slack
template <int WT> constexpr int tc_smem() { return tc_bar_offset<WT>() + tc_bar_bytes<WT>() + 1024; }
static_assert(tc_raw_bytes<CPQ_TYPE_Q4_K>() % 1024 == 0 && tc_raw_bytes<CPQ_TYPE_Q8_0>() % 1024 == 0 &&
                  tc_raw_bytes<CPQ_TYPE_Q6_K>() % 1024 == 0 && kTcBBytes % 1024 == 0,
              "1024-byte stage bases");
static_assert(tc_smem<CPQ_TYPE_Q4_K>() <= 227 * 1024 && tc_smem<CPQ_TYPE_Q8_0>() <= 227 * 1024 &&
                  tc_smem<CPQ_TYPE_Q6_K>() <= 227 * 1024,
              "shared memory");
static_assert(TcW<CPQ_TYPE_Q6_K>::kRowBytes >= kQ6K_Bytes + 14 && TcW<CPQ_TYPE_Q6_K>::kRowBytes % 16 == 0,
              "Q6_K row window");

struct alignas(64) TcArgs {
    CUtensorMap tmap_x;  // fp16 activations [m][k], box 64 x tile_n/2 (one atom), SWIZZLE_128B
    CUtensorMap tmap_w;  // Q4_K / Q8_0 rows as u64, box (one slot's bytes / 8) x 128 rows
    int64_t w_rs;        // Q6_K: bytes between rows
    int q6_l;            // Q6_K: rows per 16-byte-aligned group (the tensor map's row)
    float *y;            // [m][y_stride]
    int64_t y_stride;
    int64_t n;           // weight rows
    int64_t m;           // tokens
    int nbk;             // superblocks per row
    int tile_n;          // tokens per pair tile (multiple of 32, 32..256)
    int n_pairs;         // 256-row tiles (row pairs)
    int n_tok_tiles;     // token tiles
    int k_splits;        // K ranges per (row pair, token tile); > 1: fp32 partials to part
    float *part;         // [k_splits][m][n] partial products (k_splits > 1)
};

// ---- tcgen05 / descriptor helpers ------------------------------------------

// Shared-memory matrix descriptor for a K-major SWIZZLE_128B operand whose
// 8-row x 128-byte atoms are 1024 bytes apart: start address >> 4 (bits 0-13),
// leading byte offset 16 B >> 4 (16-29; unused by this layout), stride byte
// offset 1024 B >> 4 (32-45), descriptor version 1 (46-47), base offset 0
// (49-51; atoms are 1024-byte aligned), layout SWIZZLE_128B = 2 (61-63).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
    return uint64_t((saddr >> 4) & 0x3fffu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
           (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// Instruction descriptor, kind::f16: D F32 (bits 4-5 = 1), A and B F16
// (7-9, 10-12 = 0), both K-major (15, 16 = 0), N >> 3 (17-22), M >> 4 (24-28).
__host__ __device__ constexpr uint32_t tc_idesc_f16(int m, int n) {
    return (1u << 4) | (uint32_t(n >> 3) << 17) | (uint32_t(m >> 4) << 24);
}

// 2-SM MMA issued by rank 0: D (TMEM of both CTAs) (+)= A (TMEM of both CTAs,
// K-major: lane = row, two 16-bit K elements per 32-bit column) x B (the two
// CTAs' shared-memory halves at the same descriptor address).
__device__ __forceinline__ void tc_mma2_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` in both CTAs of the pair once every tcgen05 operation this
// thread issued so far has completed.
__device__ __forceinline__ void tc_commit2(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_addr(bar)),
        "h"(uint16_t(3))
        : "memory");
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// The shared::cluster address of `p`'s counterpart in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
    return r;
}

__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Arrive on an mbarrier given by its shared::cluster address (this CTA's or
// the peer's), with the default (CTA-scope) release semantics.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t caddr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(caddr) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 2-D tiled TMA load (no multicast) completing as transaction bytes on `bar`.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// Same into this CTA's shared memory, completing on an mbarrier of either CTA
// of the pair (2-SM form; bar_caddr is a shared::cluster address). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map, int x, int y, uint32_t bar_caddr) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(bar_caddr)
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
        "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
          "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
          "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; i++) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive 32-bit TMEM columns of this thread's lane, without waiting
// for the store to complete (tcgen05.wait::st does).
__device__ __forceinline__ void tmem_st32_async(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%"
        "18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Bounded wait that also gives up as soon as another role of the CTA aborted.
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > wait_limit_ns()) {
                atomicOr(&g_dev_error, kDevErrWaitTimeout);
                *abort_flag = 1;
                return false;
            }
        }
    }
}

// fp16x2 (q0, q1) of the 4-bit values in bits 0-3 and 16-19 of x, exact:
// 0x6400 | q is the fp16 number 1024 + q.
__device__ __forceinline__ __half2 nib2h(uint32_t x) {
    const uint32_t h = (x & 0x000f000fu) | 0x64006400u;
    const uint32_t k1024 = 0x64006400u;
    return __hsub2(*reinterpret_cast<const __half2 *>(&h), *reinterpret_cast<const __half2 *>(&k1024));
}

__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<const uint32_t *>(&h); }

// ---- Q8_0 and Q6_K stages --------------------------------------------------
//
// A stage is 128 K elements of one row as 64 fp16x2 TMEM columns (two halves
// of 32 for tcgen05.st): column 4G + j holds elements 8G + {0,2}, {1,3},
// {4,6}, {5,7} for j = 0..3, the K order of the activation operand. Weights
// enter as fp16(s * q) with q exact in fp16 and s the block's fp16 scale
// (Q8_0: d; Q6_K: fp16(d * sc)), one rounding each.

__device__ __forceinline__ __half2 u32_h2(uint32_t u) { return *reinterpret_cast<const __half2 *>(&u); }

// Bytes b0..b3 of u as fp16 pairs (1024 + b0, 1024 + b2) and (1024 + b1, 1024 + b3), exact.
__device__ __forceinline__ void bytes_to_h2(uint32_t u, __half2 &e02, __half2 &e13) {
    e02 = u32_h2(__byte_perm(u, 0x64646464u, 0x4240));
    e13 = u32_h2(__byte_perm(u, 0x64646464u, 0x4341));
}

// Blocks 4 GRP .. 4 GRP + 3 of a Q8_0 row slot (8 blocks of 34 bytes).
template <int GRP>
__device__ __forceinline__ void dq_q8_0_stage(const uint8_t *row, uint32_t (&v)[2][32]) {
    uint32_t R[36];  // bytes 128 GRP .. 128 GRP + 143 of the row (16-byte aligned reads)
#pragma unroll
    for (int c = 0; c < 9; c++) {
        const uint4 x = *reinterpret_cast<const uint4 *>(row + 128 * GRP + 16 * c);
        R[4 * c] = x.x;
        R[4 * c + 1] = x.y;
        R[4 * c + 2] = x.z;
        R[4 * c + 3] = x.w;
    }
    const __half2 k1152 = __float2half2_rn(1152.0f);  // 1024 + the 128 that makes q unsigned
#pragma unroll
    for (int b = 0; b < 4; b++) {
        const int bo = 8 * GRP + 34 * b;  // the block's first byte in R
        const uint32_t dh = (R[bo >> 2] >> (8 * (bo & 3))) & 0xffffu;
        const __half2 d2 = u32_h2(dh | (dh << 16));
#pragma unroll
        for (int w = 0; w < 8; w++) {
            const int qo = bo + 2 + 4 * w;
            const uint32_t q = (qo & 3) ? __byte_perm(R[qo >> 2], R[(qo >> 2) + 1], 0x5432) : R[qo >> 2];
            __half2 e02, e13;
            bytes_to_h2(q ^ 0x80808080u, e02, e13);
            e02 = __hmul2(__hsub2(e02, k1152), d2);
            e13 = __hmul2(__hsub2(e13, k1152), d2);
            const int c = 4 * (4 * b + (w >> 1)) + 2 * (w & 1);
            v[c >> 5][c & 31] = h2u(e02);
            v[c >> 5][(c & 31) + 1] = h2u(e13);
        }
    }
}

// Half grp of a Q6_K superblock that starts sh bytes into this row's window
// (dequantize_row_q6_K: elements l + 32 j, l < 32, take ql[l] / ql[l + 32]
// low or high nibbles, bits 2j..2j+1 of qh[l] and scale sc[l / 16 + 2 j]).
__device__ __forceinline__ void dq_q6_k_stage(const uint8_t *win, int sh, int grp, uint32_t (&v)[2][32]) {
    const uint32_t sel = (sh & 2) ? 0x5432u : 0x3210u;  // sh is even: a 0- or 2-byte realignment
    const uint8_t *base = win + (sh & ~3);
    // superblock bytes [off, off + 4 n) as n words, from n + 1 aligned reads
    auto run = [&](int off, uint32_t *out, int n) {
        const uint32_t *p = reinterpret_cast<const uint32_t *>(base + off);
        uint32_t prev = p[0];
#pragma unroll
        for (int i = 0; i < 16; i++)
            if (i < n) {
                const uint32_t next = p[i + 1];
                out[i] = __byte_perm(prev, next, sel);
                prev = next;
            }
    };
    uint32_t ql[16], qh[8], sc[2];
    run(64 * grp, ql, 16);
    run(128 + 32 * grp, qh, 8);
    run(192 + 8 * grp, sc, 2);
    const float d = half_bits_to_float(*reinterpret_cast<const uint16_t *>(win + sh + 208));
    __half2 s2[8];
#pragma unroll
    for (int i = 0; i < 8; i++)
        s2[i] = __float2half2_rn(d * float(int8_t((sc[i >> 2] >> (8 * (i & 3))) & 0xffu)));
    const __half2 k1056 = __float2half2_rn(1056.0f);  // 1024 + the 32 of q - 32
#pragma unroll
    for (int l4 = 0; l4 < 8; l4++) {
        const uint32_t L0 = ql[l4], L1 = ql[8 + l4], H = qh[l4];
        const uint32_t Q[4] = {(L0 & 0x0f0f0f0fu) | ((H << 4) & 0x30303030u), (L1 & 0x0f0f0f0fu) | ((H << 2) & 0x30303030u),
                               ((L0 >> 4) & 0x0f0f0f0fu) | (H & 0x30303030u),
                               ((L1 >> 4) & 0x0f0f0f0fu) | ((H >> 2) & 0x30303030u)};
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const __half2 sj = s2[(l4 >> 2) + 2 * j];  // elements 4 l4 + 32 j .. + 3 share a 16-group
            __half2 e02, e13;
            bytes_to_h2(Q[j], e02, e13);
            e02 = __hmul2(__hsub2(e02, k1056), sj);
            e13 = __hmul2(__hsub2(e13, k1056), sj);
            const int e0 = 4 * l4 + 32 * j;  // first element of the word in the half
            const int c = 4 * (e0 >> 3) + 2 * ((e0 >> 2) & 1);
            v[c >> 5][c & 31] = h2u(e02);
            v[c >> 5][(c & 31) + 1] = h2u(e13);
        }
    }
}

// ---- the kernel -------------------------------------------------------------

// Persistent: grid = 2 x (number of CTA pairs), cluster (2, 1, 1). Pair c
// runs tiles c, c + pairs, ... of the (row pair, token tile) space, token
// tile fastest, so the token tiles of one weight tile run close together and
// its raw bytes come from HBM about once. Stage, slot and parity counters run
// across tiles, so the producers stream straight into the next tile; the
// accumulator is handed between the MMA issuer and the epilogue with
// acc_full (multicast commit) and acc_empty (the 12 epilogue warps of each
// CTA arrive on rank 0).
template <int WT>
__device__ __forceinline__ void gemm_tc_body(const TcArgs &a) {
    constexpr int kSlots = TcW<WT>::kSlots, kRaw = tc_raw_bytes<WT>();
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sB = smem;
    uint8_t *sRaw = sB + kTcBStages * kTcBBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + tc_bar_offset<WT>());
    uint64_t *fullA = bars, *emptyA = fullA + kTcAStages;
    uint64_t *fullB = emptyA + kTcAStages, *emptyB = fullB + kTcBStages;
    uint64_t *rawFull = emptyB + kTcBStages, *rawEmpty = rawFull + kSlots;
    uint64_t *acc_full = rawEmpty + kSlots, *acc_empty = acc_full + 1;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_empty + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();
    const int tile_n = a.tile_n, half_n = tile_n / 2;
    // a work unit ("tile") is a row pair x token tile x K range (superblocks [kb0, kb1))
    const int ks_n = a.k_splits;
    const int64_t n_tiles = int64_t(a.n_pairs) * a.n_tok_tiles * ks_n;
    auto tile_kb0 = [&](int64_t tile) { return int(int64_t(tile % ks_n) * a.nbk / ks_n); };
    auto tile_kb1 = [&](int64_t tile) { return int(int64_t(tile % ks_n + 1) * a.nbk / ks_n); };
    auto tile_nk = [&](int64_t tile) { return (tile_kb1(tile) - tile_kb0(tile)) * (kQK_K / kTcK); };  // stages
    const int64_t pair = blockIdx.x >> 1, n_pairs_grid = gridDim.x >> 1;
    // this pair's i-th tile: row pair and token tile
    auto tile_rows = [&](int64_t tile) {
        return (tile / ks_n / a.n_tok_tiles) * (2 * kTcRows) + int64_t(rank) * kTcRows;
    };
    auto tile_tok = [&](int64_t tile) { return (tile / ks_n % a.n_tok_tiles) * tile_n; };

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcAStages; s++) {
            mbar_init(&fullA[s], kTcDqWarps);  // rank 0: 4 warps of each CTA per stage
            mbar_init(&emptyA[s], 1);
        }
        for (int s = 0; s < kTcBStages; s++) {
            mbar_init(&fullB[s], 1);  // rank 0: its producer's arrive + both halves' bytes
            mbar_init(&emptyB[s], 1);
        }
        for (int s = 0; s < kSlots; s++) {
            mbar_init(&rawFull[s], 1);
            mbar_init(&rawEmpty[s], kTcDqWarps);
        }
        mbar_init(acc_full, 1);
        mbar_init(acc_empty, 2 * 4 * kTcDqGroups);  // rank 0: every epilogue warp of both CTAs
        // a wait on this device has already timed out: do no work (the error stays reported)
        *abort_flag = (*reinterpret_cast<volatile uint32_t *>(&g_dev_error) & kDevErrWaitTimeout) ? 1 : 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(kTcTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    cluster_sync();  // barriers of both CTAs initialised, TMEM allocated
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;  // lane 0, column base: accumulator at +0, A stages at +kTcAccCols

    pdl_wait();  // weights, activations and Y may all belong to earlier kernels on the stream
    pdl_launch_dependents();

    if (warp == 0) {
        // ---- MMA issue (rank 0) ----
        if (rank == 0 && lane == 0) {
            const uint32_t idesc = tc_idesc_f16(2 * kTcRows, tile_n);
            int64_t g = 0;      // stages issued so far (all tiles)
            int it = 0;         // tiles of this pair so far
            int committed = 0;  // acc_full commits issued
            bool ok = true;
            for (int64_t tile = pair; tile < n_tiles && ok; tile += n_pairs_grid, it++) {
                // the epilogue has drained the previous tile's accumulator
                if (it > 0 && !tc_wait(acc_empty, uint32_t(it - 1) & 1u, abort_flag)) break;
                tc_fence_after();
                const int nk = tile_nk(tile);
                for (int t = 0; t < nk; t++, g++) {
                    const int sa = int(g % kTcAStages), sb = int(g % kTcBStages);
                    if (!tc_wait(&fullA[sa], uint32_t(g / kTcAStages) & 1u, abort_flag) ||
                        !tc_wait(&fullB[sb], uint32_t(g / kTcBStages) & 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    const uint32_t at = tmem + kTcAccCols + kTcAStageCols * uint32_t(sa);
                    const uint64_t bd0 = smem_desc_sw128(smem_addr(sB + sb * kTcBBytes));
                    const uint64_t bd1 = smem_desc_sw128(smem_addr(sB + sb * kTcBBytes + kTcBAtomBytes));
#pragma unroll
                    for (int kk = 0; kk < kTcK / 16; kk++)  // K=16 per MMA: 8 TMEM columns of A, 32 B of a B atom
                        tc_mma2_f16_ts(tmem, at + 8u * uint32_t(kk), (kk < 4 ? bd0 : bd1) + 2 * (kk & 3), idesc,
                                       (t | kk) != 0 ? 1u : 0u);
                    tc_commit2(&emptyA[sa]);
                    tc_commit2(&emptyB[sb]);
                }
                if (!ok) break;
                tc_commit2(acc_full);
                committed++;
            }
            // every MMA issued has completed before TMEM is released: after an early stop, one
            // more commit tracks the partly issued tile
            if (!ok) {
                tc_commit2(acc_full);
                committed++;
            }
            if (committed > 0) mbar_wait_bounded(acc_full, uint32_t(committed - 1) & 1u);
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- this CTA's half of the activation stages (TMA, completing on rank 0) ----
        if (lane == 0) {
            int64_t g = 0;
            bool ok = true;
            for (int64_t tile = pair; tile < n_tiles && ok; tile += n_pairs_grid) {
                const int tok = int(tile_tok(tile)) + int(rank) * half_n;
                const int nk = tile_nk(tile), k0 = tile_kb0(tile) * (kQK_K / kTcK);
                for (int t = 0; t < nk; t++, g++) {
                    const int s = int(g % kTcBStages);
                    const uint32_t ph = uint32_t(g / kTcBStages) & 1u;
                    if (*abort_flag || !tc_wait(&emptyB[s], ph ^ 1u, abort_flag)) {
                        ok = false;
                        break;
                    }
                    if (rank == 0) mbar_arrive_expect_tx(&fullB[s], uint32_t(tile_n) * 2u * kTcK);
                    const uint32_t bar0 = cluster_addr(&fullB[s], 0);
#pragma unroll
                    for (int q = 0; q < kTcK / kTcAtomK; q++)
                        tma_load_2d_pair(sB + s * kTcBBytes + q * kTcBAtomBytes, &a.tmap_x,
                                         (k0 + t) * kTcK + q * kTcAtomK, tok, bar0);
                }
            }
            // no copy may land after the CTAs have exited: rank 0 waits for the last stages issued
            // (their barriers count both halves)
            if (rank == 0)
                for (int64_t u = g > kTcBStages ? g - kTcBStages : 0; u < g; u++)
                    mbar_wait_bounded(&fullB[u % kTcBStages], uint32_t(u / kTcBStages) & 1u);
        }
        __syncwarp();
    } else if (warp == 2) {
        // ---- raw weights: one slot per 256 K elements of the CTA's 128 rows ----
        int64_t g = 0;
        bool ok = true;
        for (int64_t tile = pair; tile < n_tiles && ok; tile += n_pairs_grid) {
            const int64_t row0 = tile_rows(tile);
            for (int kb = tile_kb0(tile); kb < tile_kb1(tile); kb++, g++) {
                const int s = int(g % kSlots);
                const uint32_t ph = uint32_t(g / kSlots) & 1u;
                int good = 0;
                if (lane == 0) good = !*abort_flag && tc_wait(&rawEmpty[s], ph ^ 1u, abort_flag);
                if (!__shfl_sync(0xffffffffu, good, 0)) {
                    ok = false;
                    break;
                }
                if constexpr (WT == CPQ_TYPE_Q6_K) {
                    if (lane == 0) {
                        const int L = a.q6_l, per = kTcRows / L;
                        mbar_arrive_expect_tx(&rawFull[s], uint32_t(kRaw));
                        for (int j = 0; j < L; j++)
                            tma_load_2d(sRaw + s * kRaw + j * per * TcW<WT>::kRowBytes, &a.tmap_w,
                                        int((int64_t(j) * a.w_rs + int64_t(kb) * kQ6K_Bytes) & ~int64_t(15)),
                                        int(row0 / L), &rawFull[s]);
                    }
                } else if (lane == 0) {
                    mbar_arrive_expect_tx(&rawFull[s], uint32_t(kRaw));
                    tma_load_2d(sRaw + s * kRaw, &a.tmap_w, kb * (TcW<WT>::kRowBytes / 8), int(row0), &rawFull[s]);
                }
            }
        }
        if (lane == 0)
            for (int64_t u = g > kSlots ? g - kSlots : 0; u < g; u++)
                mbar_wait_bounded(&rawFull[u % kSlots], uint32_t(u / kSlots) & 1u);
        __syncwarp();
    } else if (warp >= 4) {
        // ---- dequantization + epilogue (rows past n arrive zero-filled, so they dequantize to 0) ----
        const int dq = warp - 4;
        const int grp = dq >> 2;                      // this warp's group: stages s % kTcDqGroups == grp
        const int quarter = warp & 3;                 // TMEM lane quarter this warp may access
        const int r = 32 * quarter + lane;            // slot row = TMEM lane
        // the tile row it holds (Q6_K slots hold the rows grouped by box)
        const int row_of_lane = WT == CPQ_TYPE_Q6_K ? a.q6_l * (r % (kTcRows / a.q6_l)) + r / (kTcRows / a.q6_l) : r;
        const uint32_t lane_base = uint32_t(32 * quarter) << 16;
        const uint32_t acc_empty0 = cluster_addr(acc_empty, 0);
        int64_t gs = 0;   // stages of all tiles so far (an even count: two per superblock)
        int64_t gr = 0;   // superblocks of all tiles so far
        bool ok = true;

        // One stage: dequantize superblock half g_stage % 2 of the stage into A slot g_stage % kTcAStages.
        // kb: the superblock's index in the row; row0: the tile's first row of this CTA.
        auto dequant_stage = [&](int64_t g_stage, int64_t g_sb, int kb, int64_t row0) -> bool {
            const int hf = int(g_stage & 1);  // superblock half
            const int sa = int(g_stage % kTcAStages);
            const uint32_t pa = uint32_t(g_stage / kTcAStages) & 1u;
            const int rs = int(g_sb % kSlots);
            if (!__all_sync(0xffffffffu, tc_wait(&rawFull[rs], uint32_t(g_sb / kSlots) & 1u, abort_flag)))
                return false;
            if constexpr (WT != CPQ_TYPE_Q4_K) {
                uint32_t v[2][32];
                const uint8_t *raw = sRaw + rs * kRaw + r * TcW<WT>::kRowBytes;
                if constexpr (WT == CPQ_TYPE_Q8_0) {
                    if (hf) dq_q8_0_stage<1>(raw, v);
                    else dq_q8_0_stage<0>(raw, v);
                } else {
                    // where the superblock starts inside this row's window (the copy began 16-aligned)
                    const int j = r / (kTcRows / a.q6_l);  // the box (member of the row group)
                    const int sh = int((uint64_t(j) * uint64_t(a.w_rs) + uint64_t(kb) * kQ6K_Bytes) & 15u);
                    dq_q6_k_stage(raw, sh, hf, v);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(&rawEmpty[rs]);  // this warp is done with the slot
                if (!__all_sync(0xffffffffu, tc_wait(&emptyA[sa], pa ^ 1u, abort_flag))) return false;
                tc_fence_after();  // the MMAs that read this A stage have completed
#pragma unroll
                for (int p = 0; p < 2; p++)
                    tmem_st32_async(tmem + lane_base + kTcAccCols + kTcAStageCols * uint32_t(sa) + 32u * uint32_t(p),
                                    v[p]);
                tmem_wait_st();
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote(cluster_addr(&fullA[sa], 0));
                return true;
            }
            const uint8_t *raw = sRaw + rs * kRaw + r * kQ4K_Bytes;
            const uint4 hd = *reinterpret_cast<const uint4 *>(raw);
            uint4 qv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) qv[i] = *reinterpret_cast<const uint4 *>(raw + 16 + 64 * hf + 16 * i);
            __syncwarp();
            if (lane == 0) mbar_arrive(&rawEmpty[rs]);  // this warp is done with the superblock
            // scales/mins of sub-blocks 4*hf .. 4*hf+3 (get_scale_min_k4): bytes of these words
            const uint32_t scw = hf == 0 ? (hd.y & 0x3f3f3f3fu) : ((hd.w & 0x0f0f0f0fu) | ((hd.y >> 2) & 0x30303030u));
            const uint32_t mnw =
                hf == 0 ? (hd.z & 0x3f3f3f3fu) : (((hd.w >> 4) & 0x0f0f0f0fu) | ((hd.z >> 2) & 0x30303030u));
            const float d = half_bits_to_float(hd.x), dmin = half_bits_to_float(hd.x >> 16);
            if (!__all_sync(0xffffffffu, tc_wait(&emptyA[sa], pa ^ 1u, abort_flag))) return false;
            tc_fence_after();  // the MMAs that read this A stage have completed
            // two halves of 32 columns; the second is computed while the first is being stored
            uint32_t v[2][32];
#pragma unroll
            for (int p = 0; p < 2; p++) {
                // 32 bytes of nibbles: low nibbles = sub-block 4*hf+2p, high = 4*hf+2p+1
                const int sh = 16 * p;
                const __half2 slo = __float2half2_rn(d * float((scw >> sh) & 0xffu));
                const __half2 shi = __float2half2_rn(d * float((scw >> (sh + 8)) & 0xffu));
                const __half2 mlo = __float2half2_rn(-(dmin * float((mnw >> sh) & 0xffu)));
                const __half2 mhi = __float2half2_rn(-(dmin * float((mnw >> (sh + 8)) & 0xffu)));
                const uint4 qa = qv[2 * p], qb = qv[2 * p + 1];
                const uint32_t wq[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
                // columns 0-15: the low sub-block, 16-31: the high one; word 2c+h fills
                // columns 4c+2h (its elements 0, 2) and 4c+2h+1 (elements 1, 3)
#pragma unroll
                for (int c = 0; c < 4; c++) {
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const uint32_t w = wq[2 * c + h];
                        v[p][4 * c + 2 * h] = h2u(__hfma2(nib2h(w), slo, mlo));
                        v[p][4 * c + 2 * h + 1] = h2u(__hfma2(nib2h(w >> 8), slo, mlo));
                        v[p][16 + 4 * c + 2 * h] = h2u(__hfma2(nib2h(w >> 4), shi, mhi));
                        v[p][16 + 4 * c + 2 * h + 1] = h2u(__hfma2(nib2h(w >> 12), shi, mhi));
                    }
                }
                tmem_st32_async(tmem + lane_base + kTcAccCols + kTcAStageCols * uint32_t(sa) + 32u * uint32_t(p),
                                v[p]);
            }
            tmem_wait_st();
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(cluster_addr(&fullA[sa], 0));
            return true;
        };

        // The accumulator of tile `tile` (this pair's it-th) to Y, then released to the MMA issuer.
        auto epilogue = [&](int64_t tile, int it) -> bool {
            if (!__all_sync(0xffffffffu, tc_wait(acc_full, uint32_t(it) & 1u, abort_flag))) return false;
            tc_fence_after();
            const int64_t tok0 = tile_tok(tile);
            const int64_t orow = tile_rows(tile) + row_of_lane;
            const int64_t tend = a.m < tok0 + tile_n ? a.m : tok0 + tile_n;
            // a K range's partial products go to its own plane of part; a whole K to Y
            float *yb = ks_n > 1 ? a.part + (tile % ks_n) * a.m * a.n : a.y;
            const int64_t ys = ks_n > 1 ? a.n : a.y_stride;
            // group grp drains columns [grp * part, (grp + 1) * part) (part a multiple of 32)
            const int part = (((tile_n + kTcDqGroups - 1) / kTcDqGroups) + 31) & ~31;
            const int cbeg = grp * part, cend = (grp + 1) * part < tile_n ? (grp + 1) * part : tile_n;
            for (int c0 = cbeg; c0 < cend && tok0 + c0 < tend; c0 += 32) {
                float v[32];
                tmem_ld32(tmem + lane_base + uint32_t(c0), v);
                if (orow < a.n) {
                    float *yp = yb + (tok0 + c0) * ys + orow;
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (tok0 + c0 + i < tend) yp[int64_t(i) * ys] = v[i];
                }
            }
            tc_fence_before();  // the TMEM reads are complete (tmem_ld32 waits for them)
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(acc_empty0);
            return true;
        };

        int it = 0;
        int64_t prev_tile = -1;
        for (int64_t tile = pair; tile < n_tiles && ok; tile += n_pairs_grid, it++) {
            // the first stages of this tile fill the A ring while the MMA finishes the previous
            // tile; then this warp drains the previous tile's accumulator, then continues
            const int64_t g0 = gs, r0 = gr;
            int t = grp;
            const int prefill = kTcAStages;  // stages of this tile (all groups) before the epilogue
            const int64_t row0 = tile_rows(tile);
            const int nk = tile_nk(tile), kb0 = tile_kb0(tile);
            for (; t < nk && t < prefill && ok; t += kTcDqGroups)
                ok = dequant_stage(g0 + t, r0 + (t >> 1), kb0 + (t >> 1), row0);
            if (ok && prev_tile >= 0) ok = epilogue(prev_tile, it - 1);
            for (; t < nk && ok; t += kTcDqGroups) ok = dequant_stage(g0 + t, r0 + (t >> 1), kb0 + (t >> 1), row0);
            gs += nk;
            gr += tile_kb1(tile) - kb0;
            prev_tile = tile;
        }
        if (ok && prev_tile >= 0) epilogue(prev_tile, it - 1);
    }

    tc_fence_before();
    cluster_sync();  // neither CTA releases TMEM or exits while the pair's MMAs may still use it
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTcTmemCols) : "memory");
    }
}

__global__ void __launch_bounds__(kTcThreads, 1) gemm_q4k_tc_kernel(const __grid_constant__ TcArgs a) {
    gemm_tc_body<CPQ_TYPE_Q4_K>(a);
}
__global__ void __launch_bounds__(kTcThreads, 1) gemm_q8_0_tc_kernel(const __grid_constant__ TcArgs a) {
    gemm_tc_body<CPQ_TYPE_Q8_0>(a);
}
__global__ void __launch_bounds__(kTcThreads, 1) gemm_q6k_tc_kernel(const __grid_constant__ TcArgs a) {
    gemm_tc_body<CPQ_TYPE_Q6_K>(a);
}

// Y = the K ranges' partial products added in range order (deterministic).
// No early trigger of dependents: the next GEMM may overwrite part only after
// this kernel has finished reading it.
__global__ void __launch_bounds__(256) tc_split_reduce_kernel(const float *__restrict__ part, int splits, int64_t m,
                                                              int64_t n, float *__restrict__ y, int64_t y_stride) {
    pdl_wait();
    const int64_t plane = m * n;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < plane; i += int64_t(gridDim.x) * blockDim.x) {
        float v = part[i];
        for (int s = 1; s < splits; s++) v = __fadd_rn(v, part[s * plane + i]);
        const int64_t t = i / n;
        y[t * y_stride + (i - t * n)] = v;
    }
}

// The tensor-core path's activations: each 256-block of x quantized to Q8_K
// exactly as quantize_row_q8_K does (q8k_quantize_block), then stored as
// fp16(d*q), [m][k] with K permuted as (0,2,1,3,4,6,5,7) inside every group
// of 8 (the A operand's order). One warp per (token, block), grid-stride.
__global__ void __launch_bounds__(256) act_f16_kernel(const float *__restrict__ x, int64_t k, int64_t m,
                                                      int64_t x_stride, __half *__restrict__ out) {
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
        int q[8];
        const float d = q8k_quantize_block(v, lane, q);
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; e++) f[e] = __fmul_rn(d, float(q[e]));
        const uint32_t h[4] = {h2u(__floats2half2_rn(f[0], f[2])), h2u(__floats2half2_rn(f[1], f[3])),
                               h2u(__floats2half2_rn(f[4], f[6])), h2u(__floats2half2_rn(f[5], f[7]))};
        *reinterpret_cast<uint4 *>(out + row * k + b * kQK_K + lane * 8) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

// The same for Q8_0 weights: each 32-block of x quantized to Q8_0 exactly as
// quantize_q8_0_kernel does (the x86 AVX2 semantics: d = fp16(amax / 127),
// q = round-half-even(x * 127 / amax)), stored as fp16(d * q) in the permuted
// K order. Four lanes per block, grid-stride over whole warps.
__global__ void __launch_bounds__(256) act_f16_q8_0_kernel(const float *__restrict__ x, int64_t k, int64_t m,
                                                           int64_t x_stride, __half *__restrict__ out) {
    pdl_wait();
    pdl_launch_dependents();
    const int lane = threadIdx.x & 31, sub = lane & 3;
    const int64_t nb = k / kQK8_0;
    const int64_t total = m * nb;
    const int64_t groups_per_iter = int64_t(gridDim.x) * blockDim.x / 4;
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
        const float d = __half2float(__float2half_rn(__fdiv_rn(amax, 127.0f)));
        const float id = amax != 0.0f ? __fdiv_rn(127.0f, amax) : 0.0f;
        float f[8];
#pragma unroll
        for (int e = 0; e < 8; e++) {
            int t = __float2int_rn(__fmul_rn(v[e], id));
            t = t < -128 ? -128 : (t > 127 ? 127 : t);
            f[e] = __fmul_rn(d, float(t));
        }
        const uint32_t h[4] = {h2u(__floats2half2_rn(f[0], f[2])), h2u(__floats2half2_rn(f[1], f[3])),
                               h2u(__floats2half2_rn(f[4], f[6])), h2u(__floats2half2_rn(f[5], f[7]))};
        *reinterpret_cast<uint4 *>(out + row * k + b * kQK8_0 + sub * 8) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

}  // namespace cpq
