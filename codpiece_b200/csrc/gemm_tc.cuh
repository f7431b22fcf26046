// gemm_tc.cuh — Q4_K chunked-prefill GEMM on 5th-generation tensor cores (tcgen05).
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
// One CTA computes a 128-row x tile_n-token tile of Y (tile_n a multiple of
// 16, at most 256) over the whole K, in stages of 64 K elements (one 128-byte
// swizzle atom per row):
//   warp 0      one lane issues tcgen05.mma.cta_group::1.kind::f16, 4 x K=16
//               per stage, into a tile_n-column fp32 TMEM accumulator, and
//               commits each stage back to its "empty" barrier
//   warp 1      one lane TMA-loads the activation stage (box 64 x tile_n fp16,
//               SWIZZLE_128B, no multicast) onto "fullB"
//   warp 2      one lane TMA-loads the tile's raw Q4_K superblocks (box 128
//               rows x 144 bytes) into a 3-slot ring ("rawFull"/"rawEmpty")
//   warps 4-7   thread r dequantizes tile row r from the raw ring into the
//               SWIZZLE_128B K-major A stage (the layout the UMMA descriptor
//               names), fences the async proxy, and the warp arrives on
//               "fullA"; after the K loop the same warps read the accumulator
//               (tcgen05.ld 32x32b: warp w sees TMEM lanes 32*(w%4)..+31 =
//               tile rows) and store Y, 32 tokens at a time.
// Waits are bounded (kWaitLimitNs); a timeout sets g_dev_error and a CTA-wide
// abort flag, every role skips to the end, the TMA lanes wait (bounded) for
// their copies in flight, the MMA lane for its last commit, and warp 0 frees
// the TMEM columns.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>

#include "common.cuh"
#include "q8k_block.cuh"

namespace cpq {

constexpr int kTcRows = 128;      // weight rows per tile (MMA M)
constexpr int kTcMaxTok = 256;    // tokens per tile at most (MMA N)
constexpr int kTcK = 64;          // K elements per stage
constexpr int kTcStages = 3;      // A/B stage ring
constexpr int kTcRawSlots = 3;    // raw superblock ring
constexpr int kTcThreads = 256;
constexpr int kTcABytes = kTcRows * 128;
constexpr int kTcBBytes = kTcMaxTok * 128;
constexpr int kTcRawBytes = kTcRows * kQ4K_Bytes;
constexpr int kTcBarOffset = kTcStages * (kTcABytes + kTcBBytes) + kTcRawSlots * kTcRawBytes;
constexpr int kTcSmem = kTcBarOffset + 256 /* barriers, TMEM slot, abort flag */ + 1024 /* alignment slack */;
static_assert(kTcRawBytes % 1024 == 0 && kTcABytes % 1024 == 0 && kTcBBytes % 1024 == 0, "1024-byte stage bases");
static_assert(kTcSmem <= 227 * 1024, "shared memory");

struct alignas(64) TcArgs {
    CUtensorMap tmap_x;  // fp16 activations [m][k], box 64 x tile_n, SWIZZLE_128B
    CUtensorMap tmap_w;  // Q4_K rows as u64 [n][k/256*18], box 18 x 128
    float *y;            // [m][y_stride]
    int64_t y_stride;
    int64_t n;           // weight rows
    int64_t m;           // tokens
    int nbk;             // superblocks per row
    int tile_n;          // tokens per tile (multiple of 16, 16..256)
};

// TMEM columns for a tile_n-column accumulator: a power of two, at least 32.
__host__ __device__ constexpr uint32_t tc_tmem_cols(int tile_n) {
    return tile_n <= 32 ? 32u : tile_n <= 64 ? 64u : tile_n <= 128 ? 128u : 256u;
}

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

__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued so far has completed.
__device__ __forceinline__ void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar))
                 : "memory");
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

// Bounded wait that also gives up as soon as another role of the CTA aborted.
__device__ __forceinline__ bool tc_wait(uint64_t *bar, uint32_t parity, volatile int *abort_flag) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 0) {
            if (*abort_flag) return false;
            if (global_timer_ns() - t0 > kWaitLimitNs) {
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

// ---- the kernel -------------------------------------------------------------

// grid: (token tiles, row tiles) — the token tiles of one weight tile run
// side by side, so its raw bytes come from HBM about once.
__global__ void __launch_bounds__(kTcThreads, 1) gemm_q4k_tc_kernel(const __grid_constant__ TcArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t *sA = smem;
    uint8_t *sB = sA + kTcStages * kTcABytes;
    uint8_t *sRaw = sB + kTcStages * kTcBBytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kTcBarOffset);
    uint64_t *fullA = bars, *fullB = bars + kTcStages, *empty = bars + 2 * kTcStages;
    uint64_t *rawFull = bars + 3 * kTcStages, *rawEmpty = rawFull + kTcRawSlots, *done = rawEmpty + kTcRawSlots;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(done + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tile_n = a.tile_n;
    const int64_t tok0 = int64_t(blockIdx.x) * tile_n;
    const int64_t row0 = int64_t(blockIdx.y) * kTcRows;
    const int nk = a.nbk * 4;
    const uint32_t ncols = tc_tmem_cols(tile_n);

    if (threadIdx.x == 0) {
        for (int s = 0; s < kTcStages; s++) {
            mbar_init(&fullA[s], 4);  // one arrival per dequantizing warp
            mbar_init(&fullB[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < kTcRawSlots; s++) {
            mbar_init(&rawFull[s], 1);
            mbar_init(&rawEmpty[s], 4);
        }
        mbar_init(done, 1);
        *abort_flag = 0;
        fence_mbar_init();
    }
    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tmem_slot)),
                     "r"(ncols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    pdl_wait();  // weights, activations and Y may all belong to earlier kernels on the stream
    pdl_launch_dependents();

    if (warp == 0) {
        // ---- MMA issue ----
        if (lane == 0) {
            const uint32_t idesc = tc_idesc_f16(kTcRows, tile_n);
            for (int t = 0; t < nk; t++) {
                const int s = t % kTcStages;
                const uint32_t ph = uint32_t(t / kTcStages) & 1u;
                if (!tc_wait(&fullA[s], ph, abort_flag) || !tc_wait(&fullB[s], ph, abort_flag)) break;
                tc_fence_after();
                const uint64_t ad = smem_desc_sw128(smem_addr(sA + s * kTcABytes));
                const uint64_t bd = smem_desc_sw128(smem_addr(sB + s * kTcBBytes));
#pragma unroll
                for (int kk = 0; kk < kTcK / 16; kk++)  // K=16 per MMA = 32 bytes = +2 in the start-address field
                    tc_mma_f16(tmem, ad + 2 * kk, bd + 2 * kk, idesc, (t | kk) != 0 ? 1u : 0u);
                tc_commit(&empty[s]);
            }
            tc_commit(done);
            mbar_wait_bounded(done, 0);  // the accumulator is final (or idle) before TMEM is released
        }
        __syncwarp();
    } else if (warp == 1) {
        // ---- activation stages (TMA) ----
        if (lane == 0) {
            int last[kTcStages];
#pragma unroll
            for (int s = 0; s < kTcStages; s++) last[s] = -1;
            for (int t = 0; t < nk; t++) {
                const int s = t % kTcStages;
                const uint32_t ph = uint32_t(t / kTcStages) & 1u;
                if (!tc_wait(&empty[s], ph ^ 1u, abort_flag)) break;
                mbar_arrive_expect_tx(&fullB[s], uint32_t(tile_n) * 128u);
                tma_load_2d(sB + s * kTcBBytes, &a.tmap_x, t * kTcK, int(tok0), &fullB[s]);
                last[s] = t;
            }
#pragma unroll
            for (int s = 0; s < kTcStages; s++)  // no copy may land after the CTA has exited
                if (last[s] >= 0) mbar_wait_bounded(&fullB[s], uint32_t(last[s] / kTcStages) & 1u);
        }
        __syncwarp();
    } else if (warp == 2) {
        // ---- raw Q4_K superblocks (TMA) ----
        if (lane == 0) {
            int last[kTcRawSlots];
#pragma unroll
            for (int s = 0; s < kTcRawSlots; s++) last[s] = -1;
            for (int kb = 0; kb < a.nbk; kb++) {
                const int s = kb % kTcRawSlots;
                const uint32_t ph = uint32_t(kb / kTcRawSlots) & 1u;
                if (!tc_wait(&rawEmpty[s], ph ^ 1u, abort_flag)) break;
                mbar_arrive_expect_tx(&rawFull[s], uint32_t(kTcRawBytes));
                tma_load_2d(sRaw + s * kTcRawBytes, &a.tmap_w, kb * (kQ4K_Bytes / 8), int(row0), &rawFull[s]);
                last[s] = kb;
            }
#pragma unroll
            for (int s = 0; s < kTcRawSlots; s++)
                if (last[s] >= 0) mbar_wait_bounded(&rawFull[s], uint32_t(last[s] / kTcRawSlots) & 1u);
        }
        __syncwarp();
    } else if (warp >= 4) {
        // ---- dequantization: thread r owns tile row r (rows past n arrive zero-filled) ----
        const int r = threadIdx.x - 128;
        const int sw = r & 7;  // the row's 16-byte chunk permutation in the swizzle atom
        bool ok = true;
        for (int t = 0; t < nk; t++) {
            const int s = t % kTcStages;
            const uint32_t ph = uint32_t(t / kTcStages) & 1u;
            const int kb = t >> 2, j = t & 3;
            const int rs = kb % kTcRawSlots;
            if (j == 0) {
                ok = __all_sync(0xffffffffu, tc_wait(&rawFull[rs], uint32_t(kb / kTcRawSlots) & 1u, abort_flag));
                if (!ok) break;
            }
            const uint8_t *raw = sRaw + rs * kTcRawBytes + r * kQ4K_Bytes;
            const uint4 hd = *reinterpret_cast<const uint4 *>(raw);
            const uint4 qa = *reinterpret_cast<const uint4 *>(raw + 16 + 32 * j);
            const uint4 qb = *reinterpret_cast<const uint4 *>(raw + 32 + 32 * j);
            if (j == 3) {  // last read of this superblock: hand the slot back
                __syncwarp();
                if (lane == 0) mbar_arrive(&rawEmpty[rs]);
            }
            // scales/mins of sub-blocks 2j (low nibbles) and 2j+1 (high nibbles): get_scale_min_k4
            const uint32_t scw = j < 2 ? (hd.y & 0x3f3f3f3fu) : ((hd.w & 0x0f0f0f0fu) | ((hd.y >> 2) & 0x30303030u));
            const uint32_t mnw =
                j < 2 ? (hd.z & 0x3f3f3f3fu) : (((hd.w >> 4) & 0x0f0f0f0fu) | ((hd.z >> 2) & 0x30303030u));
            const int sh = 16 * (j & 1);
            const float d = half_bits_to_float(hd.x), dmin = half_bits_to_float(hd.x >> 16);
            const __half2 slo = __float2half2_rn(d * float((scw >> sh) & 0xffu));
            const __half2 shi = __float2half2_rn(d * float((scw >> (sh + 8)) & 0xffu));
            const __half2 mlo = __float2half2_rn(-(dmin * float((mnw >> sh) & 0xffu)));
            const __half2 mhi = __float2half2_rn(-(dmin * float((mnw >> (sh + 8)) & 0xffu)));

            ok = __all_sync(0xffffffffu, tc_wait(&empty[s], ph ^ 1u, abort_flag));
            if (!ok) break;
            uint8_t *arow = sA + s * kTcABytes + r * 128;
            const uint32_t wq[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
            // byte i of the 32 holds element i (low nibble) and element 32+i (high nibble) of the stage
#pragma unroll
            for (int c = 0; c < 4; c++) {
                uint32_t lo[4], hi[4];
#pragma unroll
                for (int cc = 0; cc < 2; cc++) {
                    const uint32_t w = wq[2 * c + cc];
                    const uint32_t x01 = __byte_perm(w, 0, 0x4140);  // byte0 | byte1 << 16
                    const uint32_t x23 = __byte_perm(w, 0, 0x4342);  // byte2 | byte3 << 16
                    lo[2 * cc] = h2u(__hfma2(nib2h(x01), slo, mlo));
                    lo[2 * cc + 1] = h2u(__hfma2(nib2h(x23), slo, mlo));
                    hi[2 * cc] = h2u(__hfma2(nib2h(x01 >> 4), shi, mhi));
                    hi[2 * cc + 1] = h2u(__hfma2(nib2h(x23 >> 4), shi, mhi));
                }
                // elements 8c..8c+7 are 16-byte chunk c, 32+8c.. chunk 4+c; chunk q sits at q ^ (row & 7)
                *reinterpret_cast<uint4 *>(arow + ((c ^ sw) << 4)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
                *reinterpret_cast<uint4 *>(arow + (((4 + c) ^ sw) << 4)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            }
            fence_proxy_async_smem();  // make the generic stores visible to the tensor core's async proxy
            __syncwarp();
            if (lane == 0) mbar_arrive(&fullA[s]);
        }

        // ---- epilogue: TMEM lane = tile row, column = token ----
        if (ok) ok = __all_sync(0xffffffffu, tc_wait(done, 0, abort_flag));
        if (ok) {
            tc_fence_after();
            const int q = warp & 3;
            const int64_t orow = row0 + 32 * q + lane;
            const int64_t tend = a.m < tok0 + tile_n ? a.m : tok0 + tile_n;
            for (int c0 = 0; c0 < tile_n && tok0 + c0 < tend; c0 += 32) {
                float v[32];
                tmem_ld32(tmem + (uint32_t(32 * q) << 16) + uint32_t(c0), v);
                if (orow < a.n) {
                    float *yp = a.y + (tok0 + c0) * a.y_stride + orow;
#pragma unroll
                    for (int i = 0; i < 32; i++)
                        if (tok0 + c0 + i < tend) yp[int64_t(i) * a.y_stride] = v[i];
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(ncols) : "memory");
    }
}

// The tensor-core path's activations: each 256-block of x quantized to Q8_K
// exactly as quantize_row_q8_K does (q8k_quantize_block), then stored as
// fp16(d*q), dense [m][k]. One warp per (token, block), grid-stride.
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
        uint32_t h[4];
#pragma unroll
        for (int e = 0; e < 4; e++)
            h[e] = h2u(__floats2half2_rn(__fmul_rn(d, float(q[2 * e])), __fmul_rn(d, float(q[2 * e + 1]))));
        *reinterpret_cast<uint4 *>(out + row * k + b * kQK_K + lane * 8) = make_uint4(h[0], h[1], h[2], h[3]);
    }
}

}  // namespace cpq
