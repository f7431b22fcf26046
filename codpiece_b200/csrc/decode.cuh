// decode.cuh — persistent decode step: a chain of Q4_K GEMV phases in one launch.
//
// Batch-1 decode streams every weight once per token, so the step is bound by
// HBM as long as the weight stream never stops. Launched one GEMV at a time,
// it stops at every kernel boundary: the next GEMV cannot prefetch until the
// previous one has left its SMs, and its activations are produced by yet
// another kernel. This kernel runs the whole chain (a table of phases; a
// phase = up to three Q4_K weights sharing one input, e.g. q/k/v or
// gate/up) as one cooperative launch with one CTA per SM:
//
//  * every warp owns a ring of TMA stages (32 rows x one superblock each,
//    no multicast) whose issue cursor walks the warp's stream-K share of
//    phase 0, then of phase 1, ...: while a phase's input is still being
//    produced, the next phase's weights are already in flight;
//  * a phase starts after a grid barrier (all CTAs finished the previous
//    phase). Its Q8_K activation image (with the fused prologue: RMS norm
//    with residual add, SwiGLU, or none) is then built across the grid, one
//    256-element block per warp (warp c*8+w builds block c*8+w; CTAs that
//    build RMS blocks first compute the row's scale), through the same
//    device functions as act_prep_kernel, into a global image; after a
//    second grid barrier every CTA copies the image (at most a few tens of
//    KB) into its shared memory with vector loads;
//  * the dot products and the stream-K fix-up are gemv_row.cuh's (row_dot,
//    row_segment_end) with the same warp count, so a phase's output is bit
//    for bit what the separate act_prep + GEMV launches produce.
//
// Inputs written by an earlier phase are read with L2-coherent loads
// (ld.global.cg). Every wait is bounded: a timeout sets the device error
// word, the CTA stops at the next phase boundary, waits (bounded) for its
// copies in flight and exits; the other CTAs then time out on the barrier.
#pragma once

#include "act_prep.cuh"
#include "gemv_row.cuh"

namespace cpq {

constexpr int kDecWarps = 8;
constexpr int kDecStages = 5;
constexpr int kDecMaxW = 3;  // weights per phase
constexpr int kDecBarBytes = 512;  // stage barriers, rms scratch, abort flag
constexpr int kDecRingBytes = kDecWarps * kDecStages * kRowStageBytes;
static_assert(kDecWarps * kDecStages * 8 + 8 * 8 + 8 <= kDecBarBytes, "barrier area");

struct alignas(64) DecWeight {
    CUtensorMap tmap;  // [n rows][row bytes / 8] u64, box 32 rows x one superblock
    float *y;          // output [n] (fp32)
    int64_t n;
    int64_t pad[6];
};
static_assert(sizeof(DecWeight) == 192, "DecWeight layout");

struct DecPhase {
    int mode;          // kActPlain / kActRms / kActSwiglu
    int nbk;           // superblocks per weight row (K / 256)
    int n_w;           // weights in this phase (1..kDecMaxW)
    int w0;            // first weight in the weight table
    const float *x;    // input [K]
    const float *r;    // RMS residual (may be null) / SwiGLU up
    const float *g;    // RMS weight (may be null)
    float *h_out;      // RMS: x + r stored here when non-null
    float eps;
    int pad;
    int64_t mb_start[kDecMaxW + 1];  // prefix sums of 32-row blocks per weight
};

struct DecArgs {
    const DecPhase *ph;
    const DecWeight *w;
    int n_ph;
    int act_bytes;       // shared-memory activation region (largest phase image)
    uint8_t *act_g;      // global activation image (act_bytes)
    uint64_t *pieces;    // [warp][2][kPieceWords] stream-K piece words, zero between phases
    int *counters;       // [row block], zero between phases
    unsigned *bar;       // grid barrier counter, zero at launch
};

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Thread 0: wait until `target` CTAs have arrived at the counter (bounded).
__device__ __forceinline__ bool grid_wait(const unsigned *bar, unsigned target) {
    if (ld_acquire_gpu(bar) >= target) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (ld_acquire_gpu(bar) >= target) return true;
        if ((it & 63u) == 0 && global_timer_ns() - t0 > wait_limit_ns()) {
            atomicOr(&g_dev_error, kDevErrWaitTimeout);
            return false;
        }
    }
}

// This CTA's share of a phase's activation image (block blockIdx.x*8+warp of
// the input row, if it exists), into the global image; h_out for the blocks
// it builds.
__device__ __forceinline__ void dec_build_act(const DecPhase &P, uint8_t *img_g, double *part) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int nbk = P.nbk;
    const int64_t k = int64_t(nbk) * kQK_K;
    const int b0 = int(blockIdx.x) * kDecWarps;
    if (b0 >= nbk) return;  // CTA-uniform
    float scale = 1.0f;
    if (P.mode == kActRms) {
        float vk[kActBatch][8];
        act_rms_row<true>(P.x, P.r, k, P.eps, part, scale, vk);
    }
    const int b = b0 + warp;
    if (b >= nbk) return;
    float v[8];
    act_load_v<true>(P.mode, P.x, P.r, b, v);
    if (P.mode == kActRms && P.r && P.h_out) store8(P.h_out + int64_t(b) * kQK_K + lane * 8, v);
    act_quantize_store(P.mode, v, scale, P.g, b, 0, k, 1, img_g);
}

// The whole image from global into this CTA's shared memory (256 threads, 16 B each per step).
__device__ __forceinline__ void dec_fetch_act(const uint8_t *img_g, uint8_t *img, int bytes) {
    for (int o = int(threadIdx.x) * 16; o < bytes; o += 256 * 16)
        *reinterpret_cast<uint4 *>(img + o) = __ldcg(reinterpret_cast<const uint4 *>(img_g + o));
}

__global__ void __launch_bounds__(kDecWarps * 32, 1) decode_step_kernel(const __grid_constant__ DecArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * kDecStages;
    double *part = reinterpret_cast<double *>(smem + kDecWarps * kDecStages * 8);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(smem + kDecWarps * kDecStages * 8 + 64);
    uint8_t *act = smem + kDecBarBytes;
    uint8_t *ring = act + a.act_bytes + warp * kDecStages * kRowStageBytes;
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < kDecStages; s++) mbar_init(&bars[s], 1);
    }
    if (threadIdx.x == 0) *abort_flag = 0;
    fence_mbar_init();
    __syncthreads();

    const int64_t G = int64_t(gridDim.x) * kDecWarps;
    const int64_t g = int64_t(blockIdx.x) * kDecWarps + warp;
    const uint64_t policy = l2_policy_evict_first();
    auto share = [&](int p, int64_t &b, int64_t &e) {
        const int64_t T = a.ph[p].mb_start[a.ph[p].n_w] * a.ph[p].nbk;
        b = g * T / G;
        e = (g + 1) * T / G;
    };

    // ---- issue cursor: this warp's stages of phase ip, then the following phases ----
    int ip = 0, i_nbk = 0, i_kb = 0;
    int64_t i_it = 0, i_end = 0, i_mb = 0;
    auto seek = [&](int p) {  // first phase >= p in which this warp has work
        for (ip = p; ip < a.n_ph; ip++) {
            share(ip, i_it, i_end);
            if (i_it < i_end) break;
        }
        if (ip < a.n_ph) {
            i_nbk = a.ph[ip].nbk;
            i_mb = i_it / i_nbk;
            i_kb = int(i_it - i_mb * i_nbk);
        }
    };
    int64_t issued = 0;
    auto issue = [&](int slot) {
        if (ip >= a.n_ph) return;
        if (lane == 0) {
            const DecPhase &P = a.ph[ip];  // lane 0 only, once per stage
            int wi = 0;
#pragma unroll
            for (int q = 1; q < kDecMaxW; q++)
                if (q < P.n_w && i_mb >= P.mb_start[q]) wi = q;
            const int row0 = int((i_mb - P.mb_start[wi]) * kRowRows);
            mbar_arrive_expect_tx(&bars[slot], kRowStageBytes);
            tma_load_2d(ring + slot * kRowStageBytes, &a.w[P.w0 + wi].tmap, i_kb * (kQ4K_Bytes / 8), row0, &bars[slot],
                        policy);
        }
        issued++;
        if (++i_it == i_end) {
            seek(ip + 1);
        } else if (++i_kb == i_nbk) {
            i_kb = 0;
            i_mb++;
        }
    };
    seek(0);
    for (int s = 0; s < kDecStages; s++) issue(s);

    int64_t consumed = 0;
    int slot = 0;
    uint32_t phase_bit = 0;
    for (int p = 0; p < a.n_ph; p++) {
        const DecPhase &P = a.ph[p];
        // barrier A: every CTA has finished phase p-1 (two arrivals per phase)
        if (p > 0) {
            if (threadIdx.x == 0 && !grid_wait(a.bar, unsigned(2 * p) * gridDim.x)) *abort_flag = 1;
            __syncthreads();
            if (*abort_flag) break;
        }
        dec_build_act(P, a.act_g, part);
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            atomicAdd(a.bar, 1u);
            // barrier B: the whole image is built
            if (!grid_wait(a.bar, unsigned(2 * p + 1) * gridDim.x)) *abort_flag = 1;
        }
        __syncthreads();
        if (*abort_flag) break;
        {
            const int64_t kk = int64_t(P.nbk) * kQK_K;
            dec_fetch_act(a.act_g, act, row_act_bytes(kk, 1));
        }
        __syncthreads();

        // the compute loop's phase fields as scalars: the global table is not re-read after every store
        const int nbk = P.nbk, n_w = P.n_w, w0 = P.w0;
        const int64_t mb1 = P.mb_start[1], mb2 = P.mb_start[2], mb3 = P.mb_start[3];
        const int64_t k = int64_t(nbk) * kQK_K;
        const int8_t *xs = reinterpret_cast<const int8_t *>(act);
        const float *xd = reinterpret_cast<const float *>(act + align_up(size_t(k), 16));
        const uint8_t *xb = act + align_up(size_t(k), 16) + align_up(size_t(nbk) * 4, 16);
        int64_t c_it, c_end;
        share(p, c_it, c_end);
        const int64_t T = (n_w == 1 ? mb1 : n_w == 2 ? mb2 : mb3) * nbk;
        const RowSeg sg{G, T, g, c_it / nbk, a.pieces, a.counters};
        int64_t c_mb = c_it / nbk;
        int c_kb = int(c_it - c_mb * nbk);
        int64_t seg_start = c_it;
        float acc[1] = {0.0f};
        while (c_it < c_end) {
            if (!mbar_wait_bounded(&bars[slot], phase_bit)) {
                *abort_flag = 1;
                break;
            }
            __syncwarp();
            const uint8_t *blk = ring + slot * kRowStageBytes + lane * kQ4K_Bytes;
            const uint4 h = *reinterpret_cast<const uint4 *>(blk);
            uint4 qv[8];
#pragma unroll
            for (int i = 0; i < 8; i++) qv[i] = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * i);
            __syncwarp();
            consumed++;
            issue(slot);  // the stage is in registers: refill it (possibly with a later phase's weights)

            row_dot<1>(h, qv, xs, xd, xb, k, nbk, c_kb, acc);

            c_it++;
            if (++slot == kDecStages) {
                slot = 0;
                phase_bit ^= 1u;
            }
            const bool blk_end = (++c_kb == nbk);
            if (blk_end || c_it == c_end) {
                const int wi = (n_w > 1 && c_mb >= mb1) + (n_w > 2 && c_mb >= mb2);
                float *const wy = a.w[w0 + wi].y;
                const int64_t wn = a.w[w0 + wi].n;
                const int64_t row0 = (c_mb - (wi == 0 ? 0 : wi == 1 ? mb1 : mb2)) * kRowRows;
                row_segment_end<1>(sg, c_mb, nbk, seg_start == c_mb * nbk && blk_end, acc, wy, 0, 1, row0 + lane < wn,
                                   row0 + lane);
                acc[0] = 0.0f;
                seg_start = c_it;
                if (blk_end) {
                    c_kb = 0;
                    c_mb++;
                }
            }
        }
        __syncthreads();  // the CTA's outputs of phase p are written; the image may be rebuilt
        if (*abort_flag) break;
        if (threadIdx.x == 0) {
            __threadfence();
            atomicAdd(a.bar, 1u);
        }
    }
    // stages still in flight (normally none: the cursor ends with the last phase)
    for (int64_t u = consumed; u < issued; u++) {
        const int s = int(u % kDecStages);
        mbar_wait_bounded(&bars[s], uint32_t(u / kDecStages) & 1u);
    }
}

}  // namespace cpq
