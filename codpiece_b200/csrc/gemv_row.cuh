// gemv_row.cuh — Q4_K x Q8_K decode GEMV (M = 1..3), one lane per weight row.
//
// Same arithmetic as ggml_vec_dot_q4_K_q8_K: exact integer sub-block dots
// (dp4a), six-bit scales and mins applied as integers, fp32 per superblock.
//
// Layout. A warp owns 32 consecutive rows and walks K one superblock at a
// time; lane r holds row r's 144-byte block in registers (9 x 16-byte shared
// loads; the dense 144-byte pitch written by the TMA puts 8 consecutive rows
// in distinct bank groups, so the loads are conflict-free) and dots it with
// the activation block, which every lane reads from the same shared address
// (broadcast). Per 256 weights a lane spends ~200 instructions, ~6 warp
// instructions per block, against ~25 that the HBM stream leaves room for.
//
// Activations. The quantized activation image (act_prep.cuh, a few KB) is
// pulled into shared memory with one bulk copy right after
// griddepcontrol.wait; the weight stages were issued before that wait, so
// under programmatic dependent launch the weight stream overlaps the
// producer of the activations.
//
// Memory path and work split are those of gemv_mma.cuh: a private ring of
// 2-D TMA tensor copies per warp (box 32 rows x 1 superblock, no multicast)
// and a stream-K split of (32-row block, superblock) iterations with a
// deterministic last-arriver fix-up.
#pragma once

#include "act_prep.cuh"
#include "gemv_mma.cuh"

namespace cpq {

#ifndef CPQ_ROW_WARPS
#define CPQ_ROW_WARPS 8
#endif
#ifndef CPQ_ROW_STAGES
#define CPQ_ROW_STAGES 4
#endif

constexpr int kRowWarps = CPQ_ROW_WARPS;
constexpr int kRowStages = CPQ_ROW_STAGES;
constexpr int kRowRows = 32;
constexpr int kRowStageBytes = kRowRows * kQ4K_Bytes;  // one superblock of 32 rows
constexpr int kRowBarBytes = 128 * ((kRowWarps * kRowStages * 8 + 8 + 127) / 128);  // + the activation barrier
constexpr int kRowRingBytes = kRowWarps * kRowStages * kRowStageBytes;
constexpr int kRowMaxTokens = 3;
static_assert(kQ4K_Bytes % 128 == 16, "per-lane 16-byte row loads must hit distinct bank groups");

struct alignas(64) RowArgs {
    CUtensorMap tmap[4];  // weight i as [n rows][row bytes / 8] u64, box 32 x 18 (one superblock)
    float *y[4];
    int64_t n[4];
    int64_t y_stride[4];
    int64_t mb_start[5];  // prefix sums of 32-row blocks per weight
    int n_w;
    int nbk;
    int m;                // tokens (1..3)
    const uint8_t *act;   // activation image (act_prep.cuh), row_act_bytes(K, m) bytes
    int64_t n_warps;
    float *partials;      // [warp][2 segments][256 floats]
    int *counters;        // [row block], zero between calls
    ArOut ar;             // on: weight 0's output is all-reduced through this channel
};

// Lane = row: this lane's 144-byte superblock (h = header, qv = nibbles)
// against block kb of the activation image, MT tokens, accumulated into acc
// (ggml_vec_dot_q4_K_q8_K's integer sub-block dots, fp32 per superblock).
template <int MT>
__device__ __forceinline__ void row_dot(const uint4 &h, const uint4 (&qv)[8], const int8_t *xs, const float *xd,
                                        const uint8_t *xb, int64_t k, int nbk, int kb, float (&acc)[MT]) {
    const uint32_t sca = h.y & 0x3f3f3f3fu, scb = (h.w & 0x0f0f0f0fu) | ((h.y >> 2) & 0x30303030u);
    const uint32_t mna = h.z & 0x3f3f3f3fu, mnb = ((h.w >> 4) & 0x0f0f0f0fu) | ((h.z >> 2) & 0x30303030u);
    const float dw = half_bits_to_float(h.x), dm = half_bits_to_float(h.x >> 16);
    int isc[MT];
#pragma unroll
    for (int t = 0; t < MT; t++) isc[t] = 0;
#pragma unroll
    for (int jj = 0; jj < 4; jj++) {
        const uint4 wa = qv[2 * jj], wb = qv[2 * jj + 1];
        const uint32_t w[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
        const uint32_t sw = jj < 2 ? sca : scb;
        const int slo = byte_of(sw, (2 * jj) & 3), shi = byte_of(sw, (2 * jj + 1) & 3);
#pragma unroll
        for (int t = 0; t < MT; t++) {
            const int4 *xp = reinterpret_cast<const int4 *>(xs + t * k + kb * kQK_K + 64 * jj);
            const int4 x0 = xp[0], x1 = xp[1], x2 = xp[2], x3 = xp[3];
            const int xl[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            const int xh[8] = {x2.x, x2.y, x2.z, x2.w, x3.x, x3.y, x3.z, x3.w};
            int dl = 0, dh = 0;
#pragma unroll
            for (int i = 0; i < 8; i++) {
                dl = __dp4a(int(w[i] & 0x0f0f0f0fu), xl[i], dl);
                dh = dp4a_us(w[i] & 0xf0f0f0f0u, xh[i], dh);  // 16 * q_hi
            }
            isc[t] += slo * dl + shi * (dh >> 4);
        }
    }
#pragma unroll
    for (int t = 0; t < MT; t++) {
        const uint4 bsv = *reinterpret_cast<const uint4 *>(xb + (size_t(t) * nbk + kb) * 16);
        const int imn = 256 * (__dp4a(int(mna), int(bsv.z), 0) + __dp4a(int(mnb), int(bsv.w), 0)) +
                        dp4a_uu(mna, bsv.x, dp4a_uu(mnb, bsv.y, 0));
        const float dx = xd[t * nbk + kb];
        acc[t] += (dw * dx) * float(isc[t]) - (dm * dx) * float(imn);
    }
}

// End of a warp's segment of 32-row block mb (its last superblock, or the end
// of its stream-K share). A segment covering the whole row block stores Y;
// otherwise the warp parks its partial sums and the last of the row block's
// npieces owners (atomic counter, acq_rel) adds them in K order, stores Y and
// resets the counter. The warp's slot is 0 for the row block it starts in,
// 1 for any later one (a share spans at most two partial row blocks).
struct RowSeg {
    int64_t G, T;          // warps, iterations of the whole split
    int64_t g;             // this warp
    int64_t first_mb;      // the row block this warp's share starts in
    float *partials;       // [warp][2][256]
    int *counters;         // [row block]
};

// The finished values of one 32-row block (lane = row): stored in Y, or,
// for an all-reduced output (ar non-null, sequence number ar_e), written to
// slot (ar_e & 1, rank) of every rank's receive buffer over NVLink as LL
// words (ar_e << 32 | value), one 64-bit store each: nothing else to publish.
template <int MT>
__device__ __forceinline__ void row_block_out(const float (&v)[MT], float *y, int64_t y_stride, int m, bool row_ok,
                                              int64_t row, const ArOut *ar, unsigned ar_e) {
    if (!ar) {
#pragma unroll
        for (int t = 0; t < MT; t++)
            if (t < m && row_ok) y[size_t(t) * y_stride + row] = v[t];
        return;
    }
    const int64_t slot = (int64_t(ar_e & 1u) * ar->world + ar->rank) * ar->n_max;
    for (int d = 0; d < ar->world; d++) {
        uint64_t *dst = ar->peer[d] + slot;
#pragma unroll
        for (int t = 0; t < MT; t++)
            if (t < m && row_ok)
                st_relaxed_sys_u64(dst + int64_t(t) * ar->n + row, (uint64_t(ar_e) << 32) | __float_as_uint(v[t]));
    }
}

template <int MT>
__device__ __forceinline__ void row_segment_end(const RowSeg &sg, int64_t mb, int nbk, bool whole, float (&acc)[MT],
                                                float *y, int64_t y_stride, int m, bool row_ok, int64_t row,
                                                const ArOut *ar = nullptr, unsigned ar_e = 0u) {
    const int lane = threadIdx.x & 31;
    if (whole) {
        row_block_out<MT>(acc, y, y_stride, m, row_ok, row, ar, ar_e);
        return;
    }
    const int64_t first = owner_warp(mb * nbk, sg.G, sg.T);
    const int64_t last = owner_warp(mb * nbk + nbk - 1, sg.G, sg.T);
    const int npieces = int(last - first + 1);
    const int my_slot = (mb == sg.first_mb) ? 0 : 1;
    float *pp = sg.partials + (size_t(sg.g) * 2 + my_slot) * 256;
#pragma unroll
    for (int t = 0; t < MT; t++) pp[lane * 4 + t] = acc[t];
    __syncwarp();
    int old = 0;
    if (lane == 0) old = atom_add_acq_rel_gpu(&sg.counters[mb], 1);
    old = __shfl_sync(0xffffffffu, old, 0);
    __syncwarp();
    if (old == npieces - 1) {
        // Piece p > 0 starts inside this row block (slot 0); piece 0 uses slot 1
        // when its share began in an earlier row block. The loads of a batch of
        // pieces are issued together, then added in piece order.
        const int first_slot = (first * sg.T / sg.G < mb * nbk) ? 1 : 0;
        constexpr int kBatch = 8;
        float sum[MT];
#pragma unroll
        for (int t = 0; t < MT; t++) sum[t] = 0.0f;
        for (int p0 = 0; p0 < npieces; p0 += kBatch) {
            float pv[kBatch][MT];
#pragma unroll
            for (int j = 0; j < kBatch; j++) {
                if (p0 + j < npieces) {
                    const int sl = (p0 + j == 0) ? first_slot : 0;
                    const float *q = sg.partials + (size_t(first + p0 + j) * 2 + sl) * 256;
#pragma unroll
                    for (int t = 0; t < MT; t++) pv[j][t] = __ldcg(q + lane * 4 + t);
                }
            }
#pragma unroll
            for (int j = 0; j < kBatch; j++) {
                if (p0 + j < npieces) {
#pragma unroll
                    for (int t = 0; t < MT; t++) sum[t] += pv[j][t];
                }
            }
        }
        if (lane == 0) sg.counters[mb] = 0;
        row_block_out<MT>(sum, y, y_stride, m, row_ok, row, ar, ar_e);
    }
}

template <int MT>
__global__ void __launch_bounds__(kRowWarps * 32, 1) gemv_q4k_row_kernel(const __grid_constant__ RowArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nbk = a.nbk;
    const int64_t k = int64_t(nbk) * kQK_K;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * kRowStages;
    uint64_t *act_bar = reinterpret_cast<uint64_t *>(smem) + kRowWarps * kRowStages;
    int8_t *xs = reinterpret_cast<int8_t *>(smem + kRowBarBytes);
    float *xd = reinterpret_cast<float *>(smem + kRowBarBytes + align_up(size_t(MT) * size_t(k), 16));
    uint8_t *xb = reinterpret_cast<uint8_t *>(xd) + align_up(size_t(MT) * nbk * 4, 16);
    uint8_t *ring = smem + kRowBarBytes + row_act_bytes(k, MT) + warp * kRowStages * kRowStageBytes;
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < kRowStages; s++) mbar_init(&bars[s], 1);
        if (warp == 0) mbar_init(act_bar, 1);
        fence_mbar_init();
    }
    __syncthreads();

    const int64_t T = a.mb_start[a.n_w] * nbk;
    const int64_t G = a.n_warps;
    const int64_t g = int64_t(blockIdx.x) * kRowWarps + warp;
    const bool active = g < G;
    const int64_t it_begin = active ? g * T / G : 0, it_end = active ? (g + 1) * T / G : 0;
    const uint64_t policy = l2_policy_evict_first();

    auto weight_of = [&](int64_t mb) {
        int wi = 0;
#pragma unroll
        for (int q = 1; q < 4; q++)
            if (q < a.n_w && mb >= a.mb_start[q]) wi = q;
        return wi;
    };

    int64_t p_it = it_begin, p_mb = it_begin / nbk;
    int p_kb = int(it_begin - p_mb * nbk);
    auto issue = [&](int slot) {
        if (lane == 0) {
            const int wi = weight_of(p_mb);
            const int row0 = int((p_mb - a.mb_start[wi]) * kRowRows);
            mbar_arrive_expect_tx(&bars[slot], kRowStageBytes);
            tma_load_2d(ring + slot * kRowStageBytes, &a.tmap[wi], p_kb * (kQ4K_Bytes / 8), row0, &bars[slot], policy);
        }
        p_it++;
        if (++p_kb == nbk) {
            p_kb = 0;
            p_mb++;
        }
    };
    for (int j = 0; j < kRowStages && p_it < it_end; j++) issue(j);

    // ---- activations: one bulk copy of the image the previous kernel wrote ----
    pdl_wait();
    const uint32_t act_bytes = uint32_t(row_act_bytes(k, MT));
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(act_bar, act_bytes);
        bulk_g2s(xs, a.act, act_bytes, act_bar);
    }
    if (!mbar_wait_bounded(act_bar, 0)) {
        // error recorded in the device word: wait (bounded) for this warp's weight copies, then leave
        for (int64_t j = 0; j < p_it - it_begin; j++) mbar_wait_bounded(&bars[j], 0);
        return;
    }
    pdl_launch_dependents();
    if (!active) return;
    const ArOut *arp = a.ar.on ? &a.ar : nullptr;
    const unsigned ar_e = a.ar.on ? *a.ar.seq + 1u : 0u;  // this call's sequence number

    float acc[MT];
#pragma unroll
    for (int t = 0; t < MT; t++) acc[t] = 0.0f;
    int64_t c_it = it_begin, c_mb = it_begin / nbk;
    int c_kb = int(it_begin - c_mb * nbk);
    int64_t seg_start = it_begin;
    int slot = 0;
    uint32_t phase = 0;
    const RowSeg sg{G, T, g, it_begin / nbk, a.partials, a.counters};
    while (c_it < it_end) {
        if (!mbar_wait_bounded(&bars[slot], phase)) {
            // error recorded in the device word: wait (bounded) for this warp's other copies, then leave
            for (int k2 = 1; k2 < kRowStages && p_it > c_it + k2; k2++)
                mbar_wait_bounded(&bars[(slot + k2) % kRowStages], phase ^ uint32_t(slot + k2 >= kRowStages));
            return;
        }
        __syncwarp();
        const uint8_t *blk = ring + slot * kRowStageBytes + lane * kQ4K_Bytes;
        const uint4 h = *reinterpret_cast<const uint4 *>(blk);
        uint4 qv[8];
#pragma unroll
        for (int i = 0; i < 8; i++) qv[i] = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * i);
        __syncwarp();
        if (p_it < it_end) issue(slot);  // the stage is in registers: refill it now

        row_dot<MT>(h, qv, xs, xd, xb, k, nbk, c_kb, acc);

        c_it++;
        if (++slot == kRowStages) {
            slot = 0;
            phase ^= 1u;
        }
        const bool blk_end = (++c_kb == nbk);
        if (blk_end || c_it == it_end) {
            const int wi = weight_of(c_mb);
            const int64_t row0 = (c_mb - a.mb_start[wi]) * kRowRows;
            const bool row_ok = row0 + lane < a.n[wi];
            row_segment_end<MT>(sg, c_mb, nbk, seg_start == c_mb * nbk && blk_end, acc, a.y[wi], a.y_stride[wi], a.m,
                                row_ok, row0 + lane, arp, ar_e);
#pragma unroll
            for (int t = 0; t < MT; t++) acc[t] = 0.0f;
            seg_start = c_it;
            if (blk_end) {
                c_kb = 0;
                c_mb++;
            }
        }
    }
}

}  // namespace cpq
