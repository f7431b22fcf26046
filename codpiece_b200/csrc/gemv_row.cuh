// gemv_row.cuh — Q4_K x Q8_K decode GEMV (M = 1..3), one lane per weight row.
//
// Same arithmetic as ggml_vec_dot_q4_K_q8_K: exact integer sub-block dots
// (dp4a), six-bit scales and mins applied as integers, fp32 per superblock.
//
// Layout. A stage is one superblock of 32 consecutive rows; lane r holds row
// r's 144-byte block in registers (9 x 16-byte shared loads; the dense
// 144-byte pitch written by the TMA puts 8 consecutive rows in distinct bank
// groups, so the loads are conflict-free) and dots it with the activation
// block, which every lane reads from the same shared address (broadcast).
//
// Activations. The quantized activation image (act_prep.cuh, a few KB) is
// pulled into shared memory with one bulk copy right after
// griddepcontrol.wait; the first weight stages were issued before that
// wait, so under programmatic dependent launch the weight stream overlaps
// the producer of the activations.
//
// Memory path: a private ring of 2-D TMA tensor copies per warp (box 32 rows
// x 1 superblock, no multicast). The work split (a contiguous range of
// (row block, superblock) iterations per CTA, swept by its warps together)
// is described above the kernel.
#pragma once

#include "act_prep.cuh"
#include "gemv_mma.cuh"

namespace cpq {

#ifndef CPQ_ROW_WARPS
#define CPQ_ROW_WARPS 8
#endif
// Ring depth per warp and how much of it is issued before griddepcontrol.wait
// (measured on B200, config-2 shapes: 3 and 2 beat 4 and 4, whose early
// copies compete with the previous kernel's last stages).
#ifndef CPQ_ROW_STAGES
#define CPQ_ROW_STAGES 3
#endif
#ifndef CPQ_ROW_PRE
#define CPQ_ROW_PRE 2
#endif

constexpr int kRowWarps = CPQ_ROW_WARPS;
constexpr int kRowStages = CPQ_ROW_STAGES;
constexpr int kRowPre = CPQ_ROW_PRE < CPQ_ROW_STAGES ? CPQ_ROW_PRE : CPQ_ROW_STAGES;
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
    uint64_t *pieces;     // [CTA][warp][kPieceWords] tail-cut words, zero between calls
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
            // four independent dp4a chains of depth 4 (not two of depth 8)
            int dl0 = 0, dl1 = 0, dh0 = 0, dh1 = 0;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                dl0 = __dp4a(int(w[i] & 0x0f0f0f0fu), xl[i], dl0);
                dh0 = dp4a_us(w[i] & 0xf0f0f0f0u, xh[i], dh0);  // 16 * q_hi
                dl1 = __dp4a(int(w[i + 4] & 0x0f0f0f0fu), xl[i + 4], dl1);
                dh1 = dp4a_us(w[i + 4] & 0xf0f0f0f0u, xh[i + 4], dh1);
            }
            isc[t] += slo * (dl0 + dl1) + shi * ((dh0 + dh1) >> 4);
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

// Stream-K pieces. A row block cut between warps is summed by the last of its
// npieces owners to arrive. A piece is published as flagged words, one 64-bit
// word (kPieceFlag << 32 | float bits) per lane and token, stored without a
// fence; the owner then bumps the row block's counter with a relaxed atomic.
// The last arriver (counter value npieces - 1) waits, bounded, for each word's
// flag, adds the pieces in K order (deterministic), clears the words and the
// counter (both are zero between calls) and stores the row block's outputs.
// Nothing orders the stores of a piece before its counter increment, and
// nothing has to: the reader waits on the words themselves, and their owner
// has already issued them. A warp's slot is 0 for the row block its share
// starts in, 1 for a later one (a share cuts at most two row blocks).
constexpr uint32_t kPieceFlag = 0x9a5e0001u;
constexpr int kPieceWords = 4 * 32;  // one slot: [token 0..3][lane]

struct RowSeg {
    int64_t G, T;          // warps, iterations of the whole split
    int64_t g;             // this warp
    int64_t first_mb;      // the row block this warp's share starts in
    uint64_t *pieces;      // [warp][2 slots][kPieceWords] flagged words, zero between calls
    int *counters;         // [row block], zero between calls
};

// The finished values of one 32-row block (lane = row): stored in Y, or,
// for an all-reduced output (ar non-null, sequence number ar_e), written to
// slot (ar_e % kArSlots, rank) of every rank's receive buffer over NVLink as LL
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
    const int64_t slot = (int64_t(ar_e % kArSlots) * ar->world + ar->rank) * ar->n_max;
    for (int d = 0; d < ar->world; d++) {
        uint64_t *dst = ar->peer[d] + slot;
#pragma unroll
        for (int t = 0; t < MT; t++)
            if (t < m && row_ok)
                st_relaxed_sys_u64(dst + int64_t(t) * ar->n + row, (uint64_t(ar_e) << 32) | __float_as_uint(v[t]));
    }
}

// Publishes this warp's piece of row block mb. Returns, in lane 0, the
// counter value before the increment; the caller may hold it unread (the
// warp does not stall on the atomic until row_piece_finish reads it).
template <int MT>
__device__ __forceinline__ int row_piece_publish(const RowSeg &sg, int64_t mb, const float (&acc)[MT]) {
    const int lane = threadIdx.x & 31;
    uint64_t *pw = sg.pieces + (size_t(sg.g) * 2 + (mb == sg.first_mb ? 0 : 1)) * kPieceWords;
#pragma unroll
    for (int t = 0; t < MT; t++)
        st_relaxed_gpu_u64(pw + t * 32 + lane, (uint64_t(kPieceFlag) << 32) | __float_as_uint(acc[t]));
    int old = 0;
    if (lane == 0) old = atom_add_relaxed_gpu(&sg.counters[mb], 1);
    return old;
}

// The other half: if this warp was the last of row block mb's owners to
// arrive (old_lane0 from row_piece_publish), sum the pieces and store the row
// block. The first batch of piece words is loaded before the counter value is
// read, so a pending atomic and those loads overlap.
template <int MT>
__device__ __forceinline__ void row_piece_finish(const RowSeg &sg, int64_t mb, int nbk, int old_lane0, float *y,
                                                 int64_t y_stride, int m, bool row_ok, int64_t row, const ArOut *ar,
                                                 unsigned ar_e) {
    const int lane = threadIdx.x & 31;
    const int64_t first = owner_warp(mb * nbk, sg.G, sg.T);
    const int64_t last = owner_warp(mb * nbk + nbk - 1, sg.G, sg.T);
    const int npieces = int(last - first + 1);
    // Piece p > 0 starts inside this row block (slot 0); piece 0 uses slot 1
    // when its owner's share began in an earlier row block.
    const int first_slot = (first * sg.T / sg.G < mb * nbk) ? 1 : 0;
    auto words = [&](int p) {
        return sg.pieces + (size_t(first + p) * 2 + (p == 0 ? first_slot : 0)) * kPieceWords + lane;
    };
    constexpr int kBatch = MT == 1 ? 8 : 4;
    uint64_t w[kBatch][MT];
#pragma unroll
    for (int j = 0; j < kBatch; j++)
        if (j < npieces) {
#pragma unroll
            for (int t = 0; t < MT; t++) w[j][t] = ld_relaxed_gpu_u64(words(j) + t * 32);
        }
    if (__shfl_sync(0xffffffffu, old_lane0, 0) != npieces - 1) return;
    float sum[MT];
#pragma unroll
    for (int t = 0; t < MT; t++) sum[t] = 0.0f;
    for (int p0 = 0; p0 < npieces; p0 += kBatch) {
        if (p0 > 0) {
#pragma unroll
            for (int j = 0; j < kBatch; j++)
                if (p0 + j < npieces) {
#pragma unroll
                    for (int t = 0; t < MT; t++) w[j][t] = ld_relaxed_gpu_u64(words(p0 + j) + t * 32);
                }
        }
#pragma unroll
        for (int j = 0; j < kBatch; j++)
            if (p0 + j < npieces) {
                uint64_t *q = words(p0 + j);
#pragma unroll
                for (int t = 0; t < MT; t++) {
                    const uint64_t v =
                        uint32_t(w[j][t] >> 32) == kPieceFlag ? w[j][t] : flagged_word_gpu(q + t * 32, kPieceFlag);
                    sum[t] += __uint_as_float(uint32_t(v));
                    st_relaxed_gpu_u64(q + t * 32, 0ull);
                }
            }
    }
    if (lane == 0) sg.counters[mb] = 0;
    row_block_out<MT>(sum, y, y_stride, m, row_ok, row, ar, ar_e);
}

// Publish and finish in one go (callers without later work to overlap).
template <int MT>
__device__ __forceinline__ void row_segment_end(const RowSeg &sg, int64_t mb, int nbk, bool whole, float (&acc)[MT],
                                                float *y, int64_t y_stride, int m, bool row_ok, int64_t row,
                                                const ArOut *ar = nullptr, unsigned ar_e = 0u) {
    if (whole) {
        row_block_out<MT>(acc, y, y_stride, m, row_ok, row, ar, ar_e);
        return;
    }
    const int old = row_piece_publish<MT>(sg, mb, acc);
    row_piece_finish<MT>(sg, mb, nbk, old, y, y_stride, m, row_ok, row, ar, ar_e);
}

// ---- the decode GEMV ---------------------------------------------------------
//
// Work split. The iteration space is (32-row block, superblock) in row-block
// order, T = row blocks x nbk. CTA c of C takes the contiguous range
// [c*T/C, (c+1)*T/C); the host keeps C <= T / nbk, so every range holds at
// least nbk iterations and a row block is cut between at most two CTAs. The
// CTA's warps sweep the range interleaved (list position j goes to warp
// j % kRowWarps) in this order: first the head of the row block the range
// ends in (its "tail cut", whose rest belongs to CTA c+1), then the range from
// its start. So each CTA publishes its tail cut within its first stages, and
// finishes the row block its range starts in (CTA c-1's tail cut plus its
// own part) after having streamed that part, by which time CTA c-1's part
// is normally long published: no CTA waits at the end of its range.
//
// Inside a CTA, a warp's part of a row block goes to a shared-memory ring of
// kRowRedSlots row-block slots; the last warp to arrive (shared-memory atomic)
// sums the parts in warp order and stores the block. A tail cut travels as
// flagged words (kPieceFlag << 32 | float bits) to the piece region, slot
// [CTA][warp]. The row block the range starts in, when it is CTA c-1's tail
// cut, keeps its parts in a slot of its own and is finished by the warp that
// holds the range's last list position, after its last stage: that warp
// issues the loads of CTA c-1's words one stage ahead, waits (bounded) on each
// word's flag, adds them in warp order ahead of this CTA's parts, and clears
// them (the words are zero between calls). The grid is at most one CTA per SM (one CTA fits an SM),
// so every CTA whose words another waits for is resident. Sums run in the
// same order for the same shape and grid: results are deterministic.
constexpr int kRowRedSlots = 4;

__host__ __device__ constexpr int row_red_bytes(int mt) {  // ring slots + the cut's slot, counters, generations
    return int(align_up(size_t(kRowRedSlots + 1) * kRowWarps * mt * 32 * 4 + (2 * kRowRedSlots + 1) * 4, 128));
}

// Position in the CTA's list, with the iteration it stands for.
struct RowCursor {
    int64_t j, it, mb;
    int kb;
};

// The shared-memory word at p once it equals v (bounded; gives up, setting
// the device error word, after the wait limit or once another wait gave up).
__device__ __forceinline__ bool smem_wait_eq(const int *p, int v) {
    if (*reinterpret_cast<const volatile int *>(p) == v) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (*reinterpret_cast<const volatile int *>(p) == v) return true;
        if ((it & 63u) == 0 && ((*reinterpret_cast<volatile uint32_t *>(&g_dev_error) & kDevErrWaitTimeout) ||
                                global_timer_ns() - t0 > wait_limit_ns())) {
            atomicOr(&g_dev_error, kDevErrWaitTimeout);
            return false;
        }
    }
}

template <int MT>
__global__ void __launch_bounds__(kRowWarps * 32, 1) gemv_q4k_row_kernel(const __grid_constant__ RowArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nbk = a.nbk;
    const int64_t k = int64_t(nbk) * kQK_K;
    const int act_sz = row_act_bytes(k, MT);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * kRowStages;
    uint64_t *act_bar = reinterpret_cast<uint64_t *>(smem) + kRowWarps * kRowStages;
    int8_t *xs = reinterpret_cast<int8_t *>(smem + kRowBarBytes);
    float *xd = reinterpret_cast<float *>(smem + kRowBarBytes + align_up(size_t(MT) * size_t(k), 16));
    uint8_t *xb = reinterpret_cast<uint8_t *>(xd) + align_up(size_t(MT) * nbk * 4, 16);
    uint8_t *ring = smem + kRowBarBytes + act_sz + warp * kRowStages * kRowStageBytes;
    // [slot 0..kRowRedSlots][warp][MT][32]: ring slots, then the cut row block's slot
    float *red = reinterpret_cast<float *>(smem + kRowBarBytes + act_sz + kRowRingBytes);
    int *red_cnt = reinterpret_cast<int *>(red + (kRowRedSlots + 1) * kRowWarps * MT * 32);  // [kRowRedSlots + 1]
    int *red_gen = red_cnt + kRowRedSlots + 1;
    if (threadIdx.x <= kRowRedSlots) red_cnt[threadIdx.x] = 0;
    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < kRowStages; s++) mbar_init(&bars[s], 1);
        if (warp == 0) mbar_init(act_bar, 1);
        fence_mbar_init();
    }
    __syncthreads();

    const int64_t T = a.mb_start[a.n_w] * nbk;
    const int64_t C = gridDim.x, c = blockIdx.x;
    const int64_t lo = c * T / C, hi = (c + 1) * T / C, L = hi - lo;
    const int64_t b0 = (hi % nbk) ? (hi - hi % nbk > lo ? hi - hi % nbk : lo) : hi;  // tail cut [b0, hi)
    const int64_t LB = hi - b0;
    const int64_t mbA = lo / nbk;          // the row block the range starts in
    const bool cutA = (lo % nbk) != 0;     // ... and whose head is CTA c-1's tail cut
    const uint64_t policy = l2_policy_evict_first();
    // slot s first holds row block s of the range (row block 0 skips the ring when it is the cut)
    if (threadIdx.x < kRowRedSlots) red_gen[threadIdx.x] = (threadIdx.x == 0 && cutA) ? kRowRedSlots : int(threadIdx.x);
    __syncthreads();

    auto weight_of = [&](int64_t mb) {
        int wi = 0;
#pragma unroll
        for (int q = 1; q < 4; q++)
            if (q < a.n_w && mb >= a.mb_start[q]) wi = q;
        return wi;
    };
    auto seek = [&](RowCursor &r, int64_t j) {
        r.j = j;
        if (j < L) {
            r.it = j < LB ? b0 + j : lo + (j - LB);
            r.mb = r.it / nbk;
            r.kb = int(r.it - r.mb * nbk);
        }
    };
    auto advance = [&](RowCursor &r) {
        const int64_t j = r.j + kRowWarps;
        if (j >= L) {
            r.j = j;
        } else if (r.j < LB && j >= LB) {
            seek(r, j);
        } else {
            r.j = j;
            r.it += kRowWarps;
            r.kb += kRowWarps;
            while (r.kb >= nbk) {
                r.kb -= nbk;
                r.mb++;
            }
        }
    };

    RowCursor pc;
    seek(pc, warp);
    int issued = 0;
    auto issue = [&](int slot) {
        if (lane == 0) {
            const int wi = weight_of(pc.mb);
            const int row0 = int((pc.mb - a.mb_start[wi]) * kRowRows);
            mbar_arrive_expect_tx(&bars[slot], kRowStageBytes);
            tma_load_2d(ring + slot * kRowStageBytes, &a.tmap[wi], pc.kb * (kQ4K_Bytes / 8), row0, &bars[slot], policy);
        }
        issued++;
        advance(pc);
    };
    for (int s = 0; s < kRowPre && pc.j < L; s++) issue(s);

    // ---- activations: one bulk copy of the image the previous kernel wrote ----
    pdl_wait();
    const uint32_t act_bytes = uint32_t(act_sz);
    if (threadIdx.x == 0) {
        mbar_arrive_expect_tx(act_bar, act_bytes);
        bulk_g2s(xs, a.act, act_bytes, act_bar);
    }
    if (!mbar_wait_bounded(act_bar, 0)) {
        // error recorded in the device word: wait (bounded) for this warp's weight copies, then leave
        for (int s = 0; s < issued; s++) mbar_wait_bounded(&bars[s], 0);
        return;
    }
    pdl_launch_dependents();
    for (int s = issued; s < kRowStages && pc.j < L; s++) issue(s);  // the rest of the ring
    const ArOut *arp = a.ar.on ? &a.ar : nullptr;
    const unsigned ar_e = a.ar.on ? *a.ar.seq + 1u : 0u;  // this call's sequence number

    auto store_block = [&](int64_t mb, const float (&v)[MT]) {
        const int wi = weight_of(mb);
        const int64_t row0 = (mb - a.mb_start[wi]) * kRowRows;
        row_block_out<MT>(v, a.y[wi], a.y_stride[wi], a.m, row0 + lane < a.n[wi], row0 + lane, arp, ar_e);
    };
    // Row block mbA when it is the cut: CTA c-1's tail cut (its warps
    // w < min(lo % nbk, kRowWarps)) ahead of this CTA's parts. Run by warp fw
    // after its last stage; pre[] holds the first kPre warps' words, loaded
    // one stage earlier (a word without its flag yet is waited for here).
    constexpr int kPre = 8;
    const int fw = int((L - 1) % kRowWarps);
    const int nw_prev = int(lo % nbk < kRowWarps ? lo % nbk : kRowWarps);
    uint64_t *prev = a.pieces + size_t(c - 1) * kRowWarps * kPieceWords + lane;
    auto finish_cut = [&](const uint64_t (&pre)[kPre][MT]) -> bool {
        const int64_t la = ((mbA + 1) * nbk < b0 ? (mbA + 1) * nbk : b0) - lo;  // list positions of this CTA's part
        const int len = int(la < kRowWarps ? la : kRowWarps);
        if (!smem_wait_eq(&red_cnt[kRowRedSlots], len)) return false;
        __threadfence_block();
        float s[MT];
#pragma unroll
        for (int t = 0; t < MT; t++) s[t] = 0.0f;
        for (int u0 = 0; u0 < nw_prev; u0 += kPre) {
            uint64_t w[kPre][MT];
#pragma unroll
            for (int u = 0; u < kPre; u++)
                if (u0 + u < nw_prev) {
#pragma unroll
                    for (int t = 0; t < MT; t++)
                        w[u][t] = u0 == 0 ? pre[u][t] : ld_relaxed_gpu_u64(prev + (u0 + u) * kPieceWords + t * 32);
                }
#pragma unroll
            for (int u = 0; u < kPre; u++)
                if (u0 + u < nw_prev) {
#pragma unroll
                    for (int t = 0; t < MT; t++) {
                        uint64_t *p = prev + (u0 + u) * kPieceWords + t * 32;
                        const uint64_t v =
                            uint32_t(w[u][t] >> 32) == kPieceFlag ? w[u][t] : flagged_word_gpu(p, kPieceFlag);
                        s[t] += __uint_as_float(uint32_t(v));
                        st_relaxed_gpu_u64(p, 0ull);
                    }
                }
        }
        const int p0 = int(LB % kRowWarps);  // this CTA's parts, in warp order
#pragma unroll
        for (int u = 0; u < kRowWarps; u++)
            if (((u - p0 + kRowWarps) % kRowWarps) < len) {
                const float *src = red + (kRowRedSlots * kRowWarps + u) * MT * 32;
#pragma unroll
                for (int t = 0; t < MT; t++) s[t] += src[t * 32 + lane];
            }
        store_block(mbA, s);
        return true;
    };
    // This warp's part of row block mb (in [lo, b0)) is done.
    auto arrive = [&](int64_t mb, const float (&part)[MT]) -> bool {
        const int64_t s_it = mb * nbk > lo ? mb * nbk : lo;
        const int64_t e_it = (mb + 1) * nbk < b0 ? (mb + 1) * nbk : b0;
        const int len = int(e_it - s_it < kRowWarps ? e_it - s_it : kRowWarps);  // warps holding a part
        const int q = int(mb - mbA);
        if (cutA && q == 0) {  // the cut's own slot; warp fw finishes it at the end
            float *mine = red + (kRowRedSlots * kRowWarps + warp) * MT * 32;
#pragma unroll
            for (int t = 0; t < MT; t++) mine[t * 32 + lane] = part[t];
            __syncwarp();
            if (lane == 0) {
                __threadfence_block();
                atomicAdd(&red_cnt[kRowRedSlots], 1);
            }
            return true;
        }
        const int s = q % kRowRedSlots;
        // slots pass from row block q to q + kRowRedSlots in order, also when
        // a row block has a single part and needs no slot
        if (!smem_wait_eq(&red_gen[s], q)) return false;
        if (len == 1) {
            __syncwarp();
            if (lane == 0) *reinterpret_cast<volatile int *>(&red_gen[s]) = q + kRowRedSlots;
            store_block(mb, part);
            return true;
        }
        float *mine = red + (s * kRowWarps + warp) * MT * 32;
#pragma unroll
        for (int t = 0; t < MT; t++) mine[t * 32 + lane] = part[t];
        __syncwarp();
        int old = 0;
        if (lane == 0) {
            __threadfence_block();
            old = atomicAdd(&red_cnt[s], 1);
        }
        old = __shfl_sync(0xffffffffu, old, 0);
        if (old != len - 1) return true;
        __threadfence_block();
        // parts in warp order; warp u holds one iff its residue is among the
        // len consecutive list positions starting at p0
        const int p0 = int((LB + (s_it - lo)) % kRowWarps);
        float sum[MT];
#pragma unroll
        for (int t = 0; t < MT; t++) sum[t] = 0.0f;
#pragma unroll
        for (int u = 0; u < kRowWarps; u++)
            if (((u - p0 + kRowWarps) % kRowWarps) < len) {
                const float *src = red + (s * kRowWarps + u) * MT * 32;
#pragma unroll
                for (int t = 0; t < MT; t++) sum[t] += src[t * 32 + lane];
            }
        __syncwarp();
        if (lane == 0) {
            red_cnt[s] = 0;
            __threadfence_block();
            *reinterpret_cast<volatile int *>(&red_gen[s]) = q + kRowRedSlots;  // the slot is free again
        }
        store_block(mb, sum);
        return true;
    };

    float acc[MT];
#pragma unroll
    for (int t = 0; t < MT; t++) acc[t] = 0.0f;
    RowCursor cc;
    seek(cc, warp);
    int slot = 0;
    uint32_t phase = 0;
    int consumed = 0;
    // After an error (recorded in the device word): wait, bounded, for this
    // warp's copies still in flight (stages consumed+skip .. issued-1), then leave.
    auto drain = [&](int skip) {
        for (int k2 = skip; k2 < kRowStages && issued > consumed + k2; k2++)
            mbar_wait_bounded(&bars[(slot + k2) % kRowStages], phase ^ uint32_t(slot + k2 >= kRowStages));
    };
    uint64_t pre[kPre][MT];
    while (cc.j < L) {
        if (cutA && warp == fw && cc.j + kRowWarps >= L) {  // the last stage of the finisher: load CTA c-1's words
#pragma unroll
            for (int u = 0; u < kPre; u++)
                if (u < nw_prev) {
#pragma unroll
                    for (int t = 0; t < MT; t++) pre[u][t] = ld_relaxed_gpu_u64(prev + u * kPieceWords + t * 32);
                }
        }
        if (!mbar_wait_bounded(&bars[slot], phase)) {
            drain(1);
            return;
        }
        __syncwarp();
        const uint8_t *blk = ring + slot * kRowStageBytes + lane * kQ4K_Bytes;
        const uint4 h = *reinterpret_cast<const uint4 *>(blk);
        uint4 qv[8];
#pragma unroll
        for (int i = 0; i < 8; i++) qv[i] = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * i);
        __syncwarp();
        consumed++;
        if (pc.j < L) issue(slot);  // the stage is in registers: refill it now

        row_dot<MT>(h, qv, xs, xd, xb, k, nbk, cc.kb, acc);

        if (++slot == kRowStages) {
            slot = 0;
            phase ^= 1u;
        }
        const int64_t mb = cc.mb;
        const bool in_tail = cc.j < LB;
        advance(cc);
        if (cc.j >= L || cc.mb != mb) {  // this warp's part of row block mb is complete
            if (in_tail) {
                uint64_t *p = a.pieces + (size_t(c) * kRowWarps + warp) * kPieceWords + lane;
#pragma unroll
                for (int t = 0; t < MT; t++)
                    st_relaxed_gpu_u64(p + t * 32, (uint64_t(kPieceFlag) << 32) | __float_as_uint(acc[t]));
            } else if (!arrive(mb, acc)) {
                drain(0);
                return;
            }
#pragma unroll
            for (int t = 0; t < MT; t++) acc[t] = 0.0f;
        }
    }
    if (cutA && warp == fw) finish_cut(pre);  // on a give-up the error is recorded; nothing is in flight
}

}  // namespace cpq
