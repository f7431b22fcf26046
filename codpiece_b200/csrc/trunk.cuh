// trunk.cuh — the decode trunk of one rank as one persistent kernel.
//
// A batch-1 decode step streams every weight of the trunk once (qwen35.rs:
// 2554-2786 per layer: rms -> q/k/v, o, rms -> gate/up, swiglu -> down).
// Issued as one launch per projection, the weight stream stops at every
// kernel boundary, and under tensor parallelism every rank also waits for
// the slowest rank at each all-reduce; at 8 ranks the projections are a few
// MB each and those boundaries are most of the step. This kernel runs the
// whole trunk (a table of phases, one per projection group) as one
// cooperative launch of one CTA per SM:
//
//  * Weights. Each of the 8 compute warps owns a ring of TMA stages (32 rows
//    x one superblock, no multicast). A ninth warp (the first of a third
//    warpgroup, which hands most of its registers to the compute warps)
//    issues the copies: its lane w walks compute warp w's share of phase p, then of phase p+1, ...,
//    and refills a stage as soon as the compute warp has read it (full /
//    empty mbarriers), so the next projections' weights are in flight while
//    the current one's input is still being produced, and no compute warp
//    ever waits for the TMA unit to accept a copy.
//  * Work split inside a phase: the CTA-range split of the decode GEMV
//    (gemv_row.cuh), with its in-CTA combination of row-block parts and the
//    tail-cut hand-off to the next CTA; or, for phases with few row blocks
//    per CTA (the small shards of tensor parallelism), ranges of whole row
//    blocks, which no CTA waits on another for.
//  * Hand-offs between phases. Every CTA that produced outputs of phase p
//    adds one to phase p's counter; a CTA that reads them waits (one thread,
//    short back-off) until the counter holds all of the phase's CTAs, then
//    loads the values (all of a lane's loads in flight together; not through
//    the TMA unit, whose queue is full of weight copies at that moment).
//    There is no grid barrier: a CTA waits only for the phase it reads, with
//    its ring of next weights already in flight. The values are
//    flagged 64-bit words (epoch << 32 | fp32 bits, one store each), so
//    every value read is checked to be this phase's (and waited for alone
//    if not): correctness rests on the words, the counter (relaxed, no fence
//    on the producer side) only says when to start copying. The residual
//    stream lives in one such vector (R, n_embd words), the q output in QB,
//    the SwiGLU product in AB; inside every 256-element block the words are
//    stored in the order tr_swz() gives (a lane's 16-byte pairs permuted).
//  * gate/up run as pairs: a stage holds 16 gate rows and the same 16 up
//    rows, so the warp that finishes them stores silu(gate) * up directly.
//  * Under tensor parallelism the row-parallel outputs (o, down) go to every
//    rank as LL words (tp_ar.inl's channel, four sequence slots). At the
//    start of the next phase every CTA folds its slice of R: the old value
//    plus the contributing ranks' words in rank order, published as the new
//    R. Ranks without attention rows in a layer skip its q/k/v and o phases
//    and contribute nothing to its o all-reduce (the mask says who does).
//  * Every CTA then builds the phase's Q8_K activation image in its own
//    shared memory (RMS norm with ggml-cpu's arithmetic and act_prep.cuh's
//    order of summation, then the Q8_K quantizer of q8k_block.cuh).
//
// Ordering. A buffer is overwritten only after every reader of its previous
// contents has finished the phase that read it: the writer's phase waited,
// directly or through the phases between, for the counter of that phase.
// Tail-cut words alternate between two halves by phase parity. The last CTA
// to leave resets the counters for the next run.
//
// Every wait is bounded (wait_limit_ns()). After a give-up the device error word
// is set, later waits return at once, the CTA skips the remaining phases,
// waits (bounded) for its copies in flight and exits.
#pragma once

#include "act_prep.cuh"
#include "gemv_row.cuh"

namespace cpq {

constexpr int kTrWarps = 8;                                // compute warps: warpgroups 0 and 1
constexpr int kTrThreads = (kTrWarps + 4) * 32;           // + warpgroup 2, whose first warp issues the copies
// Registers: launched at kTrRegLaunch per thread; the copy warpgroup gives
// back down to kTrRegCopy and the compute warpgroups take kTrRegCompute, so
// that 128 * kTrRegCopy + 256 * kTrRegCompute == 384 * kTrRegLaunch.
constexpr int kTrRegLaunch = 168, kTrRegCopy = 56, kTrRegCompute = 224;
static_assert(128 * kTrRegCopy + 256 * kTrRegCompute <= kTrThreads * kTrRegLaunch, "register split");
static_assert(kTrThreads * kTrRegLaunch <= 65536, "registers at launch");
static_assert(kTrWarps == kRowWarps, "the in-CTA combination is sized for kRowWarps");
constexpr int kTrStages = 5;
constexpr int kTrMaxW = 3;
constexpr int kTrMaxFold = 2;
constexpr int kTrRmsBlocks = 3;                           // 256-blocks per warp of an RMS image (K <= 24 * 256)
constexpr int kTrVecBatch = 2;                            // 256-blocks per warp whose loads are in flight together
constexpr int kTrBarBytes = kTrWarps * kTrStages * 8;     // one array of stage barriers
constexpr int kTrHdrBytes = 1024;                         // full and empty stage barriers, RMS partial sums
constexpr int kTrRingBytes = kTrWarps * kTrStages * kRowStageBytes;
static_assert(2 * kTrBarBytes + 64 <= kTrHdrBytes, "trunk header");

enum : int { kTrInR = 0, kTrInVec = 1 };
enum : int { kTrOutVec = 0, kTrOutPair = 1, kTrOutResid = 2, kTrOutAr = 3 };
enum : int { kTrBufQ = 0, kTrBufA = 1 };

struct alignas(64) TrWeight {
    CUtensorMap tmap;  // [n rows][row bytes / 8] u64; box 32 rows (16 for gate/up pairs) x one superblock
};

struct TrPhase {
    int nbk;          // superblocks per weight row (K / 256); 0 for a fold-only phase
    int n_w;          // weights (0: fold-only)
    int w0;           // first weight in the weight table (pairs: gate = w0, up = w0 + 1)
    int ctas;         // CTAs with work (at most one per row block)
    int pair;         // gate/up pairs: 16 gate + 16 up rows per row block
    int in_kind;      // kTrInR (RMS image of R) or kTrInVec (plain image of QB / AB)
    int in_buf;       // kTrBufQ / kTrBufA for kTrInVec
    int in_pub;       // phase whose words the image reads (-1: the run's input)
    int in_cnt;       // counter that says they are all written
    unsigned in_target;  // ... once it holds this many CTAs
    int n_fold;       // all-reduces folded into R at this phase's start (0..2)
    int r_prev;       // phase of R's previous publication (folds, kTrOutResid)
    int out_kind;
    unsigned fold_seq[kTrMaxFold];   // all-reduce index within the run
    unsigned fold_mask[kTrMaxFold];  // contributing ranks
    unsigned out_seq;                // all-reduce index (kTrOutAr)
    int write_h;      // this phase's publication of R also stores it to the run's h_out
    const float *g;   // RMS weight (or null)
    float eps;
    int whole;        // CTA ranges hold whole row blocks (no block cut between two CTAs)
    float *y_plain[kTrMaxW];        // kTrOutVec: plain fp32 outputs of weights 1, 2 (k, v)
    int64_t n[kTrMaxW];             // rows per weight (pairs: gate rows)
    int64_t mb_start[kTrMaxW + 1];  // prefix sums of row blocks per weight; mb_start[n_w] = total
};

struct TrArgs {
    const TrPhase *ph;
    const TrWeight *w;
    int n_ph;
    int n_embd;
    int act_bytes;      // shared-memory image region (largest phase image)
    unsigned n_ar;      // all-reduces per run
    uint64_t *R;        // [n_embd] flagged words, tr_swz order
    uint64_t *QB;       // [largest q]
    uint64_t *AB;       // [largest ffn slice]
    uint64_t *pieces;   // [2][grid][kTrWarps][32] tail-cut words
    unsigned *cnt;      // [0] the input's, [1 + 2p] phase p's folds, [2 + 2p] phase p's outputs
    unsigned *ctl;      // [0] epoch base, [1] exit counter
    const float *h_in;  // [n_embd]
    float *h_out;       // [n_embd]
    // all-reduce channel (world > 1)
    uint64_t *peer[kArMaxRanks];
    const uint64_t *ar_base;
    unsigned *ar_seq;
    int64_t ar_nmax;
    int world, rank;
};

__device__ __forceinline__ uint64_t flag_word(uint32_t ep, float v) { return (uint64_t(ep) << 32) | __float_as_uint(v); }

// Where element e of a flagged vector is stored: inside the 8 words of each
// lane (elements 8l..8l+7 of a 256-block), the four 16-byte pairs are
// XOR-permuted by bits 1-2 of l, so that 8 lanes reading "their pair c" of a
// staged block touch 8 different groups of four banks.
__device__ __forceinline__ int64_t tr_swz(int64_t e) {
    const int64_t l = (e >> 3) & 31;
    return (e & ~int64_t(7)) | ((((e >> 1) & 3) ^ ((l >> 1) & 3)) << 1) | (e & 1);
}

__device__ __forceinline__ void red_relaxed_add_gpu(unsigned *p, unsigned v) {
    asm volatile("red.relaxed.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ unsigned ld_relaxed_gpu_u32(const unsigned *p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

// Thread 0: wait (bounded, with a short back-off between polls) until the
// counter holds target CTAs. The words copied afterwards carry their own
// epochs, so the counter needs no acquire.
__device__ __forceinline__ void tr_wait_count(const unsigned *p, unsigned target) {
    if (ld_relaxed_gpu_u32(p) >= target) return;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        __nanosleep(32);
        if (ld_relaxed_gpu_u32(p) >= target) return;
        if ((it & 15u) == 0 && ((*reinterpret_cast<volatile uint32_t *>(&g_dev_error) & kDevErrWaitTimeout) ||
                                global_timer_ns() - t0 > wait_limit_ns())) {
            atomicOr(&g_dev_error, kDevErrWaitTimeout);
            return;
        }
    }
}

__device__ __forceinline__ float flagged_value(const uint64_t *p, uint32_t ep) {
    return __uint_as_float(uint32_t(flagged_word_gpu(p, ep)));
}

// Range of phase P for CTA c (the CTA-range split of gemv_row.cuh): list
// positions [0, L), the first LB of which are the tail cut [b0, hi).
struct TrRange {
    int64_t lo, hi, L, b0, LB;
    int64_t mbs1, mbs2;
    int nbk, w0, n_w, pair;
};

__device__ __forceinline__ bool tr_range(const TrPhase *P, int64_t c, TrRange &r) {
    const int n_w = P->n_w;
    const int64_t C = P->ctas;
    if (n_w == 0 || c >= C) return false;
    const int nbk = P->nbk;
    const int64_t RB = P->mb_start[n_w], T = RB * nbk;
    if (P->whole) {
        r.lo = (c * RB / C) * nbk;
        r.hi = ((c + 1) * RB / C) * nbk;
    } else {
        r.lo = c * T / C;
        r.hi = (c + 1) * T / C;
    }
    r.L = r.hi - r.lo;
    r.b0 = (r.hi % nbk) ? (r.hi - r.hi % nbk > r.lo ? r.hi - r.hi % nbk : r.lo) : r.hi;
    r.LB = r.hi - r.b0;
    r.mbs1 = P->mb_start[1];
    r.mbs2 = P->mb_start[2];
    r.nbk = nbk;
    r.w0 = P->w0;
    r.n_w = n_w;
    r.pair = P->pair;
    return r.L > 0;
}

struct TrCursor {
    int64_t j, it, mb;
    int kb;
};

__device__ __forceinline__ void tr_seek(const TrRange &r, TrCursor &q, int64_t j) {
    q.j = j;
    if (j < r.L) {
        q.it = j < r.LB ? r.b0 + j : r.lo + (j - r.LB);
        q.mb = q.it / r.nbk;
        q.kb = int(q.it - q.mb * r.nbk);
    }
}

__device__ __forceinline__ void tr_advance(const TrRange &r, TrCursor &q) {
    const int64_t j = q.j + kTrWarps;
    if (j >= r.L) {
        q.j = j;
    } else if (q.j < r.LB && j >= r.LB) {
        tr_seek(r, q, j);
    } else {
        q.j = j;
        q.it += kTrWarps;
        q.kb += kTrWarps;
        while (q.kb >= r.nbk) {
            q.kb -= r.nbk;
            q.mb++;
        }
    }
}

__device__ __forceinline__ int tr_weight_of(const TrRange &r, int64_t mb) {
    return (r.n_w > 1 && mb >= r.mbs1) + (r.n_w > 2 && mb >= r.mbs2);
}

// Barrier 1 among the 256 threads of the compute warps (the copy warp never
// joins it), plain and with a reduction of a predicate.
__device__ __forceinline__ void tr_bar() { asm volatile("bar.sync 1, 256;" ::: "memory"); }

__device__ __forceinline__ int tr_bar_or(int pred) {
    int r;
    asm volatile(
        "{\n\t.reg .pred a, b;\n\tsetp.ne.s32 a, %1, 0;\n\tbar.red.or.pred b, 1, 256, a;\n\tselp.s32 %0, 1, 0, b;\n\t}"
        : "=r"(r)
        : "r"(pred)
        : "memory");
    return r;
}

__device__ __forceinline__ void ld_relaxed_gpu_v2u64(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// This lane's 8 words (elements 8l..8l+7, in element order) of the 256-block
// at blk: four 16-byte loads issued back to back (tr_swz order in memory).
__device__ __forceinline__ void tr_load_lane(const uint64_t *blk, uint64_t (&w)[8]) {
    const int lane = threadIdx.x & 31, k = (lane >> 1) & 3;
#pragma unroll
    for (int c = 0; c < 4; c++) ld_relaxed_gpu_v2u64(blk + 8 * lane + 2 * (c ^ k), w[2 * c], w[2 * c + 1]);
}

// The values of tr_load_lane's words; a word without epoch ep is waited for
// on its own (it was loaded before its writer's store arrived).
__device__ __forceinline__ void tr_check_lane(const uint64_t *blk, uint32_t ep, const uint64_t (&w)[8], float (&v)[8]) {
    const int lane = threadIdx.x & 31, k = (lane >> 1) & 3;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const uint64_t x = uint32_t(w[i] >> 32) == ep ? w[i] : flagged_word_gpu(blk + 8 * lane + 2 * ((i >> 1) ^ k) + (i & 1), ep);
        v[i] = __uint_as_float(uint32_t(x));
    }
}

// The finished values of one row block of phase P (lane = row of the block).
__device__ __forceinline__ void tr_store(const TrArgs &a, const TrPhase *P, const TrRange &r, uint32_t ep,
                                         uint32_t ep_rprev, unsigned seq0, int64_t mb, float v) {
    const int lane = threadIdx.x & 31;
    const int kind = P->out_kind;
    if (kind == kTrOutPair) {  // lanes 0-15 gate rows, 16-31 the same up rows: silu(gate) * up
        const float u = __shfl_sync(0xffffffffu, v, lane | 16);
        const int64_t row = mb * 16 + lane;
        if (lane < 16 && row < P->n[0]) {
            const float s = __fdiv_rn(v, __fadd_rn(1.0f, expf(-v)));
            st_relaxed_gpu_u64(a.AB + tr_swz(row), flag_word(ep, __fmul_rn(s, u)));
        }
        return;
    }
    const int wi = tr_weight_of(r, mb);
    const int64_t row = (mb - (wi == 0 ? 0 : wi == 1 ? r.mbs1 : r.mbs2)) * kRowRows + lane;
    if (row >= P->n[wi]) return;
    if (kind == kTrOutVec) {
        if (wi == 0) {
            st_relaxed_gpu_u64(a.QB + tr_swz(row), flag_word(ep, v));
        } else if (P->y_plain[wi]) {
            P->y_plain[wi][row] = v;
        }
    } else if (kind == kTrOutResid) {  // one rank: R = R + y, the residual add of the next prologue
        const float nv = __fadd_rn(flagged_value(a.R + tr_swz(row), ep_rprev), v);
        st_relaxed_gpu_u64(a.R + tr_swz(row), flag_word(ep, nv));
        if (P->write_h) a.h_out[row] = nv;
    } else {  // LL words to every rank (row-parallel partial sums)
        const unsigned s = seq0 + 1u + P->out_seq;
        const int64_t off = (int64_t(s % kArSlots) * a.world + a.rank) * a.ar_nmax + row;
        const uint64_t wv = (uint64_t(s) << 32) | __float_as_uint(v);
        for (int d = 0; d < a.world; d++) st_relaxed_sys_u64(a.peer[d] + off, wv);
    }
}

// This CTA's slice of R at a phase start: the previous R plus, for each
// folded all-reduce in turn, the sum of the contributing ranks' LL words in
// rank order (the additions of act_load_v / ar_sum8; ranks that contribute
// nothing would only add zeros). One element per thread.
__device__ __forceinline__ void tr_fold(const TrArgs &a, const TrPhase *P, uint32_t ep, uint32_t ep_rprev,
                                        unsigned seq0) {
    const int64_t C = gridDim.x, c = blockIdx.x;
    const int64_t e = c * a.n_embd / C + threadIdx.x;
    if (e >= (c + 1) * a.n_embd / C) return;
    const int nf = P->n_fold;
    uint64_t w[kTrMaxFold][kArMaxRanks];
    unsigned sq[kTrMaxFold];
#pragma unroll
    for (int f = 0; f < kTrMaxFold; f++) {
        sq[f] = seq0 + 1u + P->fold_seq[f];
        const uint64_t *base = a.ar_base + int64_t(sq[f] % kArSlots) * a.world * a.ar_nmax + e;
        const unsigned mask = f < nf ? P->fold_mask[f] : 0u;
#pragma unroll
        for (int s = 0; s < kArMaxRanks; s++) {
            w[f][s] = 0;
            if (s < a.world && ((mask >> s) & 1u)) w[f][s] = ld_relaxed_sys_u64(base + int64_t(s) * a.ar_nmax);
        }
    }
    float v = flagged_value(a.R + tr_swz(e), ep_rprev);
#pragma unroll
    for (int f = 0; f < kTrMaxFold; f++) {
        if (f >= nf) continue;
        const uint64_t *base = a.ar_base + int64_t(sq[f] % kArSlots) * a.world * a.ar_nmax + e;
        const unsigned mask = P->fold_mask[f];
        float sum = 0.0f;
        bool first = true;
#pragma unroll
        for (int s = 0; s < kArMaxRanks; s++)
            if (s < a.world && ((mask >> s) & 1u)) {
                const float q = unsigned(w[f][s] >> 32) == sq[f] ? __uint_as_float(unsigned(w[f][s]))
                                                                 : ar_word(base + int64_t(s) * a.ar_nmax, sq[f]);
                sum = first ? q : __fadd_rn(sum, q);
                first = false;
            }
        v = __fadd_rn(v, sum);
    }
    st_relaxed_gpu_u64(a.R + tr_swz(e), flag_word(ep, v));
    if (P->write_h) a.h_out[e] = v;
}

// The RMS image of R: rms_norm(R) * g quantized to Q8_K into img. Order of
// summation of act_rms_row: lane l of warp w adds, for its blocks w, w+8,
// ..., elements 8l..8l+7 (fp32 squares in double), then a warp butterfly,
// then warps in order.
__device__ __forceinline__ void tr_image_rms(const TrArgs &a, const TrPhase *P, uint32_t ep, double *part,
                                             uint8_t *img) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int nbk = P->nbk;
    const int64_t k = int64_t(nbk) * kQK_K;
    const int nbw = nbk > warp ? (nbk - warp + 7) / 8 : 0;
    uint64_t w[kTrRmsBlocks][8];
#pragma unroll
    for (int jj = 0; jj < kTrRmsBlocks; jj++)
        if (jj < nbw) tr_load_lane(a.R + int64_t(warp + 8 * jj) * kQK_K, w[jj]);
    float vk[kTrRmsBlocks][8];
    double s = 0.0;
#pragma unroll
    for (int jj = 0; jj < kTrRmsBlocks; jj++)
        if (jj < nbw) {
            tr_check_lane(a.R + int64_t(warp + 8 * jj) * kQK_K, ep, w[jj], vk[jj]);
#pragma unroll
            for (int e = 0; e < 8; e++) s += double(__fmul_rn(vk[jj][e], vk[jj][e]));
        }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) part[warp] = s;
    tr_bar();
    double tot = 0.0;
#pragma unroll
    for (int i = 0; i < 8; i++) tot += part[i];
    const float mean = float(tot / double(k));
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(mean, P->eps)));
    const float *g = P->g;
#pragma unroll
    for (int jj = 0; jj < kTrRmsBlocks; jj++)
        if (jj < nbw) act_quantize_store(kActRms, vk[jj], scale, g, warp + 8 * jj, 0, k, 1, img);
}

// The plain image of a flagged vector (q for o, silu(gate) * up for down).
__device__ __forceinline__ void tr_image_vec(const uint64_t *buf, int nbk, uint32_t ep, uint8_t *img) {
    const int warp = threadIdx.x >> 5;
    const int64_t k = int64_t(nbk) * kQK_K;
    for (int b0 = warp; b0 < nbk; b0 += 8 * kTrVecBatch) {
        uint64_t w[kTrVecBatch][8];
#pragma unroll
        for (int jj = 0; jj < kTrVecBatch; jj++)
            if (b0 + 8 * jj < nbk) tr_load_lane(buf + int64_t(b0 + 8 * jj) * kQK_K, w[jj]);
#pragma unroll
        for (int jj = 0; jj < kTrVecBatch; jj++)
            if (b0 + 8 * jj < nbk) {
                float v[8];
                tr_check_lane(buf + int64_t(b0 + 8 * jj) * kQK_K, ep, w[jj], v);
                act_quantize_store(kActPlain, v, 1.0f, nullptr, b0 + 8 * jj, 0, k, 1, img);
            }
    }
}

__device__ __forceinline__ bool tr_error_set() {
    return (*reinterpret_cast<volatile uint32_t *>(&g_dev_error) & kDevErrWaitTimeout) != 0;
}

__global__ void __maxnreg__(kTrRegLaunch) trunk_kernel(const __grid_constant__ TrArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem);                  // [warp][stage]: the copy landed
    uint64_t *empty = reinterpret_cast<uint64_t *>(smem + kTrBarBytes);   // [warp][stage]: the warp has read it
    double *part = reinterpret_cast<double *>(smem + 2 * kTrBarBytes);
    uint8_t *img = smem + kTrHdrBytes;
    uint8_t *ring0 = img + a.act_bytes;  // [warp][stage] of kRowStageBytes
    float *red = reinterpret_cast<float *>(ring0 + kTrRingBytes);
    int *red_cnt = reinterpret_cast<int *>(red + (kRowRedSlots + 1) * kTrWarps * 32);
    int *red_gen = red_cnt + kRowRedSlots + 1;
    if (threadIdx.x < kTrWarps * kTrStages) {
        mbar_init(&full[threadIdx.x], 1);
        mbar_init(&empty[threadIdx.x], 1);
    }
    fence_mbar_init();
    __syncthreads();

    const int64_t c = blockIdx.x, C = gridDim.x;
    const unsigned E0 = *reinterpret_cast<volatile unsigned *>(a.ctl);
    const unsigned seq0 = a.world > 1 ? *reinterpret_cast<volatile unsigned *>(a.ar_seq) : 0u;
    auto epoch = [&](int p) { return E0 + 2u + unsigned(p); };  // p = -1: the run's input

    if (warp >= kTrWarps) {
        asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kTrRegCopy));
        // ---- the copy warp: lane w issues compute warp w's stages, phase after phase ----
        if (warp == kTrWarps && lane < kTrWarps) {
            const int w = lane;
            const uint64_t policy = l2_policy_evict_first();
            uint8_t *ring = ring0 + w * kTrStages * kRowStageBytes;
            int ip = a.n_ph;
            TrRange ir;
            TrCursor pc;
            auto i_seek = [&](int from) {
                for (ip = from; ip < a.n_ph; ip++)
                    if (tr_range(a.ph + ip, c, ir) && w < ir.L) {
                        tr_seek(ir, pc, w);
                        return;
                    }
            };
            i_seek(0);
            int64_t issued = 0;
            while (ip < a.n_ph) {
                const int s = int(issued % kTrStages);
                if (issued >= kTrStages &&
                    !mbar_wait_bounded(&empty[w * kTrStages + s], uint32_t(issued / kTrStages - 1) & 1u))
                    break;  // the compute warp stopped (error recorded)
                uint64_t *bar = &full[w * kTrStages + s];
                mbar_arrive_expect_tx(bar, kRowStageBytes);
                const int x = pc.kb * (kQ4K_Bytes / 8);
                if (ir.pair) {
                    const int row0 = int(pc.mb * 16);
                    tma_load_2d(ring + s * kRowStageBytes, &a.w[ir.w0].tmap, x, row0, bar, policy);
                    tma_load_2d(ring + s * kRowStageBytes + 16 * kQ4K_Bytes, &a.w[ir.w0 + 1].tmap, x, row0, bar, policy);
                } else {
                    const int wi = tr_weight_of(ir, pc.mb);
                    const int row0 = int((pc.mb - (wi == 0 ? 0 : wi == 1 ? ir.mbs1 : ir.mbs2)) * kRowRows);
                    tma_load_2d(ring + s * kRowStageBytes, &a.w[ir.w0 + wi].tmap, x, row0, bar, policy);
                }
                issued++;
                tr_advance(ir, pc);
                if (pc.j >= ir.L) i_seek(ip + 1);
            }
            // the copies still in flight land before the CTA leaves (normally all were read already)
            for (int64_t u = issued > kTrStages ? issued - kTrStages : 0; u < issued; u++)
                mbar_wait_bounded(&full[w * kTrStages + int(u % kTrStages)], uint32_t(u / kTrStages) & 1u);
        }
    } else {
        asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kTrRegCompute));
        // ---- the compute warps ----
        {  // the run's input: h_in -> R (this CTA's slice)
            const int64_t e = c * a.n_embd / C + threadIdx.x;
            if (e < (c + 1) * a.n_embd / C) st_relaxed_gpu_u64(a.R + tr_swz(e), flag_word(epoch(-1), a.h_in[e]));
            tr_bar();
            if (threadIdx.x == 0) red_relaxed_add_gpu(a.cnt, 1u);
        }
        uint8_t *ring = ring0 + warp * kTrStages * kRowStageBytes;
        int slot = 0;
        uint32_t phase_bit = 0;
        for (int p = 0; p < a.n_ph; p++) {
            const TrPhase *P = a.ph + p;
            const uint32_t ep = epoch(p);
            const int err = threadIdx.x == 0 && tr_error_set();
            if (P->n_fold > 0) tr_fold(a, P, ep, epoch(P->r_prev), seq0);
            if (tr_bar_or(err)) break;  // an earlier wait gave up: skip the remaining phases
            if (P->n_fold > 0 && threadIdx.x == 0) red_relaxed_add_gpu(a.cnt + 1 + 2 * p, 1u);
            TrRange r;
            if (!tr_range(P, c, r)) continue;
            const int nbk = r.nbk;
            const int64_t k = int64_t(nbk) * kQK_K;

            // ---- this phase's activation image ----
            if (threadIdx.x <= kRowRedSlots) red_cnt[threadIdx.x] = 0;
            const int64_t mbA = r.lo / nbk;      // the row block the range starts in
            const bool cutA = (r.lo % nbk) != 0;  // ... and whose head is CTA c-1's tail cut
            if (threadIdx.x < kRowRedSlots)
                red_gen[threadIdx.x] = (threadIdx.x == 0 && cutA) ? kRowRedSlots : int(threadIdx.x);
            if (threadIdx.x == 0) tr_wait_count(a.cnt + P->in_cnt, P->in_target);
            tr_bar();
            if (P->in_kind == kTrInR)
                tr_image_rms(a, P, epoch(P->in_pub), part, img);
            else
                tr_image_vec(P->in_buf == kTrBufQ ? a.QB : a.AB, nbk, epoch(P->in_pub), img);
            tr_bar();

            const int8_t *xs = reinterpret_cast<const int8_t *>(img);
            const float *xd = reinterpret_cast<const float *>(img + align_up(size_t(k), 16));
            const uint8_t *xb = img + align_up(size_t(k), 16) + align_up(size_t(nbk) * 4, 16);
            const uint32_t ep_rprev = epoch(P->r_prev);
            auto store_block = [&](int64_t mb, float v) { tr_store(a, P, r, ep, ep_rprev, seq0, mb, v); };

            // ---- compute: the CTA-range split (gemv_row.cuh), one token ----
            const int64_t L = r.L, LB = r.LB, lo = r.lo, b0 = r.b0;
            const int fw = int((L - 1) % kTrWarps);
            const int nw_prev = int(r.lo % nbk < kTrWarps ? r.lo % nbk : kTrWarps);
            uint64_t *pieces_p = a.pieces + int64_t(p & 1) * C * kTrWarps * 32;
            const uint64_t *prev = pieces_p + (c - 1) * kTrWarps * 32 + lane;
            auto finish_cut = [&](const float (&pre)[kTrWarps]) {
                const int64_t la = ((mbA + 1) * nbk < b0 ? (mbA + 1) * nbk : b0) - lo;
                const int len = int(la < kTrWarps ? la : kTrWarps);
                if (!smem_wait_eq(&red_cnt[kRowRedSlots], len)) return;
                __threadfence_block();
                float s = 0.0f;
#pragma unroll
                for (int u = 0; u < kTrWarps; u++)
                    if (u < nw_prev) s += pre[u];
                const int p0 = int(LB % kTrWarps);
#pragma unroll
                for (int u = 0; u < kTrWarps; u++)
                    if (((u - p0 + kTrWarps) % kTrWarps) < len) s += red[(kRowRedSlots * kTrWarps + u) * 32 + lane];
                store_block(mbA, s);
            };
            auto arrive = [&](int64_t mb, float part_v) -> bool {
                const int64_t s_it = mb * nbk > lo ? mb * nbk : lo;
                const int64_t e_it = (mb + 1) * nbk < b0 ? (mb + 1) * nbk : b0;
                const int len = int(e_it - s_it < kTrWarps ? e_it - s_it : kTrWarps);
                const int q = int(mb - mbA);
                if (cutA && q == 0) {
                    red[(kRowRedSlots * kTrWarps + warp) * 32 + lane] = part_v;
                    __syncwarp();
                    if (lane == 0) {
                        __threadfence_block();
                        atomicAdd(&red_cnt[kRowRedSlots], 1);
                    }
                    return true;
                }
                const int s = q % kRowRedSlots;
                if (!smem_wait_eq(&red_gen[s], q)) return false;
                if (len == 1) {
                    __syncwarp();
                    if (lane == 0) *reinterpret_cast<volatile int *>(&red_gen[s]) = q + kRowRedSlots;
                    store_block(mb, part_v);
                    return true;
                }
                red[(s * kTrWarps + warp) * 32 + lane] = part_v;
                __syncwarp();
                int old = 0;
                if (lane == 0) {
                    __threadfence_block();
                    old = atomicAdd(&red_cnt[s], 1);
                }
                old = __shfl_sync(0xffffffffu, old, 0);
                if (old != len - 1) return true;
                __threadfence_block();
                const int p0 = int((LB + (s_it - lo)) % kTrWarps);
                float sum = 0.0f;
#pragma unroll
                for (int u = 0; u < kTrWarps; u++)
                    if (((u - p0 + kTrWarps) % kTrWarps) < len) sum += red[(s * kTrWarps + u) * 32 + lane];
                __syncwarp();
                if (lane == 0) {
                    red_cnt[s] = 0;
                    __threadfence_block();
                    *reinterpret_cast<volatile int *>(&red_gen[s]) = q + kRowRedSlots;
                }
                store_block(mb, sum);
                return true;
            };

            float acc = 0.0f;
            float pre[kTrWarps];
#pragma unroll
            for (int u = 0; u < kTrWarps; u++) pre[u] = 0.0f;
            TrCursor cc;
            tr_seek(r, cc, warp);
            bool ok = true;
            while (cc.j < L) {
                if (cutA && warp == fw && cc.j + kTrWarps >= L) {  // the finisher's last stage: CTA c-1's words
                    uint64_t w[kTrWarps];
#pragma unroll
                    for (int u = 0; u < kTrWarps; u++)
                        if (u < nw_prev) w[u] = ld_relaxed_gpu_u64(prev + u * 32);
#pragma unroll
                    for (int u = 0; u < kTrWarps; u++)
                        if (u < nw_prev)
                            pre[u] = __uint_as_float(
                                uint32_t(uint32_t(w[u] >> 32) == ep ? w[u] : flagged_word_gpu(prev + u * 32, ep)));
                }
                if (!mbar_wait_bounded(&full[warp * kTrStages + slot], phase_bit)) {
                    ok = false;
                    break;
                }
                __syncwarp();
                const uint8_t *blk = ring + slot * kRowStageBytes + lane * kQ4K_Bytes;
                const uint4 h = *reinterpret_cast<const uint4 *>(blk);
                uint4 qv[8];
#pragma unroll
                for (int i = 0; i < 8; i++) qv[i] = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * i);
                __syncwarp();
                if (lane == 0) mbar_arrive(&empty[warp * kTrStages + slot]);  // the copy warp may refill it
                float accv[1] = {acc};
                row_dot<1>(h, qv, xs, xd, xb, k, nbk, cc.kb, accv);
                acc = accv[0];
                if (++slot == kTrStages) {
                    slot = 0;
                    phase_bit ^= 1u;
                }
                const int64_t mb = cc.mb;
                const bool in_tail = cc.j < LB;
                tr_advance(r, cc);
                if (cc.j >= L || cc.mb != mb) {  // this warp's part of row block mb is complete
                    if (in_tail) {
                        st_relaxed_gpu_u64(pieces_p + (c * kTrWarps + warp) * 32 + lane, flag_word(ep, acc));
                    } else if (!arrive(mb, acc)) {
                        ok = false;
                        break;
                    }
                    acc = 0.0f;
                }
            }
            if (ok && cutA && warp == fw) finish_cut(pre);
            // this CTA's phase-p outputs are stored; the image and the combination slots are free
            const int bad = tr_bar_or(!ok);
            if (threadIdx.x == 0) red_relaxed_add_gpu(a.cnt + 2 + 2 * p, 1u);
            if (bad) break;
        }
    }

    // ---- the last CTA to leave resets the counters, advances the epoch base and the channel's sequence ----
    __shared__ int last;
    __syncthreads();
    if (threadIdx.x == 0) last = atomicAdd(a.ctl + 1, 1u) == unsigned(C) - 1u;
    __syncthreads();
    if (last) {
        for (int i = threadIdx.x; i < 2 * a.n_ph + 1; i += blockDim.x) a.cnt[i] = 0u;
        if (threadIdx.x == 0) {
            a.ctl[1] = 0u;
            a.ctl[0] = E0 + 2u + unsigned(a.n_ph);
            if (a.world > 1) *a.ar_seq = seq0 + a.n_ar;
        }
    }
}

}  // namespace cpq
