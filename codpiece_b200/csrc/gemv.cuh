// gemv.cuh — small-M quantized mat-vec/mat-mat kernels (decode and verify).
//
// Y[t][n] = sum over superblocks b of row n:
//   Q4_K: d_w*d_x * sum_j sc_j sum_i q*q8  -  dmin_w*d_x * sum_j m_j * bsum_j
//   Q6_K: d_w*d_x * sum_g s_g * (sum_i q6*q8 - 32*bsum_g)
//   Q8_0: d_w*d_x * sum_i q*q8
// the ggml-cpu block dots (ggml_vec_dot_q4_K_q8_K, _q6_K_q8_K, _q8_0_q8_0)
// with integer products inside each lane's slice of a block and fp32 across.
//
// Memory path. The weight matrix is read exactly once per call, in ggml's own
// row layout. Each warp owns whole rows and streams them through a private
// ring of kStages shared-memory stages with 1-D bulk copies (cp.async.bulk,
// the TMA engine, no tensor map, no multicast), one mbarrier per stage, so a
// warp keeps kStages-1 chunks in flight while it decodes one. The copies of
// the first stages are issued before griddepcontrol.wait, so under
// programmatic dependent launch a GEMV starts streaming its weights while the
// kernel that produces its activations is still finishing. Activations (a few
// KB per token) are read through the read-only path and stay L1/L2 resident.
#pragma once

#include "common.cuh"

namespace cpq {

#ifndef CPQ_GEMV_WARPS
#define CPQ_GEMV_WARPS 8
#endif
#ifndef CPQ_Q4K_PASSES
#define CPQ_Q4K_PASSES 2
#endif
#ifndef CPQ_Q4K_STAGES
#define CPQ_Q4K_STAGES 6
#endif
#ifndef CPQ_Q6K_STAGES
#define CPQ_Q6K_STAGES 4
#endif

constexpr int kGemvWarps = CPQ_GEMV_WARPS;  // warps per CTA
constexpr int kMaxMulti = 4;   // weights sharing one activation in one launch

struct GemvArgs {
    int n_w;
    const uint8_t *w[kMaxMulti];
    const uint8_t *w_end[kMaxMulti];  // one past the last byte of each weight
    float *y[kMaxMulti];
    int64_t y_stride[kMaxMulti];       // floats between tokens in y
    int64_t row_start[kMaxMulti + 1];  // prefix sums of the row counts
    size_t rs;                         // row stride in bytes (same K and type)
    int64_t k;
    ActQ act;
};

// ---------------------------------------------------------------------------
// Format policies. Each defines the chunk geometry (kCB blocks per chunk,
// kStageBytes per ring stage including alignment slack) and accumulate(),
// which adds one chunk's contribution for MT tokens to the lane's partials.

struct FmtQ4K {
    static constexpr int kBlkBytes = kQ4K_Bytes, kBlkElems = kQK_K;
    static constexpr int kPasses = CPQ_Q4K_PASSES;  // 4 blocks per pass, 8 lanes each
    static constexpr int kCB = 4 * kPasses;         // blocks per chunk
    static constexpr int kStageBytes = kCB * kBlkBytes;  // 144 B blocks keep 16 B alignment
    static constexpr int kStages = CPQ_Q4K_STAGES;
    static constexpr bool kAligned = true;

    template <int MT>
    __device__ __forceinline__ static void accumulate(const uint8_t *chunk, int nblk, int64_t blk0, const ActQ &act,
                                                      int64_t k, float (&acc)[MT], int lane) {
        const int c = lane & 7;        // 16-byte slice of the 128 quant bytes
        const int j = c >> 1, half = c & 1;
        const int64_t nbk = k / kQK_K;
        const int64_t k16 = k / 16;
#pragma unroll
        for (int p = 0; p < kPasses; p++) {
            const int bi = p * 4 + (lane >> 3);
            if (bi >= nblk) continue;
            const uint8_t *blk = chunk + bi * kBlkBytes;
            const uint4 hdr = *reinterpret_cast<const uint4 *>(blk);
            const uint4 qv = *reinterpret_cast<const uint4 *>(blk + 16 + 16 * c);
            // six-bit scales/mins of sub-blocks 2j and 2j+1
            const uint32_t w0 = hdr.y, w1 = hdr.z, w2 = hdr.w;
            uint32_t scw, mw;
            if (j < 2) {
                scw = w0 & 0x3f3f3f3fu;
                mw = w1 & 0x3f3f3f3fu;
            } else {
                scw = (w2 & 0x0f0f0f0fu) | (((w0 >> 6) & 0x03030303u) << 4);
                mw = ((w2 >> 4) & 0x0f0f0f0fu) | (((w1 >> 6) & 0x03030303u) << 4);
            }
            const int sh = (j & 1) * 16;
            const int sc0 = (scw >> sh) & 0xff, sc1 = (scw >> (sh + 8)) & 0xff;
            const int m0 = (mw >> sh) & 0xff, m1 = (mw >> (sh + 8)) & 0xff;
            const float dw = half_bits_to_float(hdr.x), dmw = half_bits_to_float(hdr.x >> 16);
            const int lo0 = qv.x & 0x0f0f0f0f, lo1 = qv.y & 0x0f0f0f0f, lo2 = qv.z & 0x0f0f0f0f,
                      lo3 = qv.w & 0x0f0f0f0f;
            const int hi0 = (qv.x >> 4) & 0x0f0f0f0f, hi1 = (qv.y >> 4) & 0x0f0f0f0f,
                      hi2 = (qv.z >> 4) & 0x0f0f0f0f, hi3 = (qv.w >> 4) & 0x0f0f0f0f;
            const int64_t b = blk0 + bi;
            const int64_t e_lo = b * kQK_K + 64 * j + 16 * half;
            const int64_t g_lo = b * 16 + 4 * j + half;
#pragma unroll
            for (int t = 0; t < MT; t++) {
                const int8_t *xq = act.qs + t * k + e_lo;
                const int4 xa = ldg_nc_v4(xq);
                const int4 xb = ldg_nc_v4(xq + 32);
                const int dl = __dp4a(lo3, xa.w, __dp4a(lo2, xa.z, __dp4a(lo1, xa.y, __dp4a(lo0, xa.x, 0))));
                const int dh = __dp4a(hi3, xb.w, __dp4a(hi2, xb.z, __dp4a(hi1, xb.y, __dp4a(hi0, xb.x, 0))));
                const int isc = sc0 * dl + sc1 * dh;
                const int16_t *bs = act.bsums + t * k16 + g_lo;
                const int imn = m0 * int(__ldg(bs)) + m1 * int(__ldg(bs + 2));
                const float dx = __ldg(act.d + t * nbk + b);
                acc[t] += (dw * dx) * float(isc) - (dmw * dx) * float(imn);
            }
        }
    }
};

struct FmtQ6K {
    static constexpr int kBlkBytes = kQ6K_Bytes, kBlkElems = kQK_K;
    static constexpr int kCB = 8;  // 4 lanes per block
    static constexpr int kStageBytes = kCB * kBlkBytes + 32;  // 210 B blocks: up to 15 B misalignment
    static constexpr int kStages = CPQ_Q6K_STAGES;
    static constexpr bool kAligned = false;

    template <int MT>
    __device__ __forceinline__ static void accumulate(const uint8_t *chunk, int nblk, int64_t blk0, const ActQ &act,
                                                      int64_t k, float (&acc)[MT], int lane) {
        const int bi = lane >> 2;
        if (bi >= nblk) return;
        const int p = lane & 3, h = p >> 1, c = p & 1;
        const uint8_t *blk = chunk + bi * kBlkBytes;
        const uint4 qa = lds16_a2(blk + 64 * h + 16 * c);
        const uint4 qb = lds16_a2(blk + 64 * h + 32 + 16 * c);
        const uint4 qh = lds16_a2(blk + 128 + 32 * h + 16 * c);
        // scales of this lane's four 16-element groups: bytes c, c+2, c+4, c+6 of scales[8h..8h+7]
        const uint8_t *sp = blk + 192 + 8 * h;
        const uintptr_t sa = reinterpret_cast<uintptr_t>(sp);
        const uint32_t *sw = reinterpret_cast<const uint32_t *>(sa & ~uintptr_t(3));
        const uint32_t ssh = uint32_t(sa & 3u) * 8u;
        const uint32_t s_lo = __funnelshift_r(sw[0], sw[1], ssh), s_hi = __funnelshift_r(sw[1], sw[2], ssh);
        const int sc0 = int(int8_t((s_lo >> (8 * c)) & 0xff));
        const int sc1 = int(int8_t((s_lo >> (8 * (c + 2))) & 0xff));
        const int sc2 = int(int8_t((s_hi >> (8 * c)) & 0xff));
        const int sc3 = int(int8_t((s_hi >> (8 * (c + 2))) & 0xff));
        const float dw = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk + 208));
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
        const int64_t b = blk0 + bi;
        const int64_t e0 = b * kQK_K + 128 * h + 16 * c;
        const int64_t g0 = b * 16 + 8 * h + c;
        const int64_t nbk = k / kQK_K, k16 = k / 16;
#pragma unroll
        for (int t = 0; t < MT; t++) {
            const int8_t *xq = act.qs + t * k + e0;
            const int16_t *bs = act.bsums + t * k16 + g0;
            const int4 x0 = ldg_nc_v4(xq), x1 = ldg_nc_v4(xq + 32), x2 = ldg_nc_v4(xq + 64),
                       x3 = ldg_nc_v4(xq + 96);
            const int d0 = dp4a_us(r0[3], x0.w, dp4a_us(r0[2], x0.z, dp4a_us(r0[1], x0.y, dp4a_us(r0[0], x0.x, 0))));
            const int d1 = dp4a_us(r1[3], x1.w, dp4a_us(r1[2], x1.z, dp4a_us(r1[1], x1.y, dp4a_us(r1[0], x1.x, 0))));
            const int d2 = dp4a_us(r2[3], x2.w, dp4a_us(r2[2], x2.z, dp4a_us(r2[1], x2.y, dp4a_us(r2[0], x2.x, 0))));
            const int d3 = dp4a_us(r3[3], x3.w, dp4a_us(r3[2], x3.z, dp4a_us(r3[1], x3.y, dp4a_us(r3[0], x3.x, 0))));
            const int tot = sc0 * (d0 - 32 * int(__ldg(bs))) + sc1 * (d1 - 32 * int(__ldg(bs + 2))) +
                            sc2 * (d2 - 32 * int(__ldg(bs + 4))) + sc3 * (d3 - 32 * int(__ldg(bs + 6)));
            const float dx = __ldg(act.d + t * nbk + b);
            acc[t] += (dw * dx) * float(tot);
        }
    }
};

struct FmtQ8_0 {
    static constexpr int kBlkBytes = kQ8_0_Bytes, kBlkElems = kQK8_0;
    static constexpr int kCB = 16;  // 2 lanes per block
    static constexpr int kStageBytes = kCB * kBlkBytes + 32;
    static constexpr int kStages = 12;
    static constexpr bool kAligned = false;

    template <int MT>
    __device__ __forceinline__ static void accumulate(const uint8_t *chunk, int nblk, int64_t blk0, const ActQ &act,
                                                      int64_t k, float (&acc)[MT], int lane) {
        const int bi = lane >> 1;
        if (bi >= nblk) return;
        const int half = lane & 1;
        const uint8_t *blk = chunk + bi * kBlkBytes;
        const float dw = half_bits_to_float(*reinterpret_cast<const uint16_t *>(blk));
        const uint4 q = lds16_a2(blk + 2 + 16 * half);
        const int64_t b = blk0 + bi;
        const int64_t nbk = k / kQK8_0;
#pragma unroll
        for (int t = 0; t < MT; t++) {
            const int4 x = ldg_nc_v4(act.qs + t * k + b * kQK8_0 + 16 * half);
            const int dot = __dp4a(int(q.w), x.w, __dp4a(int(q.z), x.z, __dp4a(int(q.y), x.y, __dp4a(int(q.x), x.x, 0))));
            acc[t] += float(dot) * (dw * __ldg(act.d + t * nbk + b));
        }
    }
};

// ---------------------------------------------------------------------------

template <class F>
struct GemvSmem {
    static constexpr int kBarBytes = 128 * ((kGemvWarps * F::kStages * 8 + 127) / 128);
    static constexpr int kBytes = kBarBytes + kGemvWarps * F::kStages * F::kStageBytes;
};

// Where item i (the ch-th chunk of this warp's r-th row) lives.
struct ChunkSpan {
    const uint8_t *a0;  // 16-byte aligned copy start
    uint32_t bytes;     // bulk-copied bytes (multiple of 16, may be 0)
    uint32_t off;       // offset of the first block inside the stage
    uint32_t tail;      // bytes past the bulk copy that lanes copy by hand (< 16)
    int nblk;
    int ch;
    int wi;
    int64_t lrow;
};

template <class F>
__device__ __forceinline__ ChunkSpan chunk_span(const GemvArgs &a, int64_t i, int nch, int nbk, int64_t gw,
                                                int64_t G) {
    ChunkSpan s;
    const int64_t ri = i / nch;
    s.ch = int(i - ri * nch);
    const int64_t grow = gw + ri * G;
    int wi = 0;
#pragma unroll
    for (int q = 1; q < kMaxMulti; q++)
        if (q < a.n_w && grow >= a.row_start[q]) wi = q;
    s.wi = wi;
    s.lrow = grow - a.row_start[wi];
    const int blk_start = s.ch * F::kCB;
    s.nblk = min(F::kCB, nbk - blk_start);
    const uint8_t *src = a.w[wi] + size_t(s.lrow) * a.rs + size_t(blk_start) * F::kBlkBytes;
    const uint8_t *end = src + size_t(s.nblk) * F::kBlkBytes;
    if (F::kAligned) {
        s.a0 = src;
        s.bytes = uint32_t(end - src);
        s.off = 0;
        s.tail = 0;
    } else {
        const uintptr_t a0 = reinterpret_cast<uintptr_t>(src) & ~uintptr_t(15);
        uintptr_t a1 = (reinterpret_cast<uintptr_t>(end) + 15) & ~uintptr_t(15);
        const uintptr_t lim = reinterpret_cast<uintptr_t>(a.w_end[wi]) & ~uintptr_t(15);
        if (a1 > lim) a1 = lim > a0 ? lim : a0;
        s.a0 = reinterpret_cast<const uint8_t *>(a0);
        s.bytes = uint32_t(a1 - a0);
        s.off = uint32_t(reinterpret_cast<uintptr_t>(src) - a0);
        s.tail = uint32_t(reinterpret_cast<uintptr_t>(end) > a1 ? reinterpret_cast<uintptr_t>(end) - a1 : 0);
    }
    return s;
}

template <class F, int MT>
__global__ void __launch_bounds__(kGemvWarps * 32) gemv_kernel(const __grid_constant__ GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int S = F::kStages;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem) + warp * S;
    uint8_t *ring = smem + GemvSmem<F>::kBarBytes + warp * S * F::kStageBytes;

    if (lane == 0) {
#pragma unroll
        for (int s = 0; s < S; s++) mbar_init(&bars[s], 1);
        fence_mbar_init();
    }
    __syncwarp();

    const int64_t k = a.k;
    const int nbk = int(k / F::kBlkElems);
    const int nch = (nbk + F::kCB - 1) / F::kCB;
    const int64_t G = int64_t(gridDim.x) * kGemvWarps;
    const int64_t gw = int64_t(blockIdx.x) * kGemvWarps + warp;
    const int64_t ntot = a.row_start[a.n_w];
    const int64_t nrows = gw < ntot ? (ntot - 1 - gw) / G + 1 : 0;
    const int64_t total = nrows * nch;
    const uint64_t policy = l2_policy_evict_first();

    auto issue = [&](int64_t i) {
        const ChunkSpan s = chunk_span<F>(a, i, nch, nbk, gw, G);
        uint8_t *dst = ring + (i % S) * F::kStageBytes;
        if (lane == 0) {
            fence_proxy_async_smem();
            mbar_arrive_expect_tx(&bars[i % S], s.bytes);
            if (s.bytes) bulk_g2s_stream(dst, s.a0, s.bytes, &bars[i % S], policy);
        }
        if (!F::kAligned && s.tail && lane < int(s.tail)) dst[s.bytes + lane] = s.a0[s.bytes + lane];
    };

    const int64_t pro = total < S ? total : S;
    for (int64_t i = 0; i < pro; i++) issue(i);

    pdl_wait();
    pdl_launch_dependents();

    float acc[MT];
#pragma unroll
    for (int t = 0; t < MT; t++) acc[t] = 0.0f;

    for (int64_t i = 0; i < total; i++) {
        const int s = int(i % S);
        if (!mbar_wait_bounded(&bars[s], uint32_t((i / S) & 1))) {
            // drain the copies still in flight into this warp's ring, then leave
            for (int64_t r = i + 1; r < total && r < i + S; r++) mbar_wait_bounded(&bars[r % S], uint32_t((r / S) & 1));
            return;
        }
        __syncwarp();
        const ChunkSpan cs = chunk_span<F>(a, i, nch, nbk, gw, G);
        F::template accumulate<MT>(ring + s * F::kStageBytes + cs.off, cs.nblk, int64_t(cs.ch) * F::kCB, a.act, k,
                                   acc, lane);
        __syncwarp();
        if (i + S < total) issue(i + S);
        if (cs.ch == nch - 1) {
#pragma unroll
            for (int t = 0; t < MT; t++) {
                const float v = warp_sum(acc[t]);
                if (lane == 0) a.y[cs.wi][t * a.y_stride[cs.wi] + cs.lrow] = v;
                acc[t] = 0.0f;
            }
        }
    }
}

}  // namespace cpq
