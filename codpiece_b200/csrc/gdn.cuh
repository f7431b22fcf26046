// gdn.cuh — the gated delta-net recurrence (ggml_gated_delta_net) for decode,
// speculative verify and prefill chunks.
//
// Semantics (ggml-cuda gated_delta_net.cu:4-167, called from
// qwen35.rs:2719): for every sequence, v head h (q/k head h % H_qk) and token
// t, with S the head's S_v x S_v state (S[i][col], stored column-major:
// element (i, col) at col * S_v + i) and gexp = exp(g):
//
//   kv[col]    = sum_i S[i][col] * k[i]                      (KDA: gexp[i] * S[i][col] * k[i])
//   delta[col] = (v[col] - gexp * kv[col]) * beta            (KDA: (v[col] - kv[col]) * beta)
//   S[i][col]  = gexp * S[i][col] + k[i] * delta[col]        (KDA: gexp[i] * S[i][col] + ...)
//   out[col]   = scale * sum_i S[i][col] * q[i]              scale = 1 / sqrt(S_v)
//
// and the state after the last token (or, with K > 1 snapshot slots, the
// state after token t in slot T - 1 - t when that is below K).
//
// Layout on the device. One CTA per (head, sequence, group of 16 columns);
// four threads per column, each holding S_v / 4 of the column's rows in
// registers as float4s: thread j of a column owns rows 4f .. 4f + 3 for
// f = j, j + 4, j + 8, ..., so that the four threads of a column read and
// write 64 contiguous bytes per access and a warp (8 columns) 512 bytes.
// The state is read once, stays in registers for all tokens, and is written
// once (plus the snapshots, with evict-first stores). q, k, v, g and beta of
// up to kGdnChunk tokens are staged in shared memory per chunk. The column
// sums are 4-lane butterflies (two shuffles), not warp-wide reductions.
//
// Roofline: HBM-bound. Bytes per launch = 4 * S_v^2 * H * n_seqs * (1 +
// slots written) + the per-token inputs and outputs.
#pragma once

#include "common.cuh"

namespace cpq {

constexpr int kGdnChunk = 16;  // tokens staged in shared memory at a time
// Columns of a head per CTA (at most): 16 puts twice the CTAs of 32 in flight
// (48 heads x 8 = 384 for decode): T = 1 3.45 vs 3.7 us, T = 8 with 8
// snapshots 9.3 vs 10.2 us; 8 was no better.
constexpr int kGdnCols = 16;

struct GdnArgs {
    const float *q, *k, *v, *g, *beta, *s_in;
    float *attn;   // [n_seqs][T][H][S_v]
    float *s_out;  // slot 0 of the state output
    int64_t H, T, neqk1, rq3;
    int64_t sq1, sq2, sq3, sv1, sv2, sv3, sb1, sb2, sb3;  // strides in floats
    int64_t slot_stride;                                  // floats between snapshot slots
    int K;                                                // snapshot slots (<= 1: the final state only)
    float scale;
};

__device__ __forceinline__ void st_cs_f4(float *p, float4 v) {
    asm volatile("st.global.cs.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
}

// Four independent partial sums (one per float4 lane), so that a thread's
// column sum is four chains of S_v / 16 FMAs rather than one of S_v / 4.
__device__ __forceinline__ void gdn_dot4(float4 s, float4 x, float4 &acc) {
    acc.x = fmaf(s.x, x.x, acc.x);
    acc.y = fmaf(s.y, x.y, acc.y);
    acc.z = fmaf(s.z, x.z, acc.z);
    acc.w = fmaf(s.w, x.w, acc.w);
}

__device__ __forceinline__ float gdn_sum4(float4 a) { return (a.x + a.y) + (a.z + a.w); }

template <int SV, bool KDA>
__global__ void __launch_bounds__((SV < kGdnCols ? SV : kGdnCols) * 4) gdn_kernel(const __grid_constant__ GdnArgs a) {
    constexpr int COLS = SV < kGdnCols ? SV : kGdnCols;  // columns per CTA
    constexpr int NF = SV / 16;              // float4s of the column per thread
    constexpr int NT = COLS * 4;
    __shared__ __align__(16) float qs[kGdnChunk][SV];
    __shared__ __align__(16) float ks[kGdnChunk][SV];
    __shared__ __align__(16) float gs[kGdnChunk][KDA ? SV : 1];
    __shared__ float vs[kGdnChunk][COLS];
    __shared__ float bs[kGdnChunk];

    const int tid = threadIdx.x, cl = tid >> 2, j = tid & 3;
    const int64_t h = blockIdx.x, seq = blockIdx.y;
    const int64_t col0 = int64_t(blockIdx.z) * COLS;
    const int64_t col = col0 + cl;
    const int64_t iq1 = h % a.neqk1, iq3 = seq / a.rq3;
    const int64_t head = (seq * a.H + h) * int64_t(SV) * SV;  // state offset of (seq, head)

    pdl_wait();
    float4 S[NF];
    {
        const float4 *src = reinterpret_cast<const float4 *>(a.s_in + head + col * SV);
#pragma unroll
        for (int u = 0; u < NF; u++) S[u] = __ldcs(src + j + 4 * u);
    }
    float *attn = a.attn + (seq * a.T * a.H + h) * SV + col;

    for (int64_t t0 = 0; t0 < a.T; t0 += kGdnChunk) {
        const int nt = int(a.T - t0 < kGdnChunk ? a.T - t0 : kGdnChunk);
        __syncthreads();  // the previous chunk's values are consumed
        for (int x = tid; x < nt * SV; x += NT) {
            const int t = x / SV, i = x % SV;
            const int64_t off = iq3 * a.sq3 + (t0 + t) * a.sq2 + iq1 * a.sq1 + i;
            qs[t][i] = a.q[off];
            ks[t][i] = a.k[off];
        }
        for (int x = tid; x < nt * COLS; x += NT) {
            const int t = x / COLS, c = x % COLS;
            vs[t][c] = a.v[seq * a.sv3 + (t0 + t) * a.sv2 + h * a.sv1 + col0 + c];
        }
        for (int x = tid; x < nt * (KDA ? SV : 1); x += NT) {
            const int t = KDA ? x / SV : x, i = KDA ? x % SV : 0;
            const int64_t gb = seq * a.sb3 + (t0 + t) * a.sb2 + h * a.sb1;
            gs[t][i] = expf(a.g[gb * (KDA ? SV : 1) + i]);
            if (i == 0) bs[t] = a.beta[gb];
        }
        __syncthreads();

#pragma unroll 1
        for (int t = 0; t < nt; t++) {
            const float4 *k4 = reinterpret_cast<const float4 *>(ks[t]);
            const float4 *q4 = reinterpret_cast<const float4 *>(qs[t]);
            float4 kv4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            if constexpr (KDA) {
                const float4 *g4 = reinterpret_cast<const float4 *>(gs[t]);
#pragma unroll
                for (int u = 0; u < NF; u++) {
                    const float4 gg = g4[j + 4 * u], s = S[u];
                    gdn_dot4(make_float4(gg.x * s.x, gg.y * s.y, gg.z * s.z, gg.w * s.w), k4[j + 4 * u], kv4);
                }
            } else {
#pragma unroll
                for (int u = 0; u < NF; u++) gdn_dot4(S[u], k4[j + 4 * u], kv4);
            }
            float kv = gdn_sum4(kv4);
            kv += __shfl_xor_sync(0xffffffffu, kv, 1);
            kv += __shfl_xor_sync(0xffffffffu, kv, 2);
            const float gexp = gs[t][0];
            const float delta = KDA ? (vs[t][cl] - kv) * bs[t] : (vs[t][cl] - gexp * kv) * bs[t];
            float4 o4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
            for (int u = 0; u < NF; u++) {
                const float4 kk = k4[j + 4 * u];
                float4 g = make_float4(gexp, gexp, gexp, gexp);
                if constexpr (KDA) g = reinterpret_cast<const float4 *>(gs[t])[j + 4 * u];
                float4 &s = S[u];
                s.x = fmaf(g.x, s.x, kk.x * delta);
                s.y = fmaf(g.y, s.y, kk.y * delta);
                s.z = fmaf(g.z, s.z, kk.z * delta);
                s.w = fmaf(g.w, s.w, kk.w * delta);
                gdn_dot4(s, q4[j + 4 * u], o4);
            }
            float o = gdn_sum4(o4);
            o += __shfl_xor_sync(0xffffffffu, o, 1);
            o += __shfl_xor_sync(0xffffffffu, o, 2);
            if (j == 0) attn[(t0 + t) * a.H * SV] = o * a.scale;
            if (a.K > 1) {
                const int64_t slot = a.T - 1 - (t0 + t);
                if (slot < a.K) {
                    float *dst = a.s_out + slot * a.slot_stride + head + col * SV;
#pragma unroll
                    for (int u = 0; u < NF; u++) st_cs_f4(dst + 4 * (j + 4 * u), S[u]);
                }
            }
        }
    }
    if (a.K <= 1) {
        float *dst = a.s_out + head + col * SV;
#pragma unroll
        for (int u = 0; u < NF; u++) st_cs_f4(dst + 4 * (j + 4 * u), S[u]);
    }
}

}  // namespace cpq
