/*
 * cpq_oracle_gdn.c — CPU restatement of ggml's gated delta-net recurrence.
 *
 * TEST INFRASTRUCTURE ONLY (the parity checker of cpq_gated_delta_net; the
 * product never links or calls it).
 *
 * Restates ggml-cuda gated_delta_net.cu:4-167 (the op codpiece's GDN layers
 * call, qwen35.rs:2719), including its order of summation: a column's sums
 * are formed as the kernel's warp forms them, lane l adding rows l, l + w,
 * l + 2w, ... (w = min(32, S_v)) and the lanes then combined by the xor
 * butterfly of warp_reduce_sum (offsets w/2 .. 1).
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "cpq_oracle.h"

/* warp_reduce_sum over w lanes: p[l] += p[l ^ o] for o = w/2 .. 1; every lane ends equal */
static float butterfly(float *p, int w) {
    float n[32];
    for (int o = w / 2; o > 0; o >>= 1) {
        for (int l = 0; l < w; l++) n[l] = p[l] + p[l ^ o];
        memcpy(p, n, sizeof(float) * (size_t)w);
    }
    return p[0];
}

int oq_gated_delta_net(const float *q, const float *k, const float *v, const float *g, const float *beta,
                       const float *state, float *attn, float *state_out, int64_t sv, int64_t H, int64_t H_qk,
                       int64_t T, int64_t n_seqs, int64_t n_seqs_qk, int kda, int K, int64_t slot_stride) {
    if (sv < 1 || sv > 128 || H < 1 || H_qk < 1 || T < 1 || n_seqs < 1 || n_seqs_qk < 1 || n_seqs % n_seqs_qk) return -1;
    const int w = sv < 32 ? (int)sv : 32; /* lanes of the column's warp */
    const int rpl = (int)((sv + w - 1) / w);
    const int64_t rq3 = n_seqs / n_seqs_qk;
    const float scale = 1.0f / sqrtf((float)sv);
    float s[128], part[32];
    for (int64_t seq = 0; seq < n_seqs; seq++)
        for (int64_t h = 0; h < H; h++) {
            const int64_t iq1 = h % H_qk, iq3 = seq / rq3;
            const int64_t head = (seq * H + h) * sv * sv;
            for (int64_t col = 0; col < sv; col++) {
                for (int64_t i = 0; i < sv; i++) s[i] = state[head + col * sv + i];
                for (int64_t t = 0; t < T; t++) {
                    const float *qt = q + ((iq3 * T + t) * H_qk + iq1) * sv;
                    const float *kt = k + ((iq3 * T + t) * H_qk + iq1) * sv;
                    const int64_t gb = (seq * T + t) * H + h;
                    const float b = beta[gb];
                    const float vc = v[gb * sv + col];
                    float gexp = 0.0f;
                    if (!kda) gexp = expf(g[gb]);
                    for (int l = 0; l < w; l++) {
                        float acc = 0.0f;
                        for (int r = 0; r < rpl; r++) {
                            const int64_t i = (int64_t)r * w + l;
                            acc += kda ? expf(g[gb * sv + i]) * s[i] * kt[i] : s[i] * kt[i];
                        }
                        part[l] = acc;
                    }
                    const float kv = butterfly(part, w);
                    const float delta = kda ? (vc - kv) * b : (vc - gexp * kv) * b;
                    for (int l = 0; l < w; l++) {
                        float acc = 0.0f;
                        for (int r = 0; r < rpl; r++) {
                            const int64_t i = (int64_t)r * w + l;
                            const float gi = kda ? expf(g[gb * sv + i]) : gexp;
                            s[i] = gi * s[i] + kt[i] * delta;
                            acc += s[i] * qt[i];
                        }
                        part[l] = acc;
                    }
                    attn[((seq * T + t) * H + h) * sv + col] = butterfly(part, w) * scale;
                    if (K > 1) {
                        const int64_t slot = T - 1 - t;
                        if (slot < K)
                            for (int64_t i = 0; i < sv; i++) state_out[slot * slot_stride + head + col * sv + i] = s[i];
                    }
                }
                if (K <= 1)
                    for (int64_t i = 0; i < sv; i++) state_out[head + col * sv + i] = s[i];
            }
        }
    return 0;
}
