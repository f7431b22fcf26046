// gdn.inl — cpq_gated_delta_net: host side of gdn.cuh.
//
// Replaces ggml_cuda_op_gated_delta_net and its _fused_cache variant
// (ggml-cuda gated_delta_net.cuh:10-14, gated_delta_net.cu:223-327): the same
// source tensors (q, k, v, g, beta, state), the same op parameter K (snapshot
// slots), the attention rows at the start of dst and the state(s) after them,
// or in a caller's cache when one is given.

namespace cpq {

static bool f32_rows(const cpq_tensor *t) { return t && t->type == CPQ_TYPE_F32 && t->data && t->nb[0] == 4; }

static bool f32_contiguous(const cpq_tensor *t) {
    if (!f32_rows(t)) return false;
    size_t nb = 4;
    for (int d = 0; d < 4; d++) {
        if (t->ne[d] < 1) return false;
        if (t->ne[d] > 1 && t->nb[d] != nb) return false;
        nb *= size_t(t->ne[d]);
    }
    return true;
}

static int64_t nelem(const cpq_tensor *t) { return t->ne[0] * t->ne[1] * t->ne[2] * t->ne[3]; }

template <int SV, bool KDA>
static cudaError_t launch_gdn_t(const GdnArgs &a, int64_t n_seqs, cudaStream_t st) {
    constexpr int cols = SV < kGdnCols ? SV : kGdnCols;
    return launch(gdn_kernel<SV, KDA>, dim3(unsigned(a.H), unsigned(n_seqs), unsigned(SV / cols)), dim3(cols * 4), 0, st,
                  a);
}

template <bool KDA>
static cudaError_t launch_gdn(int64_t sv, const GdnArgs &a, int64_t n_seqs, cudaStream_t st) {
    switch (sv) {
        case 16: return launch_gdn_t<16, KDA>(a, n_seqs, st);
        case 32: return launch_gdn_t<32, KDA>(a, n_seqs, st);
        case 64: return launch_gdn_t<64, KDA>(a, n_seqs, st);
        default: return launch_gdn_t<128, KDA>(a, n_seqs, st);
    }
}

}  // namespace cpq

extern "C" cpq_status cpq_gated_delta_net(const cpq_tensor *q, const cpq_tensor *k, const cpq_tensor *v,
                                          const cpq_tensor *g, const cpq_tensor *beta, const cpq_tensor *state,
                                          cpq_tensor *dst, int32_t n_snap, float *cache, int64_t cache_slot_stride,
                                          void *stream) {
    using namespace cpq;
    if (!f32_rows(q) || !f32_rows(k) || !f32_rows(v))
        return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: q, k and v must be F32 tensors with contiguous rows");
    if (!f32_contiguous(g) || !f32_contiguous(beta) || !f32_contiguous(state) || !f32_contiguous(dst))
        return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: g, beta, state and dst must be contiguous F32 tensors");
    for (int d = 1; d < 4; d++)
        if (q->nb[d] % 4 || v->nb[d] % 4)
            return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: q, k and v strides must be whole floats");
    const int64_t sv = v->ne[0], H = v->ne[1], T = v->ne[2], n_seqs = v->ne[3];
    if (sv != 16 && sv != 32 && sv != 64 && sv != 128)
        return fail(CPQ_ERR_UNSUPPORTED, "gated_delta_net: S_v=%lld (16, 32, 64 or 128)", (long long)sv);
    if (H < 1 || T < 1 || n_seqs < 1 || H > 2147483647 || n_seqs > 65535)
        return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: v has ne=[%lld, %lld, %lld, %lld]", (long long)sv,
                    (long long)H, (long long)T, (long long)n_seqs);
    for (int d = 0; d < 4; d++)
        if (q->ne[d] != k->ne[d] || q->nb[d] != k->nb[d])
            return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: q and k differ in shape or strides");
    if (q->ne[0] != sv || q->ne[1] < 1 || q->ne[2] != T || q->ne[3] < 1 || n_seqs % q->ne[3])
        return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: q ne=[%lld, %lld, %lld, %lld] does not fit v's",
                    (long long)q->ne[0], (long long)q->ne[1], (long long)q->ne[2], (long long)q->ne[3]);
    const bool kda = g->ne[0] == sv;
    if ((g->ne[0] != 1 && !kda) || g->ne[1] != H || g->ne[2] != T || g->ne[3] != n_seqs)
        return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: g must be [1 or S_v, H, T, n_seqs]");
    if (beta->ne[0] != 1 || beta->ne[1] != H || beta->ne[2] != T || beta->ne[3] != n_seqs)
        return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: beta must be [1, H, T, n_seqs]");
    const int64_t D = sv * sv * H;  // one sequence's state
    if (nelem(state) != D * n_seqs)
        return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: state has %lld elements, expected S_v*S_v*H*n_seqs = %lld",
                    (long long)nelem(state), (long long)(D * n_seqs));
    if (n_snap < 0) return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: K=%d", n_snap);
    const int64_t slots = n_snap > 1 ? std::min<int64_t>(n_snap, T) : 1;  // state slots written
    const int64_t n_attn = sv * H * T * n_seqs;
    float *s_out;
    int64_t slot_stride;
    if (cache) {
        s_out = cache;
        slot_stride = cache_slot_stride;
        if (slots > 1 && slot_stride < D * n_seqs)
            return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: cache slot stride %lld < one state set (%lld)",
                        (long long)slot_stride, (long long)(D * n_seqs));
    } else {
        s_out = static_cast<float *>(dst->data) + n_attn;
        slot_stride = D * n_seqs;
    }
    if (nelem(dst) < n_attn + (cache ? 0 : slots * D * n_seqs))
        return fail(CPQ_ERR_INVALID_ARG, "gated_delta_net: dst holds %lld floats, needs %lld", (long long)nelem(dst),
                    (long long)(n_attn + (cache ? 0 : slots * D * n_seqs)));
    if (!aligned(state->data, 16) || !aligned(s_out, 16) || slot_stride % 4)
        return fail(CPQ_ERR_UNSUPPORTED, "gated_delta_net: state input and output must be 16-byte aligned");

    GdnArgs a{};
    a.q = static_cast<const float *>(q->data);
    a.k = static_cast<const float *>(k->data);
    a.v = static_cast<const float *>(v->data);
    a.g = static_cast<const float *>(g->data);
    a.beta = static_cast<const float *>(beta->data);
    a.s_in = static_cast<const float *>(state->data);
    a.attn = static_cast<float *>(dst->data);
    a.s_out = s_out;
    a.H = H;
    a.T = T;
    a.neqk1 = q->ne[1];
    a.rq3 = n_seqs / q->ne[3];
    a.sq1 = int64_t(q->nb[1] / 4);
    a.sq2 = int64_t(q->nb[2] / 4);
    a.sq3 = int64_t(q->nb[3] / 4);
    a.sv1 = int64_t(v->nb[1] / 4);
    a.sv2 = int64_t(v->nb[2] / 4);
    a.sv3 = int64_t(v->nb[3] / 4);
    a.sb1 = int64_t(beta->nb[1] / 4);
    a.sb2 = int64_t(beta->nb[2] / 4);
    a.sb3 = int64_t(beta->nb[3] / 4);
    a.slot_stride = slot_stride;
    a.K = n_snap;
    a.scale = 1.0f / sqrtf(float(sv));
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const cudaError_t e = kda ? launch_gdn<true>(sv, a, n_seqs, st) : launch_gdn<false>(sv, a, n_seqs, st);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "gated_delta_net launch");
}
