// plan.inl — cpq_decode_plan_*: host side of the persistent decode kernel (decode.cuh).
//
// A plan is the device-side description of a decode chain: one DecPhase per
// phase, one DecWeight (TMA tensor map + output pointer) per weight, the
// stream-K scratch (per-warp piece words, per-row-block counters) and the
// grid-barrier counter. Creating it validates every phase with the same
// checks as cpq_mul_mat_fused; running it clears the counters and the
// barrier and launches one cooperative grid of one CTA per SM.

struct cpq_decode_plan {
    int device = -1;
    int n_ph = 0;
    int grid = 0;
    int smem = 0;
    int act_bytes = 0;
    cpq::DecPhase *d_ph = nullptr;
    cpq::DecWeight *d_w = nullptr;
    uint64_t *pieces = nullptr;
    int *counters = nullptr;
    size_t counter_bytes = 0;
    unsigned *bar = nullptr;
    uint8_t *act_g = nullptr;
};

namespace cpq {

static void plan_free(cpq_decode_plan *p) {
    if (!p) return;
    int cur = -1;
    cudaGetDevice(&cur);
    if (p->device >= 0) cudaSetDevice(p->device);
    cudaFree(p->d_ph);
    cudaFree(p->d_w);
    cudaFree(p->pieces);
    cudaFree(p->counters);
    cudaFree(p->bar);
    cudaFree(p->act_g);
    if (cur >= 0) cudaSetDevice(cur);
    delete p;
}

static cpq_status check_vec(const void *p, const char *what, int i) {
    if (!p) return fail(CPQ_ERR_INVALID_ARG, "decode phase %d: %s is null", i, what);
    if (!aligned(p, 16)) return fail(CPQ_ERR_UNSUPPORTED, "decode phase %d: %s is not 16-byte aligned", i, what);
    return CPQ_SUCCESS;
}

}  // namespace cpq

extern "C" cpq_status cpq_decode_plan_create(const cpq_decode_phase *phases, int n_phases, int device,
                                             cpq_decode_plan **out) {
    using namespace cpq;
    if (!out) return fail(CPQ_ERR_INVALID_ARG, "cpq_decode_plan_create: plan pointer is null");
    *out = nullptr;
    if (!phases || n_phases < 1 || n_phases > 65536)
        return fail(CPQ_ERR_INVALID_ARG, "cpq_decode_plan_create: n_phases=%d must be in 1..65536", n_phases);
    if (device < 0 || device >= kMaxDevices) return fail(CPQ_ERR_INVALID_ARG, "device %d", device);

    std::vector<DecPhase> ph(static_cast<size_t>(n_phases));
    std::vector<DecWeight> wt;
    int64_t max_mb = 1;
    int act_bytes = 0;
    for (int i = 0; i < n_phases; i++) {
        const cpq_decode_phase &q = phases[i];
        if (q.mode != CPQ_PRO_NONE && q.mode != CPQ_PRO_RMS && q.mode != CPQ_PRO_SWIGLU)
            return fail(CPQ_ERR_INVALID_ARG, "decode phase %d: prologue mode %d", i, int(q.mode));
        if (q.n_w < 1 || q.n_w > kDecMaxW)
            return fail(CPQ_ERR_INVALID_ARG, "decode phase %d: n_w=%d must be in 1..%d", i, int(q.n_w), kDecMaxW);
        cpq_status rc;
        if ((rc = check_vec(q.x, "x", i))) return rc;
        if (q.mode == CPQ_PRO_SWIGLU && (rc = check_vec(q.r, "r (up)", i))) return rc;
        if (q.r && (rc = check_vec(q.r, "r", i))) return rc;
        if (q.h_out && (rc = check_vec(q.h_out, "h_out", i))) return rc;
        if (q.h_out && (q.h_out == q.x || q.h_out == q.r))
            return fail(CPQ_ERR_INVALID_ARG, "decode phase %d: h_out aliases an input", i);
        DecPhase &P = ph[size_t(i)];
        std::memset(&P, 0, sizeof P);
        P.mode = q.mode;
        P.n_w = q.n_w;
        P.w0 = int(wt.size());
        P.x = q.x;
        P.r = q.r;
        P.g = q.g;
        P.h_out = q.mode == CPQ_PRO_RMS ? q.h_out : nullptr;
        P.eps = q.eps;
        int64_t k = -1;
        size_t rs = 0;
        for (int j = 0; j < q.n_w; j++) {
            MMShape s;
            if ((rc = check_weight(q.w[j], &s))) return rc;
            if (s.wtype != CPQ_TYPE_Q4_K)
                return fail(CPQ_ERR_UNSUPPORTED, "decode phase %d: weight %d is %s (plans run Q4_K)", i, j,
                            type_name(s.wtype));
            if (j == 0) {
                k = s.k;
                rs = q.w[j]->nb[1];
            } else if (s.k != k || q.w[j]->nb[1] != rs) {
                return fail(CPQ_ERR_INVALID_ARG, "decode phase %d: weights must share K and row stride", i);
            }
            if (s.n < 1) return fail(CPQ_ERR_INVALID_ARG, "decode phase %d: weight %d has no rows", i, j);
            if ((rc = check_vec(q.y[j], "y", i))) return rc;
            DecWeight W;
            std::memset(&W, 0, sizeof W);
            if ((rc = q4k_tensor_map(static_cast<const uint8_t *>(q.w[j]->data), s.n, s.k, rs, &W.tmap, kRowRows, 1)))
                return rc;
            W.y = q.y[j];
            W.n = s.n;
            wt.push_back(W);
            P.mb_start[j + 1] = P.mb_start[j] + (s.n + kRowRows - 1) / kRowRows;
        }
        for (int j = q.n_w; j < kDecMaxW; j++) P.mb_start[j + 1] = P.mb_start[q.n_w];
        P.nbk = int(k / kQK_K);
        max_mb = std::max<int64_t>(max_mb, P.mb_start[q.n_w]);
        act_bytes = std::max(act_bytes, row_act_bytes(k, 1));
    }
    const int smem = kDecBarBytes + act_bytes + kDecRingBytes;
    if (smem > kSmemMax)
        return fail(CPQ_ERR_UNSUPPORTED, "decode plan: K too large (%d B of shared memory needed)", smem);

    int cur = -1;
    cudaGetDevice(&cur);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cpq_decode_plan_create: cudaSetDevice");
    cpq_decode_plan *p = new cpq_decode_plan;
    p->device = device;
    p->n_ph = n_phases;
    p->act_bytes = act_bytes;
    p->smem = smem;
    auto done = [&](cpq_status s) {
        if (cur >= 0) cudaSetDevice(cur);
        if (s != CPQ_SUCCESS) plan_free(p);
        return s;
    };
    e = cudaFuncSetAttribute(decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return done(cuda_fail(e, "decode plan: shared-memory attribute"));
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, decode_step_kernel, kDecWarps * 32, size_t(smem));
    if (e != cudaSuccess || per_sm < 1) return done(fail(CPQ_ERR_CUDA, "decode plan: kernel does not fit on an SM"));
    p->grid = sm_count(device);
    p->counter_bytes = align_up(size_t(max_mb) * sizeof(int), 256);
    const size_t piece_bytes = size_t(p->grid) * kDecWarps * 2 * kPieceWords * sizeof(uint64_t);
    if ((e = cudaMalloc(&p->d_ph, ph.size() * sizeof(DecPhase))) != cudaSuccess ||
        (e = cudaMalloc(&p->d_w, wt.size() * sizeof(DecWeight))) != cudaSuccess ||
        (e = cudaMalloc(&p->pieces, piece_bytes)) != cudaSuccess ||
        (e = cudaMalloc(&p->counters, p->counter_bytes)) != cudaSuccess ||
        (e = cudaMalloc(&p->bar, 256)) != cudaSuccess ||
        (e = cudaMalloc(&p->act_g, size_t(act_bytes))) != cudaSuccess)
        return done(cuda_fail(e, "decode plan: cudaMalloc"));
    if ((e = cudaMemcpy(p->d_ph, ph.data(), ph.size() * sizeof(DecPhase), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(p->d_w, wt.data(), wt.size() * sizeof(DecWeight), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemset(p->pieces, 0, piece_bytes)) != cudaSuccess)
        return done(cuda_fail(e, "decode plan: table upload"));
    *out = p;
    return done(CPQ_SUCCESS);
}

extern "C" cpq_status cpq_decode_plan_run(cpq_decode_plan *p, void *stream) {
    using namespace cpq;
    if (!p) return fail(CPQ_ERR_INVALID_ARG, "cpq_decode_plan_run: plan is null");
    if (current_device() != p->device)
        return fail(CPQ_ERR_INVALID_ARG, "cpq_decode_plan_run: plan belongs to device %d, current is %d", p->device,
                    current_device());
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    cudaError_t e = cudaMemsetAsync(p->counters, 0, p->counter_bytes, st);
    if (e == cudaSuccess) e = cudaMemsetAsync(p->bar, 0, sizeof(unsigned), st);
    if (e != cudaSuccess) return cuda_fail(e, "cpq_decode_plan_run: clearing the scratch");
    DecArgs a;
    a.ph = p->d_ph;
    a.w = p->d_w;
    a.n_ph = p->n_ph;
    a.act_bytes = p->act_bytes;
    a.pieces = p->pieces;
    a.counters = p->counters;
    a.bar = p->bar;
    a.act_g = p->act_g;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(p->grid));
    cfg.blockDim = dim3(kDecWarps * 32);
    cfg.dynamicSmemBytes = size_t(p->smem);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // all CTAs resident: the phases meet at grid barriers
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, decode_step_kernel, a);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "cpq_decode_plan_run: launch");
}

extern "C" void cpq_decode_plan_destroy(cpq_decode_plan *p) { cpq::plan_free(p); }
