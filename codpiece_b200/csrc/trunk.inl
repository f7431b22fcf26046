// trunk.inl — cpq_trunk_*: host side of the persistent decode trunk (trunk.cuh).
//
// cpq_trunk_create turns a rank's layers into the kernel's phase table:
//
//   q/k/v   RMS image of R (attn_norm), after folding the pending all-reduces
//   o       plain image of q; one rank: R += o (kTrOutResid), else LL words to every rank
//   gate/up RMS image of R (ffn_norm), pending folds; stores silu(gate) * up
//   down    plain image of silu(gate) * up; one rank: R += down, else LL words
//
// and, under tensor parallelism, a last fold-only phase for the final
// all-reduce. h_out receives the residual stream after the last layer, the
// input of the LM head's RMS norm (qwen35.rs:2797).

struct cpq_trunk {
    int device = -1;
    int n_ph = 0;
    int grid = 0;
    int smem = 0;
    int act_bytes = 0;
    unsigned n_ar = 0;
    int64_t n_embd = 0;
    cpq::TrPhase *d_ph = nullptr;
    cpq::TrWeight *d_w = nullptr;
    uint64_t *R = nullptr, *QB = nullptr, *AB = nullptr, *pieces = nullptr;
    unsigned *cnt = nullptr, *ctl = nullptr;
    float *kv = nullptr;
    cpq_tp_ar *ar = nullptr;
};

namespace cpq {

static void trunk_free(cpq_trunk *t) {
    if (!t) return;
    int cur = -1;
    cudaGetDevice(&cur);
    if (t->device >= 0) cudaSetDevice(t->device);
    cudaFree(t->d_ph);
    cudaFree(t->d_w);
    cudaFree(t->R);
    cudaFree(t->QB);
    cudaFree(t->AB);
    cudaFree(t->pieces);
    cudaFree(t->cnt);
    cudaFree(t->ctl);
    cudaFree(t->kv);
    if (cur >= 0) cudaSetDevice(cur);
    delete t;
}

// A Q4_K weight of a trunk layer: type, K and N as expected (n < 0: any N >= 1).
static cpq_status trunk_weight(const cpq_tensor *w, const char *what, int il, int64_t k, int64_t n, MMShape *s) {
    if (!w) return fail(CPQ_ERR_INVALID_ARG, "trunk layer %d: %s is null", il, what);
    cpq_status rc = check_weight(w, s);
    if (rc) return rc;
    if (s->wtype != CPQ_TYPE_Q4_K)
        return fail(CPQ_ERR_UNSUPPORTED, "trunk layer %d: %s is %s (the trunk runs Q4_K)", il, what, type_name(s->wtype));
    if (s->k != k)
        return fail(CPQ_ERR_INVALID_ARG, "trunk layer %d: %s has K=%lld, expected %lld", il, what, (long long)s->k,
                    (long long)k);
    if (s->n < 1 || (n >= 0 && s->n != n))
        return fail(CPQ_ERR_INVALID_ARG, "trunk layer %d: %s has N=%lld, expected %lld", il, what, (long long)s->n,
                    (long long)n);
    return CPQ_SUCCESS;
}

}  // namespace cpq

extern "C" cpq_status cpq_trunk_create(const cpq_trunk_layer *layers, int n_layers, int64_t n_embd, float eps,
                                       cpq_tp_ar *ar, int device, cpq_trunk **out) {
    using namespace cpq;
    if (!out) return fail(CPQ_ERR_INVALID_ARG, "cpq_trunk_create: output pointer is null");
    *out = nullptr;
    if (!layers || n_layers < 1 || n_layers > 4096)
        return fail(CPQ_ERR_INVALID_ARG, "cpq_trunk_create: n_layers=%d must be in 1..4096", n_layers);
    if (device < 0 || device >= kMaxDevices) return fail(CPQ_ERR_INVALID_ARG, "cpq_trunk_create: device %d", device);
    if (n_embd < kQK_K || n_embd % kQK_K || n_embd > int64_t(kQK_K) * 8 * kTrRmsBlocks)
        return fail(CPQ_ERR_UNSUPPORTED, "cpq_trunk_create: n_embd=%lld must be a multiple of 256 up to %d",
                    (long long)n_embd, kQK_K * 8 * kTrRmsBlocks);
    int world = 1, rank = 0;
    if (ar) {
        if (!ar->connected) return fail(CPQ_ERR_INVALID_ARG, "cpq_trunk_create: the channel is not connected");
        if (ar->device != device)
            return fail(CPQ_ERR_INVALID_ARG, "cpq_trunk_create: the channel is on device %d", ar->device);
        if (ar->n_max < n_embd) return fail(CPQ_ERR_INVALID_ARG, "cpq_trunk_create: channel n_max < n_embd");
        world = ar->world;
        rank = ar->rank;
    }
    const unsigned all = (1u << world) - 1u;
    const int grid = sm_count(device);

    std::vector<TrPhase> ph;
    std::vector<TrWeight> wt;
    int64_t max_q = 1, max_ff = 1, max_kv = 1;
    int act_bytes = row_act_bytes(n_embd, 1);
    int r_pub = -1;                                     // phase that last published R (-1: the run's input)
    int r_cnt = 0;                                      // ... its counter and how many CTAs complete it
    unsigned r_target = unsigned(grid);
    std::vector<std::pair<unsigned, unsigned>> pending;  // (all-reduce index, contributing ranks)
    unsigned ar_idx = 0;
    cpq_status rc;
    auto add_weight = [&](const cpq_tensor *w, const MMShape &s, int box_rows) -> cpq_status {
        TrWeight W;
        std::memset(&W, 0, sizeof W);
        cpq_status r = q4k_tensor_map(static_cast<const uint8_t *>(w->data), s.n, s.k, w->nb[1], &W.tmap, box_rows, 1);
        if (r) return r;
        wt.push_back(W);
        return CPQ_SUCCESS;
    };
    auto new_phase = [&]() {
        TrPhase P;
        std::memset(&P, 0, sizeof P);
        P.w0 = int(wt.size());
        P.eps = eps;
        P.r_prev = r_pub;
        return P;
    };
    // an RMS input: fold the pending all-reduces into R here (then this phase publishes R)
    auto take_folds = [&](TrPhase &P) {
        if (pending.empty()) {
            P.in_pub = r_pub;
            return;
        }
        P.n_fold = int(pending.size());
        for (size_t f = 0; f < pending.size(); f++) {
            P.fold_seq[f] = pending[f].first;
            P.fold_mask[f] = pending[f].second;
        }
        pending.clear();
        P.in_pub = int(ph.size());
        r_pub = P.in_pub;
    };
    auto finish = [&](TrPhase &P) {  // row blocks -> CTAs with work; the counter of the phase's input
        if (P.n_w > 0) {
            const int64_t rb = P.mb_start[P.n_w];
            P.ctas = int(std::min<int64_t>(grid, rb));
            // whole row blocks per CTA when that costs a warp no more stages than the balanced
            // split, or one more when phases are a few stages per warp (the small shards of tensor
            // parallelism: there the balanced split's block cuts, which make CTAs wait on their
            // neighbours' words, cost more than a stage; TP8-shaped trunk 34.1 -> 31.3 us/layer)
            const int64_t whole_stages = ((rb + P.ctas - 1) / P.ctas * P.nbk + kTrWarps - 1) / kTrWarps;
            const int64_t range_stages = (rb * P.nbk + int64_t(P.ctas) * kTrWarps - 1) / (int64_t(P.ctas) * kTrWarps);
            P.whole = whole_stages <= range_stages || (range_stages <= 4 && whole_stages <= range_stages + 1);
        }
        const int idx = int(ph.size());
        if (P.n_fold > 0) {
            r_cnt = 1 + 2 * idx;
            r_target = unsigned(grid);
        }
        if (P.in_kind == kTrInR) {
            P.in_cnt = r_cnt;
            P.in_target = r_target;
        } else {
            P.in_cnt = 2 + 2 * P.in_pub;
            P.in_target = unsigned(ph[size_t(P.in_pub)].ctas);
        }
        if (P.out_kind == kTrOutResid && P.n_w > 0) {  // this phase's outputs publish R
            r_pub = idx;
            r_cnt = 2 + 2 * idx;
            r_target = unsigned(P.ctas);
        }
        ph.push_back(P);
        return idx;
    };
    for (int il = 0; il < n_layers; il++) {
        const cpq_trunk_layer &L = layers[il];
        const unsigned o_mask = L.o_ranks ? L.o_ranks : all;
        if (world > 1 && (o_mask & ~all))
            return fail(CPQ_ERR_INVALID_ARG, "trunk layer %d: o_ranks 0x%x names ranks outside the group", il, o_mask);
        if ((L.q == nullptr) != (L.o == nullptr))
            return fail(CPQ_ERR_INVALID_ARG, "trunk layer %d: q and o must both be given or both be NULL", il);
        if (L.q) {
            if (world > 1 && !((o_mask >> rank) & 1u))
                return fail(CPQ_ERR_INVALID_ARG, "trunk layer %d: this rank holds q but is not in o_ranks", il);
            // ---- q/k/v ----
            TrPhase P = new_phase();
            P.in_kind = kTrInR;
            P.g = L.attn_norm;
            P.out_kind = kTrOutVec;
            const cpq_tensor *qkv[3] = {L.q, L.k, L.v};
            const char *names[3] = {"q", "k", "v"};
            MMShape sq = {};
            for (int j = 0; j < 3; j++) {
                if (!qkv[j]) continue;
                MMShape s;
                if ((rc = trunk_weight(qkv[j], names[j], il, n_embd, -1, &s))) return rc;
                if (j == 0) sq = s;
                if ((rc = add_weight(qkv[j], s, kRowRows))) return rc;
                P.n[P.n_w] = s.n;
                P.mb_start[P.n_w + 1] = P.mb_start[P.n_w] + (s.n + kRowRows - 1) / kRowRows;
                if (P.n_w > 0) max_kv = std::max(max_kv, s.n);
                P.n_w++;
            }
            for (int j = P.n_w; j < kTrMaxW; j++) P.mb_start[j + 1] = P.mb_start[P.n_w];
            if (sq.n % kQK_K)
                return fail(CPQ_ERR_UNSUPPORTED, "trunk layer %d: q rows %lld not a multiple of 256", il, (long long)sq.n);
            P.nbk = int(n_embd / kQK_K);
            max_q = std::max(max_q, sq.n);
            take_folds(P);
            const int p_qkv = finish(P);
            // ---- o ----
            TrPhase O = new_phase();
            O.in_kind = kTrInVec;
            O.in_buf = kTrBufQ;
            O.in_pub = p_qkv;
            MMShape so;
            if ((rc = trunk_weight(L.o, "o", il, sq.n, n_embd, &so))) return rc;
            if ((rc = add_weight(L.o, so, kRowRows))) return rc;
            O.n_w = 1;
            O.n[0] = so.n;
            O.mb_start[1] = O.mb_start[2] = O.mb_start[3] = (so.n + kRowRows - 1) / kRowRows;
            O.nbk = int(sq.n / kQK_K);
            act_bytes = std::max(act_bytes, row_act_bytes(sq.n, 1));
            if (world == 1) {
                O.out_kind = kTrOutResid;
            } else {
                O.out_kind = kTrOutAr;
                O.out_seq = ar_idx;
                pending.emplace_back(ar_idx++, o_mask);
            }
            finish(O);
        } else {
            if (world == 1) return fail(CPQ_ERR_INVALID_ARG, "trunk layer %d: q/o missing on a single rank", il);
            if ((o_mask >> rank) & 1u)
                return fail(CPQ_ERR_INVALID_ARG, "trunk layer %d: o_ranks names this rank, which holds no q", il);
            pending.emplace_back(ar_idx++, o_mask);  // the other ranks' o all-reduce
        }
        // ---- gate/up pairs ----
        MMShape sg, su, sd;
        if ((rc = trunk_weight(L.gate, "gate", il, n_embd, -1, &sg))) return rc;
        if ((rc = trunk_weight(L.up, "up", il, n_embd, sg.n, &su))) return rc;
        if (sg.n % kQK_K)
            return fail(CPQ_ERR_UNSUPPORTED, "trunk layer %d: ffn rows %lld not a multiple of 256", il, (long long)sg.n);
        TrPhase G = new_phase();
        G.in_kind = kTrInR;
        G.g = L.ffn_norm;
        G.out_kind = kTrOutPair;
        G.pair = 1;
        if ((rc = add_weight(L.gate, sg, 16)) || (rc = add_weight(L.up, su, 16))) return rc;
        G.n_w = 2;
        G.n[0] = sg.n;
        G.mb_start[1] = G.mb_start[2] = G.mb_start[3] = (sg.n + 15) / 16;
        G.nbk = int(n_embd / kQK_K);
        max_ff = std::max(max_ff, sg.n);
        take_folds(G);
        const int p_gu = finish(G);
        // ---- down ----
        TrPhase D = new_phase();
        D.in_kind = kTrInVec;
        D.in_buf = kTrBufA;
        D.in_pub = p_gu;
        if ((rc = trunk_weight(L.down, "down", il, sg.n, n_embd, &sd))) return rc;
        if ((rc = add_weight(L.down, sd, kRowRows))) return rc;
        D.n_w = 1;
        D.n[0] = sd.n;
        D.mb_start[1] = D.mb_start[2] = D.mb_start[3] = (sd.n + kRowRows - 1) / kRowRows;
        D.nbk = int(sg.n / kQK_K);
        act_bytes = std::max(act_bytes, row_act_bytes(sg.n, 1));
        if (world == 1) {
            D.out_kind = kTrOutResid;
        } else {
            D.out_kind = kTrOutAr;
            D.out_seq = ar_idx;
            pending.emplace_back(ar_idx++, all);
        }
        finish(D);
    }
    if (!pending.empty()) {  // the last all-reduce, folded into R and stored to h_out
        TrPhase F = new_phase();
        take_folds(F);
        F.write_h = 1;
        finish(F);
    } else {
        ph.back().write_h = 1;  // the last down's residual add
    }
    const int smem = kTrHdrBytes + act_bytes + kTrRingBytes + row_red_bytes(1);
    if (smem > kSmemMax)
        return fail(CPQ_ERR_UNSUPPORTED, "cpq_trunk_create: a layer's K is too large (%d B of shared memory)", smem);

    int cur = -1;
    cudaGetDevice(&cur);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cpq_trunk_create: cudaSetDevice");
    cpq_trunk *t = new cpq_trunk;
    t->device = device;
    t->n_ph = int(ph.size());
    t->grid = grid;
    t->smem = smem;
    t->act_bytes = act_bytes;
    t->n_ar = ar_idx;
    t->n_embd = n_embd;
    t->ar = ar;
    auto done = [&](cpq_status s) {
        if (cur >= 0) cudaSetDevice(cur);
        if (s != CPQ_SUCCESS) trunk_free(t);
        return s;
    };
    e = cudaFuncSetAttribute(trunk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return done(cuda_fail(e, "cpq_trunk_create: shared-memory attribute"));
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, trunk_kernel, kTrThreads, size_t(smem));
    if (e != cudaSuccess || per_sm < 1)
        return done(fail(CPQ_ERR_CUDA, "cpq_trunk_create: the kernel does not fit on an SM"));
    const size_t piece_bytes = size_t(2) * grid * kTrWarps * 32 * sizeof(uint64_t);
    const size_t cnt_bytes = (size_t(2) * ph.size() + 1) * sizeof(unsigned);
    if ((e = cudaMalloc(&t->d_ph, ph.size() * sizeof(TrPhase))) != cudaSuccess ||
        (e = cudaMalloc(&t->d_w, std::max<size_t>(1, wt.size()) * sizeof(TrWeight))) != cudaSuccess ||
        (e = cudaMalloc(&t->R, size_t(n_embd) * 8)) != cudaSuccess ||
        (e = cudaMalloc(&t->QB, size_t(max_q) * 8)) != cudaSuccess ||
        (e = cudaMalloc(&t->AB, size_t(max_ff) * 8)) != cudaSuccess ||
        (e = cudaMalloc(&t->pieces, piece_bytes)) != cudaSuccess ||
        (e = cudaMalloc(&t->cnt, cnt_bytes)) != cudaSuccess || (e = cudaMalloc(&t->ctl, 256)) != cudaSuccess ||
        (e = cudaMalloc(&t->kv, size_t(2) * max_kv * 4)) != cudaSuccess)
        return done(cuda_fail(e, "cpq_trunk_create: cudaMalloc"));
    // k/v outputs: [max_kv] each, written by the q/k/v phases (the attention stand-in reads none)
    for (auto &P : ph)
        if (P.out_kind == kTrOutVec) {
            if (P.n_w > 1) P.y_plain[1] = t->kv;
            if (P.n_w > 2) P.y_plain[2] = t->kv + max_kv;
        }
    if ((e = cudaMemcpy(t->d_ph, ph.data(), ph.size() * sizeof(TrPhase), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemcpy(t->d_w, wt.data(), wt.size() * sizeof(TrWeight), cudaMemcpyHostToDevice)) != cudaSuccess ||
        (e = cudaMemset(t->R, 0, size_t(n_embd) * 8)) != cudaSuccess ||
        (e = cudaMemset(t->QB, 0, size_t(max_q) * 8)) != cudaSuccess ||
        (e = cudaMemset(t->AB, 0, size_t(max_ff) * 8)) != cudaSuccess ||
        (e = cudaMemset(t->pieces, 0, piece_bytes)) != cudaSuccess ||
        (e = cudaMemset(t->cnt, 0, cnt_bytes)) != cudaSuccess || (e = cudaMemset(t->ctl, 0, 256)) != cudaSuccess)
        return done(cuda_fail(e, "cpq_trunk_create: table upload"));
    *out = t;
    return done(CPQ_SUCCESS);
}

extern "C" cpq_status cpq_trunk_run(cpq_trunk *t, const float *h_in, float *h_out, void *stream) {
    using namespace cpq;
    if (!t) return fail(CPQ_ERR_INVALID_ARG, "cpq_trunk_run: trunk is null");
    if (!h_in || !h_out || h_in == h_out) return fail(CPQ_ERR_INVALID_ARG, "cpq_trunk_run: h_in/h_out null or equal");
    if (!aligned(h_in, 4) || !aligned(h_out, 4))
        return fail(CPQ_ERR_INVALID_ARG, "cpq_trunk_run: misaligned h_in/h_out");
    if (current_device() != t->device)
        return fail(CPQ_ERR_INVALID_ARG, "cpq_trunk_run: trunk belongs to device %d, current is %d", t->device,
                    current_device());
    TrArgs a;
    std::memset(&a, 0, sizeof a);
    a.ph = t->d_ph;
    a.w = t->d_w;
    a.n_ph = t->n_ph;
    a.n_embd = int(t->n_embd);
    a.act_bytes = t->act_bytes;
    a.n_ar = t->n_ar;
    a.R = t->R;
    a.QB = t->QB;
    a.AB = t->AB;
    a.pieces = t->pieces;
    a.cnt = t->cnt;
    a.ctl = t->ctl;
    a.h_in = h_in;
    a.h_out = h_out;
    a.world = 1;
    if (t->ar) {
        for (int r = 0; r < t->ar->world; r++) a.peer[r] = t->ar->peer[r];
        a.ar_base = t->ar->buf;
        a.ar_seq = t->ar->local;
        a.ar_nmax = t->ar->n_max;
        a.world = t->ar->world;
        a.rank = t->ar->rank;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(unsigned(t->grid));
    cfg.blockDim = dim3(kTrThreads);
    cfg.dynamicSmemBytes = size_t(t->smem);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: CTAs wait for one another's words
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, trunk_kernel, a);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "cpq_trunk_run: launch");
}

extern "C" int cpq_trunk_phases(const cpq_trunk *t) { return t ? t->n_ph : 0; }

extern "C" void cpq_trunk_destroy(cpq_trunk *t) { cpq::trunk_free(t); }
