// tp_ar.inl — cpq_tp_ar_*: the fused allreduce channel over NVLink peer memory.
//
// Each rank allocates one receive buffer of LL words, [kArSlots][world]
// [n_max] u64 (common.cuh), exports it with a CUDA IPC handle and maps the
// other ranks' buffers (cudaIpcOpenMemHandle, peer access enabled lazily).
// Its sequence number and the consumers' arrival counter live in a separate,
// rank-local allocation. The kernels' side is ArOut (gemv_row.cuh,
// row_block_out) and ArIn (act_prep.cuh act_prep_kernel, elementwise.cuh
// ar_add_kernel).

struct cpq_tp_ar {
    int device = -1;
    int world = 0;
    int rank = 0;
    int64_t n_max = 0;
    uint64_t *buf = nullptr;                       // this rank's receive buffer
    unsigned *local = nullptr;                     // [0] sequence number, [1] consumer arrivals
    uint64_t *peer[cpq::kArMaxRanks] = {};         // every rank's buffer as mapped here
    bool connected = false;
};

namespace cpq {

static void ar_free(cpq_tp_ar *ar) {
    if (!ar) return;
    int cur = -1;
    cudaGetDevice(&cur);
    if (ar->device >= 0) cudaSetDevice(ar->device);
    for (int r = 0; r < ar->world && r < kArMaxRanks; r++)
        if (ar->peer[r] && ar->peer[r] != ar->buf) cudaIpcCloseMemHandle(ar->peer[r]);
    cudaFree(ar->buf);
    cudaFree(ar->local);
    if (cur >= 0) cudaSetDevice(cur);
    delete ar;
}

static ArOut ar_out_of(const cpq_tp_ar *ar, int64_t n) {
    ArOut o = {};
    for (int r = 0; r < ar->world; r++) o.peer[r] = ar->peer[r];
    o.seq = ar->local;
    o.n_max = ar->n_max;
    o.n = n;
    o.world = ar->world;
    o.rank = ar->rank;
    o.on = 1;
    return o;
}

// n_ctas (the consumer launch's CTA count) is set by the launcher.
static ArIn ar_in_of(const cpq_tp_ar *ar, int64_t n) {
    ArIn i = {};
    i.base = ar->buf;
    i.seq = ar->local;
    i.arrive = ar->local + 1;
    i.n_max = ar->n_max;
    i.n = n;
    i.world = ar->world;
    i.on = 1;
    return i;
}

static bool ar_ready(const cpq_tp_ar *ar, int64_t need, const char **why) {
    if (!ar->connected) {
        *why = "the channel is not connected (cpq_tp_ar_connect)";
        return false;
    }
    if (need > ar->n_max) {
        *why = "M * N exceeds the channel's n_max";
        return false;
    }
    if (current_device() != ar->device) {
        *why = "the channel belongs to another device";
        return false;
    }
    return true;
}

}  // namespace cpq

extern "C" cpq_status cpq_tp_ar_create(int device, int world, int rank, int64_t n_max, cpq_tp_ar **out,
                                       void *handle64) {
    using namespace cpq;
    if (!out || !handle64) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_create: null output pointer");
    *out = nullptr;
    if (world < 1 || world > kArMaxRanks || rank < 0 || rank >= world)
        return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_create: world=%d rank=%d (world <= %d)", world, rank, kArMaxRanks);
    if (n_max < 1 || n_max > (int64_t(1) << 28)) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_create: n_max=%lld", (long long)n_max);
    int cur = -1;
    cudaGetDevice(&cur);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cpq_tp_ar_create: cudaSetDevice");
    cpq_tp_ar *ar = new cpq_tp_ar;
    ar->device = device;
    ar->world = world;
    ar->rank = rank;
    ar->n_max = int64_t(align_up(size_t(n_max), 64));
    const size_t bytes = size_t(kArSlots) * world * size_t(ar->n_max) * sizeof(uint64_t);
    auto done = [&](cpq_status s) {
        if (cur >= 0) cudaSetDevice(cur);
        if (s != CPQ_SUCCESS) ar_free(ar);
        return s;
    };
    if ((e = cudaMalloc(&ar->buf, bytes)) != cudaSuccess || (e = cudaMalloc(&ar->local, 256)) != cudaSuccess)
        return done(cuda_fail(e, "cpq_tp_ar_create: cudaMalloc"));
    if ((e = cudaMemset(ar->buf, 0, bytes)) != cudaSuccess || (e = cudaMemset(ar->local, 0, 256)) != cudaSuccess)
        return done(cuda_fail(e, "cpq_tp_ar_create: cudaMemset"));
    cudaIpcMemHandle_t h;
    if ((e = cudaIpcGetMemHandle(&h, ar->buf)) != cudaSuccess) return done(cuda_fail(e, "cpq_tp_ar_create: IPC handle"));
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    std::memcpy(handle64, &h, 64);
    ar->peer[rank] = ar->buf;
    *out = ar;
    return done(CPQ_SUCCESS);
}

extern "C" cpq_status cpq_tp_ar_connect(cpq_tp_ar *ar, const void *handles) {
    using namespace cpq;
    if (!ar || !handles) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_connect: null argument");
    if (ar->connected) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_connect: already connected");
    int cur = -1;
    cudaGetDevice(&cur);
    cudaError_t e = cudaSetDevice(ar->device);
    if (e != cudaSuccess) return cuda_fail(e, "cpq_tp_ar_connect: cudaSetDevice");
    cpq_status rc = CPQ_SUCCESS;
    for (int r = 0; r < ar->world && rc == CPQ_SUCCESS; r++) {
        if (r == ar->rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, static_cast<const uint8_t *>(handles) + 64 * r, 64);
        void *p = nullptr;
        e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            rc = cuda_fail(e, "cpq_tp_ar_connect: opening a peer's buffer");
        } else {
            ar->peer[r] = static_cast<uint64_t *>(p);
        }
    }
    if (cur >= 0) cudaSetDevice(cur);
    if (rc == CPQ_SUCCESS) ar->connected = true;
    return rc;
}

extern "C" void cpq_tp_ar_destroy(cpq_tp_ar *ar) { cpq::ar_free(ar); }

extern "C" cpq_status cpq_tp_ar_add(cpq_tp_ar *ar, const float *x, float *out, int64_t k, int64_t m, void *stream) {
    using namespace cpq;
    if (!ar || !x || !out) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_add: null argument");
    if (k <= 0 || m <= 0 || k % 8 != 0) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_add: k=%lld m=%lld", (long long)k, (long long)m);
    if (!aligned(x, 16) || !aligned(out, 16)) return fail(CPQ_ERR_UNSUPPORTED, "cpq_tp_ar_add: 16-byte alignment");
    const char *why = "";
    if (!ar_ready(ar, m * k, &why)) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_add: %s", why);
    ArIn in = ar_in_of(ar, k);
    const dim3 grid(unsigned((k + 2047) / 2048), unsigned(m));
    in.n_ctas = grid.x * grid.y;
    const cudaError_t e = launch(ar_add_kernel, grid, dim3(256), 0, static_cast<cudaStream_t>(stream), in, x, out, k);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "cpq_tp_ar_add: launch");
}

extern "C" cpq_status cpq_tp_ar_argmax(cpq_tp_ar *ar, const float *logits, int64_t n, int64_t m, int64_t ld,
                                       int64_t row0, int32_t *out, void *stream) {
    using namespace cpq;
    if (!ar || !logits || !out) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_argmax: null argument");
    if (n <= 0 || m <= 0 || ld < n || row0 < 0 || row0 + n > 2147483647 || m > 65535)
        return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_argmax: n=%lld m=%lld ld=%lld row0=%lld", (long long)n,
                    (long long)m, (long long)ld, (long long)row0);
    const char *why = "";
    if (!ar_ready(ar, 2 * m, &why)) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_argmax: %s", why);
    ArIn in = ar_in_of(ar, 2);
    in.n_ctas = unsigned(m);
    const ArOut o = ar_out_of(ar, 2);
    const cudaError_t e = launch(ar_argmax_kernel, dim3(unsigned(m)), dim3(1024), 0, static_cast<cudaStream_t>(stream),
                                 in, o, logits, n, ld, row0, out);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "cpq_tp_ar_argmax: launch");
}

extern "C" cpq_status cpq_tp_ar_zero(cpq_tp_ar *ar, int64_t n, int64_t m, void *stream) {
    using namespace cpq;
    if (!ar) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_zero: null channel");
    if (n <= 0 || m <= 0) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_zero: n=%lld m=%lld", (long long)n, (long long)m);
    const char *why = "";
    if (!ar_ready(ar, m * n, &why)) return fail(CPQ_ERR_INVALID_ARG, "cpq_tp_ar_zero: %s", why);
    const ArOut o = ar_out_of(ar, n);
    const int64_t total = m * n;
    const cudaError_t e = launch(ar_zero_kernel, dim3(unsigned(std::min<int64_t>((total + 255) / 256, 1024))),
                                 dim3(256), 0, static_cast<cudaStream_t>(stream), o, total);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "cpq_tp_ar_zero: launch");
}
