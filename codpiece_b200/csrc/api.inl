// api.inl — the extern "C" entry points of libcpq (host code).
//
// Validation happens here, on the host, before anything is launched: every
// shape, stride, alignment and type outside the fast path returns a status
// (CPQ_ERR_UNSUPPORTED / CPQ_ERR_INVALID_ARG) instead of aborting, where
// ggml would GGML_ASSERT (docs/BENCHMARKS.md:199-203 notes such aborts).
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <mutex>
#include <string>
#include <unordered_map>

namespace cpq {

static thread_local std::string g_last_error;

static cpq_status fail(cpq_status s, const char *fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return s;
}

static cpq_status cuda_fail(cudaError_t e, const char *what) {
    return fail(CPQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

constexpr int kMaxDevices = 64;

// Workspace carve-up: [row-block counters][per-warp partials][per-warp piece
// words][argmax scratch][activations]. The counters and piece words must be
// zero before the first call; the GEMV kernels leave them zero after every
// successful call (cpq_device_status with clear also re-zeroes them).
constexpr size_t kWsCounters = 65536;                       // row blocks per call (>= 1M rows)
constexpr size_t kWsCountersBytes = kWsCounters * sizeof(int);
constexpr size_t kWsMaxWarps = 148 * 2 * 16;                // persistent warps, generous
constexpr size_t kWsPartialBytes = kWsMaxWarps * 2 * 16 * 16 * sizeof(float);
constexpr int kArgmaxChunks = 128;                            // CTAs per argmax row
constexpr int kArgmaxMaxRows = 64;
constexpr size_t kWsPieceBytes = kWsMaxWarps * 2 * kPieceWords * sizeof(uint64_t);  // row GEMV (gemv_row.cuh)
constexpr size_t kWsAuxBytes = align_up(size_t(kArgmaxMaxRows) * (kArgmaxChunks * 8 + 4), 256);
constexpr size_t kWsPieceOffset = kWsCountersBytes + kWsPartialBytes;
constexpr size_t kWsAuxOffset = kWsPieceOffset + kWsPieceBytes;
constexpr size_t kWsActOffset = kWsAuxOffset + kWsAuxBytes;

struct DevState {
    void *ws = nullptr;
    size_t ws_bytes = 0;
};
static std::mutex g_mu;
static DevState g_dev[kMaxDevices];

static int sm_count(int dev) {
    static std::atomic<int> cache[kMaxDevices];
    int v = cache[dev].load(std::memory_order_relaxed);
    if (v == 0) {
        cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
        if (v <= 0) v = 1;
        cache[dev].store(v, std::memory_order_relaxed);
    }
    return v;
}

static bool pdl_enabled() {
    static const bool on = [] {
        const char *e = std::getenv("CPQ_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

// Every kernel prefers the largest shared-memory carveout: the small kernels
// of a decode chain then run under the same SM configuration as the GEMVs
// they overlap with (a different split would keep them off an SM until its
// GEMV CTA has left). Set once per kernel and device.
#ifndef CPQ_CARVEOUT
#define CPQ_CARVEOUT 1
#endif
static void prefer_max_shared(const void *fn) {
#if CPQ_CARVEOUT
    static std::mutex mu;
    static std::unordered_map<const void *, uint64_t> done;  // kernel -> bit set of devices
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return;
    std::lock_guard<std::mutex> lk(mu);
    uint64_t &bits = done[fn];
    if (bits & (uint64_t(1) << dev)) return;
    bits |= uint64_t(1) << dev;
    cudaFuncSetAttribute(fn, cudaFuncAttributePreferredSharedMemoryCarveout, int(cudaSharedmemCarveoutMaxShared));
#else
    (void)fn;
#endif
}

// Every kernel is launched with programmatic stream serialization allowed,
// so its prologue can overlap the tail of the previous kernel on the stream;
// each kernel calls griddepcontrol.wait before touching its inputs.
template <typename... KArgs, typename... Args>
static cudaError_t launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                          Args &&...args) {
    prefer_max_shared(reinterpret_cast<const void *>(kern));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

static int current_device() {
    int d = 0;
    if (cudaGetDevice(&d) != cudaSuccess) return -1;
    return d;
}

// ---- type helpers -----------------------------------------------------------

static int64_t type_blck(int32_t t) {
    switch (t) {
    case CPQ_TYPE_Q8_0: return kQK8_0;
    case CPQ_TYPE_Q4_K:
    case CPQ_TYPE_Q6_K:
    case CPQ_TYPE_Q8_K: return kQK_K;
    case CPQ_TYPE_F32:
    case CPQ_TYPE_F16: return 1;
    default: return 0;
    }
}

static int64_t type_bytes(int32_t t) {
    switch (t) {
    case CPQ_TYPE_Q8_0: return kQ8_0_Bytes;
    case CPQ_TYPE_Q4_K: return kQ4K_Bytes;
    case CPQ_TYPE_Q6_K: return kQ6K_Bytes;
    case CPQ_TYPE_Q8_K: return kQ8K_Bytes;
    case CPQ_TYPE_F32: return 4;
    case CPQ_TYPE_F16: return 2;
    default: return 0;
    }
}

// ggml-cpu's vec_dot_type for each weight type on this path.
static int32_t vec_dot_type(int32_t wt) {
    switch (wt) {
    case CPQ_TYPE_Q4_K:
    case CPQ_TYPE_Q6_K: return CPQ_TYPE_Q8_K;
    case CPQ_TYPE_Q8_0: return CPQ_TYPE_Q8_0;
    default: return -1;
    }
}

static const char *type_name(int32_t t) {
    switch (t) {
    case CPQ_TYPE_F32: return "F32";
    case CPQ_TYPE_F16: return "F16";
    case CPQ_TYPE_Q8_0: return "Q8_0";
    case CPQ_TYPE_Q4_K: return "Q4_K";
    case CPQ_TYPE_Q6_K: return "Q6_K";
    case CPQ_TYPE_Q8_K: return "Q8_K";
    default: return "unknown";
    }
}

static bool aligned(const void *p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// ---- validation ------------------------------------------------------------

struct MMShape {
    int32_t wtype;
    int64_t k, n, m;
};

static cpq_status check_weight(const cpq_tensor *w, MMShape *s) {
    if (!w) return fail(CPQ_ERR_INVALID_ARG, "weight descriptor is null");
    if (vec_dot_type(w->type) < 0)
        return fail(CPQ_ERR_UNSUPPORTED, "weight type %s (%d) is not Q4_K, Q6_K or Q8_0", type_name(w->type), w->type);
    if (w->ne[2] != 1 || w->ne[3] != 1)
        return fail(CPQ_ERR_UNSUPPORTED, "weight ne[2]=%lld ne[3]=%lld: only 2-D weights", (long long)w->ne[2],
                    (long long)w->ne[3]);
    const int64_t blk = type_blck(w->type), bb = type_bytes(w->type);
    if (w->ne[0] <= 0 || w->ne[1] < 0) return fail(CPQ_ERR_INVALID_ARG, "weight ne[0]=%lld ne[1]=%lld", (long long)w->ne[0], (long long)w->ne[1]);
    if (w->ne[0] % blk != 0)
        return fail(CPQ_ERR_INVALID_ARG, "weight ne[0]=%lld is not a multiple of the %s block (%lld)",
                    (long long)w->ne[0], type_name(w->type), (long long)blk);
    const size_t row = size_t(w->ne[0] / blk) * size_t(bb);
    if (w->nb[0] != size_t(bb)) return fail(CPQ_ERR_UNSUPPORTED, "weight nb[0]=%zu != block size %lld", w->nb[0], (long long)bb);
    if (w->nb[1] < row) return fail(CPQ_ERR_INVALID_ARG, "weight nb[1]=%zu < row size %zu", w->nb[1], row);
    if (w->type == CPQ_TYPE_Q4_K && w->nb[1] % 16 != 0)
        return fail(CPQ_ERR_UNSUPPORTED, "Q4_K row stride %zu is not a multiple of 16 bytes", w->nb[1]);
    if (w->nb[1] % 2 != 0) return fail(CPQ_ERR_UNSUPPORTED, "weight row stride %zu is odd", w->nb[1]);
    if (w->ne[1] > 0 && !w->data) return fail(CPQ_ERR_INVALID_ARG, "weight data is null");
    if (!aligned(w->data, 16)) return fail(CPQ_ERR_UNSUPPORTED, "weight data is not 16-byte aligned");
    s->wtype = w->type;
    s->k = w->ne[0];
    s->n = w->ne[1];
    return CPQ_SUCCESS;
}

static cpq_status check_x(const cpq_tensor *x, int64_t k, int64_t *m) {
    if (!x) return fail(CPQ_ERR_INVALID_ARG, "activation descriptor is null");
    if (x->type != CPQ_TYPE_F32) return fail(CPQ_ERR_UNSUPPORTED, "activation type %s: only F32", type_name(x->type));
    if (x->ne[2] != 1 || x->ne[3] != 1) return fail(CPQ_ERR_UNSUPPORTED, "activation must be 2-D");
    if (x->ne[0] != k)
        return fail(CPQ_ERR_INVALID_ARG, "activation ne[0]=%lld != weight ne[0]=%lld", (long long)x->ne[0], (long long)k);
    if (x->ne[1] < 0) return fail(CPQ_ERR_INVALID_ARG, "activation ne[1] < 0");
    if (x->nb[0] != 4) return fail(CPQ_ERR_UNSUPPORTED, "activation nb[0]=%zu: rows must be contiguous", x->nb[0]);
    if (x->nb[1] < size_t(k) * 4 || x->nb[1] % 16 != 0)
        return fail(CPQ_ERR_UNSUPPORTED, "activation nb[1]=%zu must be >= 4*K and a multiple of 16", x->nb[1]);
    if (x->ne[1] > 0 && (!x->data || !aligned(x->data, 16)))
        return fail(CPQ_ERR_UNSUPPORTED, "activation data null or not 16-byte aligned");
    *m = x->ne[1];
    return CPQ_SUCCESS;
}

static cpq_status check_y(const cpq_tensor *y, int64_t n, int64_t m) {
    if (!y) return fail(CPQ_ERR_INVALID_ARG, "output descriptor is null");
    if (y->type != CPQ_TYPE_F32) return fail(CPQ_ERR_UNSUPPORTED, "output type %s: only F32", type_name(y->type));
    if (y->ne[2] != 1 || y->ne[3] != 1) return fail(CPQ_ERR_UNSUPPORTED, "output must be 2-D");
    if (y->ne[0] != n || y->ne[1] != m)
        return fail(CPQ_ERR_INVALID_ARG, "output ne=[%lld,%lld], expected [%lld,%lld]", (long long)y->ne[0],
                    (long long)y->ne[1], (long long)n, (long long)m);
    if (y->nb[0] != 4 || y->nb[1] < size_t(n) * 4 || y->nb[1] % 4 != 0)
        return fail(CPQ_ERR_UNSUPPORTED, "output strides nb[0]=%zu nb[1]=%zu", y->nb[0], y->nb[1]);
    if (n > 0 && m > 0 && (!y->data || !aligned(y->data, 4))) return fail(CPQ_ERR_INVALID_ARG, "output data null or misaligned");
    return CPQ_SUCCESS;
}

// ---- launches -----------------------------------------------------------------

static cudaError_t launch_quantize(int32_t vt, const float *x, int64_t k, int64_t m, int64_t x_stride, void *ws,
                                   const ActLayout &L, uint8_t *aos, cudaStream_t st) {
    int8_t *qs = ws ? reinterpret_cast<int8_t *>(static_cast<uint8_t *>(ws) + L.qs_off) : nullptr;
    float *d = ws ? reinterpret_cast<float *>(static_cast<uint8_t *>(ws) + L.d_off) : nullptr;
    int16_t *bs = ws ? reinterpret_cast<int16_t *>(static_cast<uint8_t *>(ws) + L.bs_off) : nullptr;
    if (vt == CPQ_TYPE_Q8_K) {
        const int64_t blocks = m * (k / kQK_K);  // one warp each, 8 per CTA
        const int64_t grid = std::min<int64_t>((blocks + 7) / 8, 65535);
        return launch(quantize_q8K_kernel, dim3(unsigned(grid)), dim3(256), 0, st, x, k, m, x_stride, qs, d, bs, aos);
    }
    const int64_t blocks = m * (k / kQK8_0);  // 4 lanes each, 64 per CTA
    const int64_t grid = std::min<int64_t>((blocks + 63) / 64, 65535);
    return launch(quantize_q8_0_kernel, dim3(unsigned(grid)), dim3(256), 0, st, x, k, m, x_stride, qs, d, aos);
}

template <class F, int MT>
static cudaError_t launch_gemv_t(const GemvArgs &a, cudaStream_t st) {
    constexpr int smem = GemvSmem<F>::kBytes;
    auto kern = gemv_kernel<F, MT>;
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    static std::atomic<int> occ[kMaxDevices];
    int bpm = occ[dev].load(std::memory_order_relaxed);
    if (bpm == 0) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bpm, kern, kGemvWarps * 32, smem);
        if (e != cudaSuccess) return e;
        if (bpm < 1) bpm = 1;
        occ[dev].store(bpm, std::memory_order_relaxed);
    }
    const int64_t ntot = a.row_start[a.n_w];
    const int64_t want = (ntot + kGemvWarps - 1) / kGemvWarps;
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(want, int64_t(sm_count(dev)) * bpm));
    return launch(kern, dim3(unsigned(grid)), dim3(kGemvWarps * 32), smem, st, a);
}

template <class F>
static cudaError_t launch_gemv(const GemvArgs &a, int mt, cudaStream_t st) {
    switch (mt) {
    case 1: return launch_gemv_t<F, 1>(a, st);
    case 2: return launch_gemv_t<F, 2>(a, st);
    case 3: return launch_gemv_t<F, 3>(a, st);
    case 4: return launch_gemv_t<F, 4>(a, st);
    case 5: return launch_gemv_t<F, 5>(a, st);
    case 6: return launch_gemv_t<F, 6>(a, st);
    case 7: return launch_gemv_t<F, 7>(a, st);
    case 8: return launch_gemv_t<F, 8>(a, st);
    default: return cudaErrorInvalidValue;
    }
}

constexpr int kGemvMaxTokens = 8;  // tokens per GEMV launch (dp4a kernels)
constexpr int kSmemMax = 227 * 1024;  // dynamic shared memory a CTA may ask for on sm_100

// Q6_K over whole row pairs (gemv_q6k.cuh): one weight, dense 16-byte aligned
// rows, K a multiple of 1024 (a row pair is then a 16-byte multiple), an
// even row count, and the activations of the token group in shared memory.
static int q6r_mt(int mt) { return mt <= 2 ? mt : mt <= 4 ? 4 : 8; }  // the kernel instance for mt tokens

static bool q6k_rows_ok(const GemvArgs &g, int mt) {
    const int64_t nbk = g.k / kQK_K;
    const int64_t n = g.row_start[1] - g.row_start[0];
    return g.n_w == 1 && g.k % 1024 == 0 && n % 2 == 0 && n > 0 && g.rs == size_t(nbk) * kQ6K_Bytes &&
           aligned(g.w[0], 16) && aligned(g.act.qs, 16) && aligned(g.act.d, 16) && aligned(g.act.bsums, 16) &&
           mt <= kQ6rMaxTokens && q6r_smem_bytes(int(nbk), q6r_mt(mt)) <= kSmemMax;
}

template <int MT>
static cudaError_t launch_q6k_rows_t(const Q6RowArgs &a, cudaStream_t st) {
    auto kern = gemv_q6k_rows_kernel<MT>;
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    static std::atomic<int> set[kMaxDevices];
    if (!set[dev].load(std::memory_order_relaxed)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        set[dev].store(1, std::memory_order_relaxed);
    }
    const int64_t pairs = a.n / 2;
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(sm_count(dev), (pairs + kQ6rWarps - 1) / kQ6rWarps));
    return launch(kern, dim3(unsigned(grid)), dim3(kQ6rWarps * 32), size_t(q6r_smem_bytes(a.nbk, MT)), st, a);
}

// Q8_0 over whole row pairs (gemv_q6k.cuh): one weight, dense 16-byte aligned
// rows, K a multiple of 256, an even row count.
static bool q8_rows_ok(const GemvArgs &g, int mt) {
    const int64_t nb = g.k / kQK8_0;
    const int64_t n = g.row_start[1] - g.row_start[0];
    const int mr = mt <= 2 ? mt : mt <= 4 ? 4 : 8;
    return g.n_w == 1 && g.k % 256 == 0 && n % 2 == 0 && n > 0 && g.rs == size_t(nb) * kQ8_0_Bytes &&
           aligned(g.w[0], 16) && aligned(g.act.qs, 16) && aligned(g.act.d, 16) && mt <= 8 &&
           q8r_smem_bytes(int(nb), mr, 4, 2) <= kSmemMax;  // the narrowest instance of launch_q8_rows_t
}

template <int MT, bool QX, int W, int S>
static cudaError_t launch_q8_rows_ws(const Q8RowArgs &a, cudaStream_t st) {
    auto kern = gemv_q8_0_rows_kernel<MT, QX, W, S>;
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    static std::atomic<int> set[kMaxDevices];
    if (!set[dev].load(std::memory_order_relaxed)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        set[dev].store(1, std::memory_order_relaxed);
    }
    const int64_t pairs = a.n / 2;
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(sm_count(dev), (pairs + W - 1) / W));
    return launch(kern, dim3(unsigned(grid)), dim3(W * 32), size_t(q8r_smem_bytes(a.nb, MT, W, S)), st, a);
}

// The widest ring that fits in shared memory: 8 warps x 2 stages, else 6 or
// 4 warps (K = 6144 at M = 3..8 needs 6: [6144 x 6144] at M = 4 42.6 -> 22.8 us
// against the generic kernel it fell back to). A deeper 6 x 3 ring for one
// token (every pair of [5120 x 5120] in flight at once) measured slower:
// 10.7 vs 10.0 us.
template <int MT, bool QX = false>
static cudaError_t launch_q8_rows_t(const Q8RowArgs &a, cudaStream_t st) {
    if (q8r_smem_bytes(a.nb, MT, kQ8rWarps, 2) <= kSmemMax) return launch_q8_rows_ws<MT, QX, kQ8rWarps, 2>(a, st);
    if (q8r_smem_bytes(a.nb, MT, 6, 2) <= kSmemMax) return launch_q8_rows_ws<MT, QX, 6, 2>(a, st);
    return launch_q8_rows_ws<MT, QX, 4, 2>(a, st);
}

// x != NULL: the kernel quantizes the fp32 activations itself (no quantizer launch).
static cudaError_t launch_q8_rows(const GemvArgs &g, int mt, cudaStream_t st, const float *x = nullptr,
                                  int64_t x_stride = 0) {
    Q8RowArgs a;
    a.w = g.w[0];
    a.y = g.y[0];
    a.y_stride = g.y_stride[0];
    a.n = g.row_start[1] - g.row_start[0];
    a.nb = int(g.k / kQK8_0);
    a.m = mt;
    a.qs = g.act.qs;
    a.d = g.act.d;
    a.x = x;
    a.x_stride = x_stride;
    if (x && mt == 1) return launch_q8_rows_t<1, true>(a, st);
    switch (mt) {
    case 1: return launch_q8_rows_t<1>(a, st);
    case 2: return launch_q8_rows_t<2>(a, st);
    case 3:
    case 4: return launch_q8_rows_t<4>(a, st);
    default: return launch_q8_rows_t<8>(a, st);
    }
}

static cudaError_t launch_q6k_rows(const GemvArgs &g, int mt, cudaStream_t st) {
    Q6RowArgs a;
    a.w = g.w[0];
    a.y = g.y[0];
    a.y_stride = g.y_stride[0];
    a.n = g.row_start[1] - g.row_start[0];
    a.nbk = int(g.k / kQK_K);
    a.m = mt;
    a.qs = g.act.qs;
    a.d = g.act.d;
    a.bsums = g.act.bsums;
    switch (mt) {
    case 1: return launch_q6k_rows_t<1>(a, st);
    case 2: return launch_q6k_rows_t<2>(a, st);
    case 3:
    case 4: return launch_q6k_rows_t<4>(a, st);
    default: return launch_q6k_rows_t<8>(a, st);
    }
}

// Q6_K on int8 MMA tiles (gemv_q6k_mma.cuh), up to 16 tokens per weight
// pass: one weight, dense rows, N a multiple of 8, K <= 30 superblocks. Used
// from q6m_min_tokens() tokens on (default 3; CPQ_Q6K_MMA_MIN_M overrides).
// Measured on the head [151936 x 5120]: 251 us at M = 1..8 against 165 /
// 222 us for the row-pair kernel at M = 1 / 2 and 285 / 505 us at M = 4 / 8.
static int q6m_min_tokens() {
    static const int v = [] {
        const char *e = std::getenv("CPQ_Q6K_MMA_MIN_M");
        const int x = e ? std::atoi(e) : 3;
        return x < 1 ? 1 : x;
    }();
    return v;
}

static bool q6m_ok(const GemvArgs &g, int64_t m) {
    const int64_t nbk = g.k / kQK_K;
    const int64_t n = g.row_start[1] - g.row_start[0];
    return g.n_w == 1 && m >= q6m_min_tokens() && n > 0 && n % 8 == 0 && nbk >= 1 && nbk * kQK_K <= kQ6mMaxK &&
           g.rs == size_t(nbk) * kQ6K_Bytes && aligned(g.w[0], 16) && q6m_smem_bytes(int(nbk), 16) <= kSmemMax;
}

template <int MT>
static cudaError_t launch_q6k_mma_t(const Q6MmaArgs &a, cudaStream_t st) {
    auto kern = gemv_q6k_mma_kernel<MT>;
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    static std::atomic<int> set[kMaxDevices];
    if (!set[dev].load(std::memory_order_relaxed)) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        set[dev].store(1, std::memory_order_relaxed);
    }
    const int64_t grid = std::max<int64_t>(1, std::min<int64_t>(sm_count(dev), a.n / 8));
    return launch(kern, dim3(unsigned(grid)), dim3(q6m_threads(MT)), size_t(q6m_smem_bytes(a.nbk, MT)), st, a);
}

static cudaError_t launch_q6k_mma(const GemvArgs &g, int mt, cudaStream_t st) {
    Q6MmaArgs a;
    a.w = g.w[0];
    a.y = g.y[0];
    a.y_stride = g.y_stride[0];
    a.n = g.row_start[1] - g.row_start[0];
    a.nbk = int(g.k / kQK_K);
    a.m = mt;
    a.qs = g.act.qs;
    a.d = g.act.d;
    a.bsums = g.act.bsums;
    return mt <= 8 ? launch_q6k_mma_t<8>(a, st) : launch_q6k_mma_t<16>(a, st);
}

// Q4_K: fragment-order quantization, then the tensor-core GEMV per group of
// up to 16 tokens.
// SM: the activation image goes to shared memory (a.act_smem bytes after the ring).
template <int NG, bool SM>
static cudaError_t launch_q4k_mma_t(MmaArgs &a, cudaStream_t st) {
    auto kern = gemv_q4k_mma_kernel<NG, SM>;
    constexpr int kMmaWarps = MmaCfg<NG>::kWarps;  // this instance's warps per CTA
    const int smem = kMmaSmem + (SM ? a.act_smem : 0);
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    static std::atomic<int> occ[kMaxDevices];
    int bpm = occ[dev].load(std::memory_order_relaxed);
    if (bpm == 0) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             SM ? int(227 * 1024) : kMmaSmem);
        if (e != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&bpm, kern, kMmaWarps * 32, SM ? 227 * 1024 : kMmaSmem);
        if (e != cudaSuccess) return e;
        if (bpm < 1) bpm = 1;
        occ[dev].store(bpm, std::memory_order_relaxed);
    }
    const int64_t T = a.mb_start[a.n_w] * a.nbk;
    const int64_t cap = std::min<int64_t>(int64_t(sm_count(dev)) * bpm * kMmaWarps, int64_t(kWsMaxWarps));
    a.n_warps = std::max<int64_t>(1, std::min<int64_t>(cap, T));
    const int64_t grid = (a.n_warps + kMmaWarps - 1) / kMmaWarps;
    return launch(kern, dim3(unsigned(grid)), dim3(kMmaWarps * 32), size_t(smem), st, a);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// link-time libcuda dependency). Maps depend only on (pointer, rows, row
// stride, K), so they are cached.
typedef CUresult (*EncodeTiledFn)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                  const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_tiled() {
    static EncodeTiledFn fn = [] {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return EncodeTiledFn(nullptr);
        return reinterpret_cast<EncodeTiledFn>(p);
    }();
    return fn;
}

struct TmapKey {
    const void *p;
    int64_t n, k;
    size_t rs;
    int box_rows, box_sb;
    bool operator==(const TmapKey &o) const {
        return p == o.p && n == o.n && k == o.k && rs == o.rs && box_rows == o.box_rows && box_sb == o.box_sb;
    }
};
struct TmapKeyHash {
    size_t operator()(const TmapKey &t) const {
        return std::hash<const void *>()(t.p) ^ (size_t(t.n) * 1000003u) ^ (size_t(t.k) << 20) ^ (t.rs << 7) ^
               (size_t(t.box_rows) << 40) ^ (size_t(t.box_sb) << 48);
    }
};

// Q4_K weight [n rows][rs bytes] as a 2-D u64 tensor; box = box_rows rows x box_sb superblocks.
static cpq_status q4k_tensor_map(const uint8_t *w, int64_t n, int64_t k, size_t rs, CUtensorMap *out,
                                 int box_rows = kMmaRows, int box_sb = kMmaSB) {
    static std::mutex mu;
    static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
    const TmapKey key{w, n, k, rs, box_rows, box_sb};
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *out = it->second;
            return CPQ_SUCCESS;
        }
    }
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return fail(CPQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {cuuint64_t(k / kQK_K) * (kQ4K_Bytes / 8), cuuint64_t(n)};
    const cuuint64_t strides[1] = {cuuint64_t(rs)};
    const cuuint32_t box[2] = {cuuint32_t(box_sb * (kQ4K_Bytes / 8)), cuuint32_t(box_rows)};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap m;
    const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t *>(w), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CPQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
    std::lock_guard<std::mutex> lk(mu);
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return CPQ_SUCCESS;
}

// Dense fp16 activations [m][k] as a 2-D tensor for the tensor-core GEMM:
// box = 64 elements (128 bytes) x tile_n rows, 128-byte swizzle.
static cpq_status f16_act_tensor_map(const __half *x, int64_t k, int64_t m, int tile_n, CUtensorMap *out) {
    static std::mutex mu;
    static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
    const TmapKey key{x, m, k, size_t(k) * 2, tile_n, 0};
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *out = it->second;
            return CPQ_SUCCESS;
        }
    }
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return fail(CPQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(m)};
    const cuuint64_t strides[1] = {cuuint64_t(k) * 2};
    const cuuint32_t box[2] = {cuuint32_t(kTcAtomK), cuuint32_t(tile_n)};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap t;
    const CUresult r = enc(&t, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half *>(x), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CPQ_ERR_CUDA, "cuTensorMapEncodeTiled (fp16 activations) failed (%d)", int(r));
    std::lock_guard<std::mutex> lk(mu);
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, t);
    *out = t;
    return CPQ_SUCCESS;
}

// Activation region bytes (the largest of the three layouts) and the fp32
// prologue region that follows it.
static size_t act_region_bytes(int32_t vt, int64_t k, int64_t m);
static size_t ws_need(int32_t vt, int64_t k, int64_t m) {
    return kWsActOffset + act_region_bytes(vt, k, m) + align_up(size_t(m) * size_t(k) * 4, 256);
}

// Bytes of the fragment-order activation region for one group of mp tokens.
static size_t frag_bytes(int64_t k, int mp) {
    const size_t nbk = size_t(k / kQK_K);
    return align_up(nbk * mp * 256, 256) + align_up(nbk * mp * 16, 256) + align_up(nbk * mp * 4, 256);
}


static int row_smem_bytes(int64_t k, int mt) {
    return kRowBarBytes + row_act_bytes(k, mt) + kRowRingBytes + row_red_bytes(mt);
}

// CTAs of the row GEMV: one per SM at most (the kernel's tail-cut hand-off
// needs every CTA resident), and at most T / nbk so that no CTA's range lies
// inside one row block.
static int64_t row_grid(const RowArgs &a, int64_t cap) {
    const int64_t row_blocks = a.mb_start[a.n_w];
    return std::max<int64_t>(1, std::min<int64_t>(cap, row_blocks));
}

template <int MT>
static cudaError_t launch_q4k_row_t(RowArgs &a, int smem, cudaStream_t st) {
    auto kern = gemv_q4k_row_kernel<MT>;
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    static std::atomic<int> set[kMaxDevices];
    if (!set[dev].load(std::memory_order_relaxed)) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        set[dev].store(1, std::memory_order_relaxed);
    }
    const int64_t grid = row_grid(a, std::min<int64_t>(sm_count(dev), int64_t(kWsMaxWarps / kRowWarps)));
    return launch(kern, dim3(unsigned(grid)), dim3(kRowWarps * 32), size_t(smem), st, a);
}

// M <= 3: the activation image is built by act_prep_kernel (with the fused
// prologue), then the row GEMV pulls it in with one bulk copy.
static cpq_status run_q4k_row(const GemvArgs &g, const float *x, int64_t x_stride, int m, const cpq_prologue &pro,
                              uint8_t *ws, cudaStream_t st, const ArIn *ar_in = nullptr,
                              const ArOut *ar_out = nullptr) {
    static thread_local RowArgs a;
    std::memset(&a, 0, sizeof a);
    const int64_t k = g.k;
    a.n_w = g.n_w;
    for (int i = 0; i < g.n_w; i++) {
        a.n[i] = g.row_start[i + 1] - g.row_start[i];
        a.y[i] = g.y[i];
        a.y_stride[i] = g.y_stride[i];
        a.mb_start[i + 1] = a.mb_start[i] + (a.n[i] + kRowRows - 1) / kRowRows;
        if (a.n[i] > 0) {
            cpq_status rc = q4k_tensor_map(g.w[i], a.n[i], k, g.rs, &a.tmap[i], kRowRows, 1);
            if (rc) return rc;
        }
    }
    uint8_t *act = ws + kWsActOffset;
    ActPrepArgs pa = {};
    pa.mode = pro.mode;
    pa.x = x;
    pa.r = pro.r;
    pa.g = pro.g;
    pa.h_out = pro.h_out;
    pa.x_stride = x_stride;
    pa.k = k;
    pa.m = m;
    pa.eps = pro.eps;
    pa.out = act;
    const int nbk = int(k / kQK_K);
    if (ar_in) {
        pa.ar = *ar_in;
        pa.ar.n_ctas = unsigned((nbk + 7) / 8) * unsigned(m);  // act_prep_kernel's grid below
    }
    cudaError_t e = ar_in ? launch(act_prep_kernel<true>, dim3(unsigned((nbk + 7) / 8), unsigned(m)), dim3(256), 0, st, pa)
                          : launch(act_prep_kernel<false>, dim3(unsigned((nbk + 7) / 8), unsigned(m)), dim3(256), 0, st, pa);
    if (e != cudaSuccess) return cuda_fail(e, "act_prep launch");
    a.nbk = nbk;
    a.m = m;
    a.act = act;
    a.pieces = reinterpret_cast<uint64_t *>(ws + kWsPieceOffset);
    if (ar_out) a.ar = *ar_out;
    const int smem = row_smem_bytes(k, m);
    switch (m) {
    case 1: e = launch_q4k_row_t<1>(a, smem, st); break;
    case 2: e = launch_q4k_row_t<2>(a, smem, st); break;
    default: e = launch_q4k_row_t<3>(a, smem, st); break;
    }
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "q4_K row gemv launch");
}

static size_t act_region_bytes(int32_t vt, int64_t k, int64_t m) {
    size_t b = act_layout(vt, k, std::max<int64_t>(m, 1)).bytes;
    if (vt == CPQ_TYPE_Q8_K) {
        b = std::max(b, frag_bytes(k, 16));
        b = std::max(b, size_t(row_act_bytes(k, kRowMaxTokens)));
        b = std::max(b, size_t(m) * size_t(k) * 2);  // fp16 activations of the tensor-core path
    }
    if (vt == CPQ_TYPE_Q8_0) b = std::max(b, size_t(m) * size_t(k) * 2);
    return align_up(b, 256);
}

// up != NULL: the input is silu(x) * up, formed inside the quantizer (x = gate rows).
// ar_out: weight 0's outputs go to every rank through the fused all-reduce channel.
// up: the SwiGLU prologue (silu(x) * up) inside the fragment quantizer; rms: the
// RMS prologue, by act_prep_kernel<false, true> (the row's RMS, then the
// fragment image, one launch; x, rms->r and rms->h_out 16-byte aligned rows).
static cpq_status run_q4k_mma(const GemvArgs &g, const float *x, int64_t x_stride, int64_t m, uint8_t *ws,
                              cudaStream_t st, const float *up = nullptr, const ArOut *ar_out = nullptr,
                              const cpq_prologue *rms = nullptr) {
    const int64_t k = g.k, nbk = k / kQK_K;
    static thread_local MmaArgs a;  // large (tensor maps); filled per call
    std::memset(&a, 0, sizeof a);
    if (ar_out) a.ar = *ar_out;
    a.n_w = g.n_w;
    a.mb_start[0] = 0;
    for (int i = 0; i < g.n_w; i++) {
        a.n[i] = g.row_start[i + 1] - g.row_start[i];
        a.y_stride[i] = g.y_stride[i];
        a.mb_start[i + 1] = a.mb_start[i] + (a.n[i] + kMmaRows - 1) / kMmaRows;
        if (a.n[i] > 0) {
            cpq_status rc = q4k_tensor_map(g.w[i], a.n[i], k, g.rs, &a.tmap[i]);
            if (rc) return rc;
        }
    }
    if (a.mb_start[g.n_w] > int64_t(kWsCounters))
        return fail(CPQ_ERR_UNSUPPORTED, "too many row blocks (%lld) for the workspace counters",
                    (long long)a.mb_start[g.n_w]);
    a.nbk = int(nbk);
    a.partials = reinterpret_cast<float *>(ws + kWsCountersBytes);
    a.counters = reinterpret_cast<int *>(ws);

    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return fail(CPQ_ERR_CUDA, "no current device");
    uint8_t *act = ws + kWsActOffset;
    for (int64_t t0 = 0; t0 < m; t0 += kMmaMaxTokens) {
        const int mt = int(std::min<int64_t>(kMmaMaxTokens, m - t0));
        const int mp = mt <= 8 ? 8 : 16;
        int8_t *qs = reinterpret_cast<int8_t *>(act);
        uint8_t *bs = act + align_up(size_t(nbk) * mp * 256, 256);
        float *d = reinterpret_cast<float *>(bs + align_up(size_t(nbk) * mp * 16, 256));
        cudaError_t e;
        if (rms) {
            ActPrepArgs pa = {};
            pa.mode = kActRms;
            pa.x = x + t0 * x_stride;
            pa.r = rms->r ? rms->r + t0 * x_stride : nullptr;
            pa.g = rms->g;
            pa.h_out = rms->h_out ? rms->h_out + t0 * x_stride : nullptr;
            pa.x_stride = x_stride;
            pa.k = k;
            pa.m = mt;
            pa.eps = rms->eps;
            pa.fq = qs;
            pa.fb = bs;
            pa.fd = d;
            pa.mp = mp;
            e = launch(act_prep_kernel<false, true>, dim3(unsigned((nbk + 7) / 8), unsigned(mp)), dim3(256), 0, st, pa);
            if (e != cudaSuccess) return cuda_fail(e, "act_prep launch");
        } else {
            const int64_t qwarps = nbk * mp;
            e = launch(quantize_q8K_frag_kernel, dim3(unsigned(std::min<int64_t>((qwarps + 7) / 8, 65535))), dim3(256),
                       0, st, x + t0 * x_stride, k, mt, mp, x_stride, qs, bs, d, up ? up + t0 * x_stride : nullptr);
            if (e != cudaSuccess) return cuda_fail(e, "quantize launch");
        }
        a.m = mt;
        a.act.qs = qs;
        a.act.bs = bs;
        a.act.d = d;
        a.act.mp = mp;
        for (int i = 0; i < g.n_w; i++) a.y[i] = g.y[i] + t0 * g.y_stride[i];
        // the image in shared memory when it fits beside the ring (M <= 8 and K up to about 7.7K)
        const size_t img = size_t(nbk) * mp * (256 + 16) + align_up(size_t(nbk) * mp * 4, 16);
        a.act_smem = (mp == 8 && size_t(kMmaSmem) + img <= size_t(227 * 1024)) ? int(img) : 0;
        if (mt <= 8)
            e = a.act_smem ? launch_q4k_mma_t<1, true>(a, st) : launch_q4k_mma_t<1, false>(a, st);
        else
            e = launch_q4k_mma_t<2, false>(a, st);
        if (e != cudaSuccess) return cuda_fail(e, "q4_K gemv launch");
    }
    return CPQ_SUCCESS;
}

// Launch with programmatic serialization and a (2, 1, 1) thread-block cluster.
template <typename... KArgs, typename... Args>
static cudaError_t launch_pair(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                               Args &&...args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

// Raw weight rows as a 2-D u64 tensor for the tensor-core GEMM: box = 128 rows x
// one slot (256 K elements: sb_bytes bytes of each row).
static cpq_status tc_weight_tensor_map(const uint8_t *w, int64_t n, int64_t nbk, int sb_bytes, size_t rs,
                                       CUtensorMap *out) {
    static std::mutex mu;
    static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
    const TmapKey key{w, n, nbk, rs, kTcRows, sb_bytes};
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *out = it->second;
            return CPQ_SUCCESS;
        }
    }
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return fail(CPQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {cuuint64_t(nbk) * cuuint64_t(sb_bytes / 8), cuuint64_t(n)};
    const cuuint64_t strides[1] = {cuuint64_t(rs)};
    const cuuint32_t box[2] = {cuuint32_t(sb_bytes / 8), cuuint32_t(kTcRows)};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap m;
    const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<uint8_t *>(w), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CPQ_ERR_CUDA, "cuTensorMapEncodeTiled (weights) failed (%d)", int(r));
    std::lock_guard<std::mutex> lk(mu);
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return CPQ_SUCCESS;
}

// Q6_K rows as a 2-D u8 tensor whose rows are groups of l weight rows (l * rs
// bytes, a multiple of 16); box = 240 bytes x 128 / l groups.
static cpq_status q6_tc_tensor_map(const uint8_t *w, int64_t n, size_t rs, int l, CUtensorMap *out) {
    static std::mutex mu;
    static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
    const TmapKey key{w, n, int64_t(l), rs, kTcRows, TcW<CPQ_TYPE_Q6_K>::kRowBytes};
    {
        std::lock_guard<std::mutex> lk(mu);
        auto it = cache.find(key);
        if (it != cache.end()) {
            *out = it->second;
            return CPQ_SUCCESS;
        }
    }
    EncodeTiledFn enc = encode_tiled();
    if (!enc) return fail(CPQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
    const cuuint64_t dims[2] = {cuuint64_t(l) * rs, cuuint64_t(n / l)};
    const cuuint64_t strides[1] = {cuuint64_t(l) * rs};
    const cuuint32_t box[2] = {cuuint32_t(TcW<CPQ_TYPE_Q6_K>::kRowBytes), cuuint32_t(kTcRows / l)};
    const cuuint32_t estr[2] = {1, 1};
    CUtensorMap m;
    const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<uint8_t *>(w), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(CPQ_ERR_CUDA, "cuTensorMapEncodeTiled (Q6_K rows) failed (%d)", int(r));
    std::lock_guard<std::mutex> lk(mu);
    if (cache.size() > 4096) cache.clear();
    cache.emplace(key, m);
    *out = m;
    return CPQ_SUCCESS;
}

// Rows per tensor-map row for Q6_K: the fewest whole rows whose bytes are a multiple of 16.
static int q6_tc_group(size_t rs) {
    int l = 1;
    while (l <= 8 && (size_t(l) * rs) % 16) l *= 2;
    return l;
}

// Whether the tensor-core GEMM takes weight type wt with these rows: K whole
// 256-element slots and 16-byte aligned weights; Q4_K / Q8_0 rows 16-byte
// aligned for the tensor map; dense Q6_K rows (210-byte superblocks) in
// groups of L rows whose bytes are 16-byte aligned, N a multiple of L.
static bool tc_ok(int32_t wt, const GemvArgs &g) {
    if (g.k % kQK_K) return false;
    if (wt != CPQ_TYPE_Q4_K && wt != CPQ_TYPE_Q8_0 && wt != CPQ_TYPE_Q6_K) return false;
    const int l = wt == CPQ_TYPE_Q6_K ? q6_tc_group(g.rs) : 1;
    if (l > 8 || (wt != CPQ_TYPE_Q6_K && g.rs % 16)) return false;
    // the Q6_K map spans whole rows of rs bytes, the last one included: dense rows only
    if (wt == CPQ_TYPE_Q6_K && g.rs != size_t(g.k / kQK_K) * kQ6K_Bytes) return false;
    for (int i = 0; i < g.n_w; i++)
        if (!aligned(g.w[i], 16) || (g.row_start[i + 1] - g.row_start[i]) % l) return false;
    return true;
}

template <int WT> static void (*tc_kernel())(TcArgs) {
    return WT == CPQ_TYPE_Q4_K ? gemm_q4k_tc_kernel : WT == CPQ_TYPE_Q8_0 ? gemm_q8_0_tc_kernel : gemm_q6k_tc_kernel;
}

// K ranges per (row pair, token tile) for the tensor-core GEMM, for chunks of
// at most kTcSplitMaxTokens tokens (one token tile): predicted time = waves of
// units (row pairs x s, over the SM pairs) times a unit's tensor time
// (2*256*tile_n*K/s FLOP at about 15.5 TFLOP/s per SM pair), plus, for s > 1,
// the partial planes and Y through HBM at about 6 TB/s; each range keeps >= 4
// superblocks. Measured on [5120 x 17408]: M = 64 92.5 -> 44.4 us with 3
// ranges; at M = 512 and 2048 the partial planes and the per-unit epilogue
// cost more than the idle SM pairs (114 -> 120 us, 359 -> 446 us), so larger
// chunks keep one range.
constexpr int kTcMaxSplits = 4;
constexpr int64_t kTcSplitMaxTokens = 128;
static int tc_k_splits(int64_t n, int64_t m, int64_t nbk, int sm_pairs) {
    if (m > kTcSplitMaxTokens) return 1;
    const int64_t n_tok = (m + kTcMaxTok - 1) / kTcMaxTok;
    const int64_t tile_n = int64_t(align_up(size_t((m + n_tok - 1) / n_tok), 32));
    const int64_t units = ((n + 2 * kTcRows - 1) / (2 * kTcRows)) * n_tok;
    const double k = double(nbk) * kQK_K;
    auto cost = [&](int s) {
        const double unit = 2.0 * 2 * kTcRows * double(tile_n) * k / s / 15.5e12;
        const double waves = double((units * s + sm_pairs - 1) / sm_pairs);
        return waves * unit + (s > 1 ? double(s + 1) * double(m) * double(n) * 4.0 / 6.0e12 : 0.0);
    };
    int best = 1;
    for (int s = 2; s <= kTcMaxSplits && nbk / s >= 4; s++)
        if (cost(s) < cost(best) * 0.97) best = s;
    return best;
}

// M > 16 (chunked prefill): X is quantized once (Q8_K for Q4_K / Q6_K, Q8_0 for
// Q8_0) into fp16 d*q, then each weight runs as one tcgen05 GEMM launch
// (gemm_tc.cuh) over CTA pairs. Token tiles are as few as possible and
// balanced (tile_n a multiple of 32, at most 256).
template <int WT>
static cpq_status run_tc(const GemvArgs &g, const float *x, int64_t x_stride, int64_t m, uint8_t *ws, size_t ws_bytes,
                         cudaStream_t st) {
    const int64_t k = g.k, nbk = k / kQK_K;
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return fail(CPQ_ERR_CUDA, "no current device");
    auto kern = tc_kernel<WT>();
    constexpr int smem = tc_smem<WT>();
    static std::atomic<int> set[kMaxDevices];
    if (!set[dev].load(std::memory_order_relaxed)) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
        if (e != cudaSuccess) return cuda_fail(e, "tensor-core gemm smem attribute");
        set[dev].store(1, std::memory_order_relaxed);
    }
    const int64_t n_tok_tiles = (m + kTcMaxTok - 1) / kTcMaxTok;
    const int tile_n = int(align_up(size_t((m + n_tok_tiles - 1) / n_tok_tiles), 32));
    if (n_tok_tiles > 65535) return fail(CPQ_ERR_UNSUPPORTED, "M=%lld tokens is too many for one call", (long long)m);
    __half *xh = reinterpret_cast<__half *>(ws + kWsActOffset);

    cudaError_t e;
    if (WT == CPQ_TYPE_Q8_0) {
        const int64_t groups = m * (k / kQK8_0);  // 4 lanes each
        e = launch(act_f16_q8_0_kernel, dim3(unsigned(std::min<int64_t>((groups + 63) / 64, 148 * 64))), dim3(256), 0,
                   st, x, k, m, x_stride, xh);
    } else {
        const int64_t qwarps = m * nbk;
        e = launch(act_f16_kernel, dim3(unsigned(std::min<int64_t>((qwarps + 7) / 8, 148 * 64))), dim3(256), 0, st, x,
                   k, m, x_stride, xh);
    }
    if (e != cudaSuccess) return cuda_fail(e, "fp16 activation launch");

    static thread_local TcArgs a;
    std::memset(&a, 0, sizeof a);
    cpq_status rc = f16_act_tensor_map(xh, k, m, tile_n / 2, &a.tmap_x);
    if (rc) return rc;
    a.m = m;
    a.nbk = int(nbk);
    a.tile_n = tile_n;
    a.w_rs = int64_t(g.rs);
    // partial products of K-split launches: after the activation and prologue regions
    const size_t part_off = kWsActOffset + act_region_bytes(vec_dot_type(WT), k, m) + align_up(size_t(m) * k * 4, 256);
    const size_t part_room = ws_bytes > part_off ? ws_bytes - part_off : 0;
    for (int i = 0; i < g.n_w; i++) {
        const int64_t n = g.row_start[i + 1] - g.row_start[i];
        if (n == 0) continue;
        const int64_t pairs = (n + 2 * kTcRows - 1) / (2 * kTcRows);
        if (pairs > (int64_t(1) << 30) / n_tok_tiles)
            return fail(CPQ_ERR_UNSUPPORTED, "N=%lld rows is too many for one call", (long long)n);
        if (WT == CPQ_TYPE_Q4_K) {
            if ((rc = q4k_tensor_map(g.w[i], n, k, g.rs, &a.tmap_w, kTcRows, 1))) return rc;
        } else if (WT == CPQ_TYPE_Q8_0) {
            if ((rc = tc_weight_tensor_map(g.w[i], n, nbk, TcW<CPQ_TYPE_Q8_0>::kRowBytes, g.rs, &a.tmap_w))) return rc;
        } else {
            a.q6_l = q6_tc_group(g.rs);
            if ((rc = q6_tc_tensor_map(g.w[i], n, g.rs, a.q6_l, &a.tmap_w))) return rc;
        }
        a.y = g.y[i];
        a.y_stride = g.y_stride[i];
        a.n = n;
        a.n_pairs = int(pairs);
        a.n_tok_tiles = int(n_tok_tiles);
        int splits = tc_k_splits(n, m, nbk, sm_count(dev) / 2);
        while (splits > 1 && size_t(splits) * size_t(m) * size_t(n) * 4 > part_room) splits--;
        a.k_splits = splits;
        a.part = splits > 1 ? reinterpret_cast<float *>(ws + part_off) : nullptr;
        // persistent: one CTA pair per two SMs (at most one per unit)
        const int64_t grid_pairs = std::min<int64_t>(sm_count(dev) / 2, pairs * n_tok_tiles * splits);
        e = launch_pair(kern, dim3(unsigned(2 * grid_pairs)), dim3(kTcThreads), size_t(smem), st, a);
        if (e != cudaSuccess) return cuda_fail(e, "tensor-core gemm launch");
        if (splits > 1) {
            e = launch(tc_split_reduce_kernel, dim3(unsigned(std::min<int64_t>((m * n + 255) / 256, 148 * 16))),
                       dim3(256), 0, st, a.part, splits, m, n, a.y, a.y_stride);
            if (e != cudaSuccess) return cuda_fail(e, "split reduce launch");
        }
    }
    return CPQ_SUCCESS;
}

// Quantize X once into the workspace, then run every weight against it.
static ArOut ar_out_of(const cpq_tp_ar *ar, int64_t n);
static ArIn ar_in_of(const cpq_tp_ar *ar, int64_t n);
static bool ar_ready(const cpq_tp_ar *ar, int64_t need, const char **why);

static cpq_status mul_mat_core(const cpq_tensor *const *w, cpq_tensor *const *y, int n_w, const cpq_tensor *x,
                               const cpq_prologue *pro_in, void *ws, size_t ws_bytes, cudaStream_t st,
                               const cpq_tp_ar *r_ar = nullptr, const cpq_tp_ar *y_ar = nullptr) {
    cpq_prologue pro = {CPQ_PRO_NONE, nullptr, nullptr, nullptr, 0.0f};
    if (pro_in) pro = *pro_in;
    if (pro.mode != CPQ_PRO_NONE && pro.mode != CPQ_PRO_RMS && pro.mode != CPQ_PRO_SWIGLU)
        return fail(CPQ_ERR_INVALID_ARG, "prologue mode %d", int(pro.mode));
    if (pro.mode == CPQ_PRO_SWIGLU && !pro.r) return fail(CPQ_ERR_INVALID_ARG, "SWIGLU prologue needs r (up)");
    if ((pro.r && !aligned(pro.r, 16)) || (pro.h_out && !aligned(pro.h_out, 16)))
        return fail(CPQ_ERR_UNSUPPORTED, "prologue r/h_out must be 16-byte aligned");
    // every CTA of a row reads the whole row for its RMS while others store x + r
    if (pro.h_out && x && (pro.h_out == x->data || pro.h_out == pro.r))
        return fail(CPQ_ERR_INVALID_ARG, "prologue h_out must not alias X or r");
    if (n_w < 1 || n_w > kMaxMulti) return fail(CPQ_ERR_INVALID_ARG, "n_w=%d must be in 1..%d", n_w, kMaxMulti);
    if (!w || !y) return fail(CPQ_ERR_INVALID_ARG, "weight/output arrays are null");
    MMShape s0;
    cpq_status rc = check_weight(w[0], &s0);
    if (rc) return rc;
    int64_t m = 0;
    if ((rc = check_x(x, s0.k, &m))) return rc;
    GemvArgs a = {};
    a.n_w = n_w;
    a.k = s0.k;
    a.rs = w[0]->nb[1];
    a.row_start[0] = 0;
    for (int i = 0; i < n_w; i++) {
        MMShape si;
        if ((rc = check_weight(w[i], &si))) return rc;
        if (si.wtype != s0.wtype || si.k != s0.k || w[i]->nb[1] != w[0]->nb[1])
            return fail(CPQ_ERR_INVALID_ARG, "weights sharing an input must have one type, K and row stride");
        if ((rc = check_y(y[i], si.n, m))) return rc;
        a.w[i] = static_cast<const uint8_t *>(w[i]->data);
        a.w_end[i] = si.n > 0 ? a.w[i] + size_t(si.n - 1) * w[i]->nb[1] + size_t(si.k / type_blck(si.wtype)) * type_bytes(si.wtype) : a.w[i];
        a.y[i] = static_cast<float *>(y[i]->data);
        a.y_stride[i] = int64_t(y[i]->nb[1] / 4);
        a.row_start[i + 1] = a.row_start[i] + si.n;
    }
    if (m == 0 || a.row_start[n_w] == 0) return CPQ_SUCCESS;  // empty product: nothing to launch
    const int32_t vt = vec_dot_type(s0.wtype);
    const ActLayout L = act_layout(vt, s0.k, m);
    if (!ws) return fail(CPQ_ERR_NOT_INITIALIZED, "no workspace (call cpq_init on this device first)");
    if (ws_bytes < ws_need(vt, s0.k, m))
        return fail(CPQ_ERR_WORKSPACE, "workspace %zu B < %zu B needed", ws_bytes, ws_need(vt, s0.k, m));
    if (!aligned(ws, 256)) return fail(CPQ_ERR_INVALID_ARG, "workspace must be 256-byte aligned");
    uint8_t *wsb = static_cast<uint8_t *>(ws);
    const float *xp = static_cast<const float *>(x->data);
    int64_t x_stride = int64_t(x->nb[1] / 4);

    cudaError_t e;
    ArOut mma_ar;  // verify (M = 4..16) with a fused all-reduce output
    const ArOut *mma_ar_p = nullptr;
    if (r_ar || y_ar) {
        const char *why = "";
        const bool row_path = s0.wtype == CPQ_TYPE_Q4_K && m <= kRowMaxTokens && row_smem_bytes(s0.k, int(m)) <= kSmemMax;
        const bool mma_path = s0.wtype == CPQ_TYPE_Q4_K && m > kRowMaxTokens && m <= kMmaMaxTokens;
        if (!row_path && !mma_path)
            return fail(CPQ_ERR_UNSUPPORTED, "fused allreduce: Q4_K with M <= %d only", kMmaMaxTokens);
        if (r_ar) {
            if (pro.mode != CPQ_PRO_RMS || pro.r)
                return fail(CPQ_ERR_INVALID_ARG, "fused allreduce input: the prologue must be RMS with r = NULL");
            if (!ar_ready(r_ar, m * s0.k, &why)) return fail(CPQ_ERR_INVALID_ARG, "fused allreduce input: %s", why);
        }
        if (y_ar) {
            if (n_w != 1) return fail(CPQ_ERR_INVALID_ARG, "fused allreduce output: one weight per call");
            if (!ar_ready(y_ar, m * a.row_start[1], &why))
                return fail(CPQ_ERR_INVALID_ARG, "fused allreduce output: %s", why);
        }
        if (row_path) {
            // decode: the all-reduce lives in the row GEMV and its act_prep
            ArIn ain;
            ArOut aout;
            if (r_ar) ain = ar_in_of(r_ar, s0.k);
            if (y_ar) aout = ar_out_of(y_ar, a.row_start[1]);
            return run_q4k_row(a, xp, x_stride, int(m), pro, wsb, st, r_ar ? &ain : nullptr, y_ar ? &aout : nullptr);
        }
        // verify: the input's all-reduce is added to x first (h_out, or a workspace row block),
        // then the RMS prologue and the MMA GEMV run as without it; the output's goes out of the GEMV
        if (r_ar) {
            if (x_stride != s0.k || s0.k % 8)
                return fail(CPQ_ERR_UNSUPPORTED, "fused allreduce input at M > %d: dense rows, K %% 8 = 0", kRowMaxTokens);
            float *hsum = pro.h_out ? pro.h_out
                                    : reinterpret_cast<float *>(wsb + kWsActOffset + act_region_bytes(vt, s0.k, m));
            ArIn in = ar_in_of(r_ar, s0.k);
            const dim3 grid(unsigned((s0.k + 2047) / 2048), unsigned(m));
            in.n_ctas = grid.x * grid.y;
            e = launch(ar_add_kernel, grid, dim3(256), 0, st, in, xp, hsum, s0.k);
            if (e != cudaSuccess) return cuda_fail(e, "all-reduce add launch");
            xp = hsum;
            pro.h_out = nullptr;
        }
        if (y_ar) {
            mma_ar = ar_out_of(y_ar, a.row_start[1]);
            mma_ar_p = &mma_ar;
        }
    }
    if (s0.wtype == CPQ_TYPE_Q4_K && m <= kRowMaxTokens && row_smem_bytes(s0.k, int(m)) <= kSmemMax)
        return run_q4k_row(a, xp, x_stride, int(m), pro, wsb, st);

    if (pro.mode == CPQ_PRO_SWIGLU && s0.wtype == CPQ_TYPE_Q4_K && m <= kMmaMaxTokens && aligned(xp, 16) &&
        x_stride % 4 == 0)
        return run_q4k_mma(a, xp, x_stride, m, wsb, st, pro.r, mma_ar_p);  // SwiGLU inside the quantizer
    if (pro.mode == CPQ_PRO_RMS && s0.wtype == CPQ_TYPE_Q4_K && m <= kMmaMaxTokens && aligned(xp, 16) &&
        x_stride % 4 == 0)
        return run_q4k_mma(a, xp, x_stride, m, wsb, st, nullptr, mma_ar_p, &pro);  // RMS + image in one launch
    if (pro.mode != CPQ_PRO_NONE) {
        // the other paths quantize an fp32 input: apply the prologue into the workspace first
        float *tmp = reinterpret_cast<float *>(wsb + kWsActOffset + act_region_bytes(vt, s0.k, m));
        if (pro.mode == CPQ_PRO_RMS && s0.k % 4 == 0 && s0.k <= kRmsFastMaxK && x_stride % 4 == 0 && aligned(xp, 16) &&
            (!pro.g || aligned(pro.g, 16)))
            e = launch(prologue_rms_fast_kernel, dim3(unsigned(m)), dim3(kRmsFastThreads), 0, st, xp, pro.r, pro.g,
                       pro.h_out, x_stride, s0.k, pro.eps, tmp);
        else
            e = launch(prologue_f32_kernel, dim3(unsigned(m)), dim3(256), 0, st, int(pro.mode), xp, pro.r, pro.g,
                       pro.h_out, x_stride, s0.k, pro.eps, tmp);
        if (e != cudaSuccess) return cuda_fail(e, "prologue launch");
        xp = tmp;
        x_stride = s0.k;
    }
    if (s0.wtype == CPQ_TYPE_Q4_K)
        return m > kMmaMaxTokens ? run_tc<CPQ_TYPE_Q4_K>(a, xp, x_stride, m, wsb, ws_bytes, st)
                                 : run_q4k_mma(a, xp, x_stride, m, wsb, st, nullptr, mma_ar_p);
    if (m > kTcMinTokens && tc_ok(s0.wtype, a))
        return s0.wtype == CPQ_TYPE_Q8_0 ? run_tc<CPQ_TYPE_Q8_0>(a, xp, x_stride, m, wsb, ws_bytes, st)
                                         : run_tc<CPQ_TYPE_Q6_K>(a, xp, x_stride, m, wsb, ws_bytes, st);

    if (s0.wtype == CPQ_TYPE_Q8_0 && m == 1 && aligned(xp, 16)) {
        // a single token: the row-pair kernel quantizes it itself (one launch instead of two)
        GemvArgs g = a;
        g.act.qs = reinterpret_cast<const int8_t *>(wsb + kWsActOffset);  // alignment checks only
        g.act.d = reinterpret_cast<const float *>(wsb + kWsActOffset);
        if (q8_rows_ok(g, 1)) {
            e = launch_q8_rows(g, 1, st, xp, x_stride);
            return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "gemv launch");
        }
    }
    void *act_ws = wsb + kWsActOffset;
    e = launch_quantize(vt, xp, s0.k, m, x_stride, act_ws, L, nullptr, st);
    if (e != cudaSuccess) return cuda_fail(e, "quantize launch");

    const uint8_t *base = static_cast<const uint8_t *>(act_ws);
    const int64_t blk = type_blck(vt);
    const bool q6m = s0.wtype == CPQ_TYPE_Q6_K && q6m_ok(a, m);
    const int64_t group = q6m ? 16 : kGemvMaxTokens;  // tokens per weight pass
    for (int64_t t0 = 0; t0 < m; t0 += group) {
        const int mt = int(std::min<int64_t>(group, m - t0));
        GemvArgs g = a;
        g.act.qs = reinterpret_cast<const int8_t *>(base + L.qs_off) + t0 * s0.k;
        g.act.d = reinterpret_cast<const float *>(base + L.d_off) + t0 * (s0.k / blk);
        g.act.bsums = reinterpret_cast<const int16_t *>(base + L.bs_off) + t0 * (s0.k / 16);
        for (int i = 0; i < n_w; i++) g.y[i] = a.y[i] + t0 * a.y_stride[i];
        switch (s0.wtype) {
        case CPQ_TYPE_Q6_K:
            e = q6m ? launch_q6k_mma(g, mt, st) : q6k_rows_ok(g, mt) ? launch_q6k_rows(g, mt, st)
                                                                     : launch_gemv<FmtQ6K>(g, mt, st);
            break;
        default: e = q8_rows_ok(g, mt) ? launch_q8_rows(g, mt, st) : launch_gemv<FmtQ8_0>(g, mt, st); break;
        }
        if (e != cudaSuccess) return cuda_fail(e, "gemv launch");
    }
    return CPQ_SUCCESS;
}

static cpq_status workspace_of_current(void **ws, size_t *bytes) {
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return fail(CPQ_ERR_CUDA, "no current CUDA device");
    std::lock_guard<std::mutex> lk(g_mu);
    *ws = g_dev[dev].ws;
    *bytes = g_dev[dev].ws_bytes;
    if (!*ws) return fail(CPQ_ERR_NOT_INITIALIZED, "cpq_init was not called for device %d", dev);
    return CPQ_SUCCESS;
}

static int64_t grid_1d(int64_t n, int threads) {
    return std::max<int64_t>(1, std::min<int64_t>((n + threads - 1) / threads, 4096));
}

}  // namespace cpq

using namespace cpq;

extern "C" {

int cpq_abi_version(void) { return CPQ_ABI_VERSION; }

const char *cpq_last_error(void) { return g_last_error.c_str(); }

const char *cpq_status_string(cpq_status s) {
    switch (s) {
    case CPQ_SUCCESS: return "success";
    case CPQ_ERR_INVALID_ARG: return "invalid argument";
    case CPQ_ERR_UNSUPPORTED: return "unsupported";
    case CPQ_ERR_NOT_INITIALIZED: return "not initialized";
    case CPQ_ERR_WORKSPACE: return "workspace too small";
    case CPQ_ERR_CUDA: return "CUDA error";
    case CPQ_ERR_NCCL: return "NCCL error";
    case CPQ_ERR_DEVICE: return "device-side error";
    default: return "unknown status";
    }
}

cpq_status cpq_init(int device, size_t workspace_bytes) {
    int ndev = 0;
    cudaError_t e = cudaGetDeviceCount(&ndev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
    if (device < 0 || device >= ndev || device >= kMaxDevices) return fail(CPQ_ERR_INVALID_ARG, "device %d out of range", device);
    std::lock_guard<std::mutex> lk(g_mu);
    DevState &ds = g_dev[device];
    if (ds.ws && ds.ws_bytes >= workspace_bytes) return CPQ_SUCCESS;
    int prev = 0;
    cudaGetDevice(&prev);
    if ((e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    if (ds.ws) {
        cudaDeviceSynchronize();
        cudaFree(ds.ws);
        ds.ws = nullptr;
        ds.ws_bytes = 0;
    }
    const size_t bytes = std::max<size_t>(workspace_bytes, kWsActOffset + 256);
    e = cudaMalloc(&ds.ws, bytes);
    if (e == cudaSuccess) e = cudaMemset(ds.ws, 0, kWsActOffset);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaSetDevice(prev);
    if (e != cudaSuccess) {
        if (ds.ws) cudaFree(ds.ws);
        ds.ws = nullptr;
        return cuda_fail(e, "cudaMalloc(workspace)");
    }
    ds.ws_bytes = bytes;
    return CPQ_SUCCESS;
}

cpq_status cpq_release(int device) {
    if (device < 0 || device >= kMaxDevices) return fail(CPQ_ERR_INVALID_ARG, "device %d out of range", device);
    std::lock_guard<std::mutex> lk(g_mu);
    DevState &ds = g_dev[device];
    if (!ds.ws) return CPQ_SUCCESS;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    cudaDeviceSynchronize();
    cudaError_t e = cudaFree(ds.ws);
    cudaSetDevice(prev);
    ds.ws = nullptr;
    ds.ws_bytes = 0;
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "cudaFree(workspace)");
}

size_t cpq_mul_mat_workspace_size(const cpq_tensor *w, const cpq_tensor *x) {
    if (!w || !x) return 0;
    const int32_t vt = vec_dot_type(w->type);
    if (vt < 0 || x->ne[1] < 0 || w->ne[0] <= 0) return 0;
    const int64_t m = std::max<int64_t>(x->ne[1], 1), k = w->ne[0], n = std::max<int64_t>(w->ne[1], 1);
    size_t need = ws_need(vt, k, m);
    if (m > kTcMinTokens && k % kQK_K == 0) {  // room for the tensor-core GEMM's K-split partials
        const int dev = current_device();
        const int splits = dev >= 0 ? tc_k_splits(n, m, k / kQK_K, sm_count(dev) / 2) : 1;
        if (splits > 1) need += size_t(splits) * size_t(m) * size_t(n) * 4;
    }
    return need;
}

cpq_status cpq_mul_mat_ws(const cpq_tensor *w, const cpq_tensor *x, cpq_tensor *y, void *workspace,
                          size_t workspace_bytes, void *stream) {
    return mul_mat_core(&w, &y, 1, x, nullptr, workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

cpq_status cpq_mul_mat(const cpq_tensor *w, const cpq_tensor *x, cpq_tensor *y, void *stream) {
    void *ws;
    size_t bytes;
    cpq_status rc = workspace_of_current(&ws, &bytes);
    if (rc) return rc;
    return mul_mat_core(&w, &y, 1, x, nullptr, ws, bytes, static_cast<cudaStream_t>(stream));
}

cpq_status cpq_mul_mat_multi(const cpq_tensor *const *w, cpq_tensor *const *y, int n_w, const cpq_tensor *x,
                             void *stream) {
    void *ws;
    size_t bytes;
    cpq_status rc = workspace_of_current(&ws, &bytes);
    if (rc) return rc;
    return mul_mat_core(w, y, n_w, x, nullptr, ws, bytes, static_cast<cudaStream_t>(stream));
}

cpq_status cpq_mul_mat_fused(const cpq_tensor *const *w, cpq_tensor *const *y, int n_w, const cpq_tensor *x,
                             const cpq_prologue *pro, void *stream) {
    void *ws;
    size_t bytes;
    cpq_status rc = workspace_of_current(&ws, &bytes);
    if (rc) return rc;
    return mul_mat_core(w, y, n_w, x, pro, ws, bytes, static_cast<cudaStream_t>(stream));
}

cpq_status cpq_mul_mat_fused_ar(const cpq_tensor *const *w, cpq_tensor *const *y, int n_w, const cpq_tensor *x,
                                const cpq_prologue *pro, cpq_tp_ar *r_ar, cpq_tp_ar *y_ar, void *stream) {
    void *ws;
    size_t bytes;
    cpq_status rc = workspace_of_current(&ws, &bytes);
    if (rc) return rc;
    return mul_mat_core(w, y, n_w, x, pro, ws, bytes, static_cast<cudaStream_t>(stream), r_ar, y_ar);
}

cpq_status cpq_quantize_act(int32_t wtype, const float *x, void *out, int64_t k, int64_t m, void *stream) {
    const int32_t vt = vec_dot_type(wtype);
    if (vt < 0) return fail(CPQ_ERR_UNSUPPORTED, "weight type %s has no quantized vec_dot_type here", type_name(wtype));
    if (k <= 0 || m < 0 || k % type_blck(vt) != 0)
        return fail(CPQ_ERR_INVALID_ARG, "k=%lld must be a positive multiple of %lld", (long long)k, (long long)type_blck(vt));
    if (m == 0) return CPQ_SUCCESS;
    if (!x || !out || !aligned(x, 16)) return fail(CPQ_ERR_INVALID_ARG, "x/out null or x not 16-byte aligned");
    if (!aligned(out, 4)) return fail(CPQ_ERR_INVALID_ARG, "out must be 4-byte aligned");
    const ActLayout L = act_layout(vt, k, m);
    cudaError_t e = launch_quantize(vt, x, k, m, k, nullptr, L, static_cast<uint8_t *>(out), static_cast<cudaStream_t>(stream));
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "quantize launch");
}

cpq_status cpq_rms_norm(const float *x, const float *g, float *out, int64_t k, int64_t m, float eps, void *stream) {
    if (!x || !out || k <= 0 || m < 0) return fail(CPQ_ERR_INVALID_ARG, "rms_norm arguments");
    if (m == 0) return CPQ_SUCCESS;
    if (m > 2147483647) return fail(CPQ_ERR_INVALID_ARG, "rms_norm: too many rows");
    cudaError_t e = launch(rms_norm_kernel, dim3(unsigned(m)), dim3(256), 0, static_cast<cudaStream_t>(stream), x, g, out, k, eps);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "rms_norm launch");
}

cpq_status cpq_swiglu(const float *gate, const float *up, float *act, int64_t n, void *stream) {
    if (!gate || !up || !act || n < 0) return fail(CPQ_ERR_INVALID_ARG, "swiglu arguments");
    if (n == 0) return CPQ_SUCCESS;
    cudaError_t e = launch(swiglu_kernel, dim3(unsigned(grid_1d(n, 256))), dim3(256), 0, static_cast<cudaStream_t>(stream), gate, up, act, n);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "swiglu launch");
}

cpq_status cpq_add_inplace(float *y, const float *x, int64_t n, void *stream) {
    if (!y || !x || n < 0) return fail(CPQ_ERR_INVALID_ARG, "add arguments");
    if (n == 0) return CPQ_SUCCESS;
    cudaError_t e = launch(add_inplace_kernel, dim3(unsigned(grid_1d(n, 256))), dim3(256), 0, static_cast<cudaStream_t>(stream), y, x, n);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "add launch");
}

cpq_status cpq_argmax(const float *x, int64_t n, int64_t m, int32_t *out, void *stream) {
    if (!x || !out || n <= 0 || m < 0 || n > 2147483647) return fail(CPQ_ERR_INVALID_ARG, "argmax arguments");
    if (m == 0) return CPQ_SUCCESS;
    if (m > kArgmaxMaxRows) return fail(CPQ_ERR_UNSUPPORTED, "argmax: at most %d rows per call", kArgmaxMaxRows);
    void *ws;
    size_t bytes;
    cpq_status rc = workspace_of_current(&ws, &bytes);
    if (rc) return rc;
    // aux area (after the counters, partials and piece words): [rows][chunks] values, indices, then row counters
    uint8_t *aux = static_cast<uint8_t *>(ws) + kWsAuxOffset;
    float *pval = reinterpret_cast<float *>(aux);
    int32_t *pidx = reinterpret_cast<int32_t *>(aux + size_t(kArgmaxMaxRows) * kArgmaxChunks * 4);
    int *cnt = reinterpret_cast<int *>(aux + size_t(kArgmaxMaxRows) * kArgmaxChunks * 8);
    const int64_t nchunk = std::min<int64_t>(kArgmaxChunks, (n + 2047) / 2048);
    const int64_t chunk = (n + nchunk - 1) / nchunk;
    cudaError_t e = launch(argmax_kernel, dim3(unsigned(nchunk), unsigned(m)), dim3(256), 0,
                           static_cast<cudaStream_t>(stream), x, n, chunk, pval, pidx, cnt, out);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "argmax launch");
}

cpq_status cpq_synth_weights(int32_t type, void *dst, int64_t n_rows, int64_t n_blk, size_t row_stride, uint64_t seed,
                             int64_t row0, int64_t blk0, void *stream) {
    if (vec_dot_type(type) < 0) return fail(CPQ_ERR_UNSUPPORTED, "synth: type %s", type_name(type));
    const int bb = int(type_bytes(type));
    if (!dst || n_rows < 0 || n_blk < 0 || row0 < 0 || blk0 < 0) return fail(CPQ_ERR_INVALID_ARG, "synth arguments");
    if (row_stride < size_t(n_blk) * size_t(bb) || row_stride % 2 || !aligned(dst, 2))
        return fail(CPQ_ERR_INVALID_ARG, "synth: row stride %zu / alignment", row_stride);
    if (n_rows == 0 || n_blk == 0) return CPQ_SUCCESS;
    if (n_rows > 2147483647) return fail(CPQ_ERR_INVALID_ARG, "synth: too many rows");
    cudaError_t e = launch(synth_kernel, dim3(unsigned(n_rows)), dim3(128), size_t(128) * bb, static_cast<cudaStream_t>(stream),
                           type, static_cast<uint8_t *>(dst), n_blk, row_stride, bb, seed, row0, blk0);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "synth launch");
}

namespace cpq {
static cudaError_t noalloc_clear_scratch();  // noalloc.inl
}

cpq_status cpq_device_status(int device, uint32_t *err_word, int clear) {
    if (!err_word) return fail(CPQ_ERR_INVALID_ARG, "err_word is null");
    if (device < 0 || device >= kMaxDevices) return fail(CPQ_ERR_INVALID_ARG, "device %d out of range", device);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
    e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(err_word, g_dev_error, sizeof(uint32_t));
    if (e == cudaSuccess && clear) {
        // A call that gave up may have left stream-K counters and piece words
        // set: both scratch areas go back to zero with the error word.
        const uint32_t z = 0;
        e = cudaMemcpyToSymbol(g_dev_error, &z, sizeof z);
        if (e == cudaSuccess) e = noalloc_clear_scratch();
        std::lock_guard<std::mutex> lk(g_mu);
        if (e == cudaSuccess && g_dev[device].ws) e = cudaMemset(g_dev[device].ws, 0, kWsActOffset);
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
    }
    cudaSetDevice(prev);
    if (e != cudaSuccess) return cuda_fail(e, "device status");
    return *err_word ? fail(CPQ_ERR_DEVICE, "device error word 0x%x", *err_word) : CPQ_SUCCESS;
}

cpq_status cpq_set_wait_limit_ns(int device, uint64_t ns) {
    if (device < 0 || device >= kMaxDevices) return fail(CPQ_ERR_INVALID_ARG, "device %d out of range", device);
    if (ns < 1000ull || ns > 60000000000ull)
        return fail(CPQ_ERR_INVALID_ARG, "wait limit %llu ns must be in 1 us .. 60 s", (unsigned long long)ns);
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_wait_limit_ns, &ns, sizeof ns);
    cudaSetDevice(prev);
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "cpq_set_wait_limit_ns");
}

// ---- NCCL -------------------------------------------------------------------

cpq_status cpq_tp_unique_id(void *id128) {
    if (!id128) return fail(CPQ_ERR_INVALID_ARG, "id buffer is null");
    auto &n = nccl::api();
    if (!n.ok) return fail(CPQ_ERR_NCCL, "libnccl.so.2 could not be loaded");
    ncclUniqueId id;
    const int r = n.GetUniqueId(&id);
    if (r != ncclSuccess) return fail(CPQ_ERR_NCCL, "ncclGetUniqueId: %d", r);
    std::memcpy(id128, &id, sizeof id);
    return CPQ_SUCCESS;
}

cpq_status cpq_tp_comm_init(cpq_comm **comm, int nranks, int rank, const void *id128, int device, int timeout_ms) {
    if (!comm || !id128 || nranks < 1 || rank < 0 || rank >= nranks || timeout_ms <= 0)
        return fail(CPQ_ERR_INVALID_ARG, "comm_init arguments (nranks=%d rank=%d timeout=%d)", nranks, rank, timeout_ms);
    *comm = nullptr;
    auto &n = nccl::api();
    if (!n.ok) return fail(CPQ_ERR_NCCL, "libnccl.so.2 could not be loaded");
    ncclUniqueId id;
    std::memcpy(&id, id128, sizeof id);
    struct Init {
        std::mutex mu;
        bool done = false;
        int rc = -1;
        ncclComm_t c = nullptr;
    };
    auto st = std::make_shared<Init>();
    std::thread th([st, nranks, rank, id, device, &n]() {
        cudaSetDevice(device);
        ncclComm_t c = nullptr;
        const int r = n.CommInitRank(&c, nranks, id, rank);
        std::lock_guard<std::mutex> lk(st->mu);
        st->rc = r;
        st->c = c;
        st->done = true;
    });
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::milliseconds(timeout_ms);
    for (;;) {
        {
            std::lock_guard<std::mutex> lk(st->mu);
            if (st->done) break;
        }
        if (std::chrono::steady_clock::now() > deadline) {
            th.detach();  // a peer never joined; the blocked init thread is abandoned
            return fail(CPQ_ERR_NCCL, "ncclCommInitRank did not finish within %d ms", timeout_ms);
        }
        std::this_thread::sleep_for(std::chrono::milliseconds(1));
    }
    th.join();
    if (st->rc != ncclSuccess) return fail(CPQ_ERR_NCCL, "ncclCommInitRank: %d", st->rc);
    cpq_comm *c = new cpq_comm;
    c->comm = st->c;
    c->nranks = nranks;
    c->rank = rank;
    c->device = device;
    c->timeout_ms = timeout_ms;
    *comm = c;
    return CPQ_SUCCESS;
}

cpq_status cpq_tp_allreduce_f32(cpq_comm *comm, float *buf, size_t n, void *stream) {
    if (!comm || (!buf && n)) return fail(CPQ_ERR_INVALID_ARG, "allreduce arguments");
    if (n == 0 || comm->nranks == 1) return CPQ_SUCCESS;
    const int r = nccl::api().AllReduce(buf, buf, n, ncclFloat32, ncclSum, comm->comm, static_cast<cudaStream_t>(stream));
    return r == ncclSuccess ? CPQ_SUCCESS : fail(CPQ_ERR_NCCL, "ncclAllReduce: %d", r);
}

cpq_status cpq_tp_comm_check(cpq_comm *comm) {
    if (!comm) return fail(CPQ_ERR_INVALID_ARG, "comm is null");
    int async = 0;
    const int r = nccl::api().CommGetAsyncError(comm->comm, &async);
    if (r != ncclSuccess) return fail(CPQ_ERR_NCCL, "ncclCommGetAsyncError: %d", r);
    if (async != ncclSuccess && async != ncclInProgress) return fail(CPQ_ERR_NCCL, "communicator async error %d", async);
    return CPQ_SUCCESS;
}

cpq_status cpq_tp_comm_destroy(cpq_comm *comm, int abort) {
    if (!comm) return CPQ_SUCCESS;
    auto &n = nccl::api();
    const int r = abort ? n.CommAbort(comm->comm) : n.CommDestroy(comm->comm);
    delete comm;
    return r == ncclSuccess ? CPQ_SUCCESS : fail(CPQ_ERR_NCCL, "comm destroy/abort: %d", r);
}

}  // extern "C"
