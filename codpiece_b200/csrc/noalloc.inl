// noalloc.inl — cpq_mul_mat_noalloc: the Q4_K decode GEMV with static scratch.
//
// Some callers cannot allocate device memory at the moment they need a
// product: host engines that hand all device memory out through their own
// arena and forbid the library from calling cudaMalloc, and latency-critical
// threads that must not take the implicit device synchronization a
// cudaMalloc/cudaFree can cause. For them
// this entry point runs the decode GEMV (gemv_row.cuh, unchanged) with every
// byte of its scratch — the quantized activation image and the tail-cut
// words the CTAs hand each other — in one file-scope device array that every
// GPU using the library holds until the process exits. CUDA loads a module
// lazily by default, so the array is set up on a device by the library's
// first use there (this entry point's first call, or any other cpq call
// that launches a kernel); that first use may itself allocate and
// synchronize, so make it at start-up, before any stream capture and away
// from latency-critical threads.
//
// In host code the array's name stands for a host-side shadow, not a device
// address, so its device address is looked up once per device with
// cudaGetSymbolAddress while that device is current and cached; kernels get
// that pointer. The first call on a device performs this set-up, so make the
// first call before any stream capture.
//
// Every call shares the one array: the tail-cut words are zero between calls
// (each call clears what it reads), and calls whose executions overlap on the
// GPU (e.g. on two streams at once) race on the array.
#include <mutex>

namespace cpq {

// Limits of the static scratch.
constexpr int64_t kNoAllocMaxRows = 262144;  // N (output rows)
constexpr int64_t kNoAllocMaxK = 32768;      // K
constexpr int kNoAllocMaxTokens = kRowMaxTokens;
constexpr int64_t kNoAllocMaxCtas = 148;  // CTAs given tail-cut slots (larger parts run on 148 SMs)
constexpr size_t kNoAllocPieceBytes = size_t(kNoAllocMaxCtas) * kRowWarps * kPieceWords * sizeof(uint64_t);
constexpr size_t kNoAllocActBytes = align_up(size_t(row_act_bytes(kNoAllocMaxK, kNoAllocMaxTokens)), 256);
constexpr size_t kNoAllocBytes = kNoAllocPieceBytes + kNoAllocActBytes;  // 1,318,400 B (about 1.3 MB)

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocBytes];

// Device address of g_noalloc_scratch on the current device (set up once per device).
static cpq_status noalloc_scratch(uint8_t **out) {
    static std::mutex mu;
    static uint8_t *addr[kMaxDevices] = {};
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return fail(CPQ_ERR_CUDA, "cpq_mul_mat_noalloc: no current CUDA device");
    std::lock_guard<std::mutex> lk(mu);
    if (!addr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) return cuda_fail(e, "cpq_mul_mat_noalloc: cudaGetSymbolAddress(scratch)");
        addr[dev] = static_cast<uint8_t *>(p);
    }
    *out = addr[dev];
    return CPQ_SUCCESS;
}

// Zeroes the tail-cut words of the current device's static scratch
// (after a device-side timeout left a call unfinished).
static cudaError_t noalloc_clear_scratch() {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e == cudaSuccess) e = cudaMemset(p, 0, kNoAllocPieceBytes);
    return e;
}

template <int MT>
static cudaError_t noalloc_launch_row(RowArgs &a, int smem, cudaStream_t st) {
    auto kern = gemv_q4k_row_kernel<MT>;
    const int dev = current_device();
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    static std::atomic<int> set[kMaxDevices];  // the shared-memory attribute, once per device and instance
    if (!set[dev].load(std::memory_order_relaxed)) {
        const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemMax);
        if (e != cudaSuccess) return e;
        set[dev].store(1, std::memory_order_relaxed);
    }
    const int64_t grid = row_grid(a, std::min<int64_t>(sm_count(dev), kNoAllocMaxCtas));
    return launch(kern, dim3(unsigned(grid)), dim3(kRowWarps * 32), size_t(smem), st, a);
}

}  // namespace cpq

extern "C" cpq_status cpq_mul_mat_noalloc(const cpq_tensor *w, const cpq_tensor *x, cpq_tensor *y, void *stream) {
    using namespace cpq;
    MMShape s;
    cpq_status rc = check_weight(w, &s);
    if (rc) return rc;
    if (s.wtype != CPQ_TYPE_Q4_K)
        return fail(CPQ_ERR_UNSUPPORTED, "cpq_mul_mat_noalloc: only Q4_K weights (got %s)", type_name(s.wtype));
    int64_t m = 0;
    if ((rc = check_x(x, s.k, &m))) return rc;
    if ((rc = check_y(y, s.n, m))) return rc;
    if (m == 0 || s.n == 0) return CPQ_SUCCESS;
    if (m > kNoAllocMaxTokens)
        return fail(CPQ_ERR_UNSUPPORTED, "cpq_mul_mat_noalloc: M=%lld tokens exceeds the static scratch limit of %d",
                    (long long)m, kNoAllocMaxTokens);
    if (s.k > kNoAllocMaxK)
        return fail(CPQ_ERR_UNSUPPORTED, "cpq_mul_mat_noalloc: K=%lld exceeds the static scratch limit of %lld",
                    (long long)s.k, (long long)kNoAllocMaxK);
    if (s.n > kNoAllocMaxRows)
        return fail(CPQ_ERR_UNSUPPORTED, "cpq_mul_mat_noalloc: N=%lld rows exceeds the static scratch limit of %lld",
                    (long long)s.n, (long long)kNoAllocMaxRows);
    const int smem = row_smem_bytes(s.k, int(m));
    if (smem > kSmemMax)
        return fail(CPQ_ERR_UNSUPPORTED, "cpq_mul_mat_noalloc: K=%lld, M=%lld needs %d B of shared memory",
                    (long long)s.k, (long long)m, smem);

    uint8_t *scratch = nullptr;
    if ((rc = noalloc_scratch(&scratch))) return rc;
    uint8_t *pieces = scratch;
    uint8_t *act = pieces + kNoAllocPieceBytes;
    cudaStream_t st = static_cast<cudaStream_t>(stream);

    static thread_local RowArgs a;
    std::memset(&a, 0, sizeof a);
    a.n_w = 1;
    a.n[0] = s.n;
    a.y[0] = static_cast<float *>(y->data);
    a.y_stride[0] = int64_t(y->nb[1] / 4);
    a.mb_start[1] = (s.n + kRowRows - 1) / kRowRows;
    if ((rc = q4k_tensor_map(static_cast<const uint8_t *>(w->data), s.n, s.k, w->nb[1], &a.tmap[0], kRowRows, 1)))
        return rc;
    a.nbk = int(s.k / kQK_K);
    a.m = int(m);
    a.act = act;
    a.pieces = reinterpret_cast<uint64_t *>(pieces);

    ActPrepArgs pa = {};
    pa.mode = kActPlain;
    pa.x = static_cast<const float *>(x->data);
    pa.r = nullptr;
    pa.g = nullptr;
    pa.h_out = nullptr;
    pa.x_stride = int64_t(x->nb[1] / 4);
    pa.k = s.k;
    pa.m = int(m);
    pa.eps = 0.0f;
    pa.out = act;
    cudaError_t e = launch(act_prep_kernel<false>, dim3(unsigned((a.nbk + 7) / 8), unsigned(m)), dim3(256), 0, st, pa);
    if (e != cudaSuccess) return cuda_fail(e, "cpq_mul_mat_noalloc: act_prep launch");
    switch (m) {
    case 1: e = noalloc_launch_row<1>(a, smem, st); break;
    case 2: e = noalloc_launch_row<2>(a, smem, st); break;
    default: e = noalloc_launch_row<3>(a, smem, st); break;
    }
    return e == cudaSuccess ? CPQ_SUCCESS : cuda_fail(e, "cpq_mul_mat_noalloc: gemv launch");
}
