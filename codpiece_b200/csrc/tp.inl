// tp.inl — NCCL communicator for the row-parallel partial-sum allreduce.
//
// codpiece's TP runs ggml's meta backend, which sums the fp32 partials of
// every row-split product with an NCCL allreduce (2 per layer; linked at
// codpiece-ggml-sys/build.rs:101-102). Here each GPU is its own process
// (torch.distributed / torchrun style) and one communicator per rank carries
// the same collective over NVLink. NCCL is loaded lazily with dlopen so the
// library itself has no link-time NCCL dependency; inside a PyTorch process
// the dlopen returns the NCCL that torch already loaded.
//
// Failure handling never waits without a bound: communicator set-up runs on
// a helper thread that the caller waits for with a deadline (a rank that
// never joins turns into CPQ_ERR_NCCL, not a hang); cpq_tp_comm_check() polls
// ncclCommGetAsyncError; destroy(abort=1) calls ncclCommAbort.
#include <nccl.h>

#include <chrono>
#include <dlfcn.h>
#include <mutex>
#include <thread>

namespace cpq {
namespace nccl {

// Types and enum values come from nccl.h (header only; no link-time NCCL).
struct Api {
    void *lib = nullptr;
    int (*GetUniqueId)(ncclUniqueId *) = nullptr;
    int (*CommInitRank)(ncclComm_t *, int, ncclUniqueId, int) = nullptr;
    int (*AllReduce)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t) = nullptr;
    int (*CommGetAsyncError)(ncclComm_t, int *) = nullptr;
    int (*CommDestroy)(ncclComm_t) = nullptr;
    int (*CommAbort)(ncclComm_t) = nullptr;
    const char *(*GetErrorString)(int) = nullptr;
    bool ok = false;
};

static Api &api() {
    static Api a;
    static std::once_flag once;
    std::call_once(once, [] {
        const char *names[] = {"libnccl.so.2", "libnccl.so"};
        for (const char *n : names) {
            a.lib = dlopen(n, RTLD_NOW | RTLD_GLOBAL);
            if (a.lib) break;
        }
        if (!a.lib) return;
        a.GetUniqueId = reinterpret_cast<int (*)(ncclUniqueId *)>(dlsym(a.lib, "ncclGetUniqueId"));
        a.CommInitRank = reinterpret_cast<int (*)(ncclComm_t *, int, ncclUniqueId, int)>(dlsym(a.lib, "ncclCommInitRank"));
        a.AllReduce = reinterpret_cast<int (*)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t)>(
            dlsym(a.lib, "ncclAllReduce"));
        a.CommGetAsyncError = reinterpret_cast<int (*)(ncclComm_t, int *)>(dlsym(a.lib, "ncclCommGetAsyncError"));
        a.CommDestroy = reinterpret_cast<int (*)(ncclComm_t)>(dlsym(a.lib, "ncclCommDestroy"));
        a.CommAbort = reinterpret_cast<int (*)(ncclComm_t)>(dlsym(a.lib, "ncclCommAbort"));
        a.GetErrorString = reinterpret_cast<const char *(*)(int)>(dlsym(a.lib, "ncclGetErrorString"));
        a.ok = a.GetUniqueId && a.CommInitRank && a.AllReduce && a.CommGetAsyncError && a.CommDestroy && a.CommAbort;
    });
    return a;
}

}  // namespace nccl
}  // namespace cpq

struct cpq_comm {
    ncclComm_t comm = nullptr;
    int nranks = 0, rank = 0, device = 0, timeout_ms = 0;
};
