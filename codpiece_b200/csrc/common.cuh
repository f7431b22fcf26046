// common.cuh — shared definitions for libcpq (sm_100a).
//
// Block formats (bytes per block from crates/codpiece-gguf/src/lib.rs:179-186):
//   Q8_0: 32 elements, 34 B  = fp16 d, int8 qs[32]
//   Q4_K: 256 elements, 144 B = fp16 d, fp16 dmin, u8 scales[12], u8 qs[128]
//   Q6_K: 256 elements, 210 B = u8 ql[128], u8 qh[64], i8 scales[16], fp16 d
//   Q8_K: 256 elements, 292 B = f32 d, i8 qs[256], i16 bsums[16]
// Inside this library activations live in a structure-of-arrays form (all
// quants of a row contiguous and 16-byte aligned, scales and 16-sums in
// separate arrays) so kernels can use vector loads; cpq_quantize_act emits
// the ggml array-of-structs bytes for callers that need them.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/cpq.h"

namespace cpq {

constexpr int kQK_K = 256;
constexpr int kQK8_0 = 32;
constexpr int kQ4K_Bytes = 144;
constexpr int kQ6K_Bytes = 210;
constexpr int kQ8_0_Bytes = 34;
constexpr int kQ8K_Bytes = 292;

// Device-side error word bits (read by cpq_device_status).
enum : uint32_t {
    kDevErrWaitTimeout = 1u << 0,  // a bounded mbarrier wait gave up
    kDevErrBadLaunch = 1u << 1,    // a kernel saw arguments it cannot handle
};

// One word per device (a __device__ variable has one instance per device).
__device__ uint32_t g_dev_error;

// Upper bound for any spin on an mbarrier, a flag or a peer's word, in
// nanoseconds of %globaltimer: 2 s unless cpq_set_wait_limit_ns changed it
// (one value per device). Read only after a wait has spun a while.
__device__ uint64_t g_wait_limit_ns = 2000000000ull;
__device__ __forceinline__ uint64_t wait_limit_ns() { return *reinterpret_cast<volatile uint64_t *>(&g_wait_limit_ns); }

// ---- PTX helpers -----------------------------------------------------------

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of an mbarrier, giving up after wait_limit_ns().
// On give-up it records kDevErrWaitTimeout and returns false.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0 && global_timer_ns() - t0 > wait_limit_ns()) {
            atomicOr(&g_dev_error, kDevErrWaitTimeout);
            return false;
        }
    }
}

// 1-D bulk copy global -> shared (TMA engine, no tensor map, no multicast).
// dst, src 16-byte aligned; bytes a multiple of 16. Completion is signalled
// as transaction bytes on `bar`.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// Same, with an L2 evict-first hint: weight bytes are streamed once per call.
__device__ __forceinline__ void bulk_g2s_stream(void *dst, const void *src, uint32_t bytes, uint64_t *bar,
                                                uint64_t policy) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(policy)
        : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
    return p;
}

// Programmatic dependent launch: wait for the preceding grid's memory, and
// let the next grid start its independent prologue early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;"); }

// Read-only global loads that bypass L1 allocation-on-miss policy games.
__device__ __forceinline__ int4 ldg_nc_v4(const void *p) {
    int4 r;
    asm volatile("ld.global.nc.v4.s32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// dot of 4 unsigned bytes (a) with 4 signed bytes (b), plus c.
__device__ __forceinline__ int dp4a_us(uint32_t a, int b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// dot of 4 unsigned bytes (a) with 4 unsigned bytes (b), plus c.
__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 16 bytes from shared memory at a 2-byte aligned address: five aligned
// words and a funnel shift (shift 0 when the address is 4-byte aligned).
__device__ __forceinline__ uint4 lds16_a2(const uint8_t *p) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    const uint32_t *w = reinterpret_cast<const uint32_t *>(a & ~uintptr_t(3));
    const uint32_t s = static_cast<uint32_t>(a & 3u) * 8u;
    const uint32_t w0 = w[0], w1 = w[1], w2 = w[2], w3 = w[3], w4 = w[4];
    return make_uint4(__funnelshift_r(w0, w1, s), __funnelshift_r(w1, w2, s), __funnelshift_r(w2, w3, s),
                      __funnelshift_r(w3, w4, s));
}

__device__ __forceinline__ float half_bits_to_float(uint32_t h16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h16 & 0xffffu)));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---- fused allreduce channel (include/cpq.h cpq_tp_ar) ----------------------
//
// LL protocol (the one NCCL's LL uses): every value crosses NVLink together
// with its sequence number in one naturally aligned 64-bit word
// (seq << 32 | fp32 bits), written with a single 64-bit store, so a reader
// that sees the expected sequence number in a word also sees that word's
// value: no fences, no flags, no counters on the producer side. Every rank's
// receive buffer holds [kArSlots][world][n_max] such words; sequence number s
// uses slot s % kArSlots. Two slots would do when every rank contributes to
// every all-reduce (a rank cannot produce s + 2 before every rank has
// consumed s); the persistent trunk (trunk.cuh) lets ranks without rows of a
// projection skip its all-reduce, and four slots keep that safe too.

constexpr int kArMaxRanks = 8;
constexpr unsigned kArSlots = 4;

// Producer side (row GEMV of a row-parallel projection).
struct ArOut {
    uint64_t *peer[kArMaxRanks];  // each rank's receive buffer (this rank's included)
    const unsigned *seq;          // this rank's count of consumed all-reduces (local)
    int64_t n_max;                // words per (slot, rank)
    int64_t n;                    // output rows (token stride in a slot)
    int world, rank;
    int on;
};

// Consumer side (the prologue that reads the all-reduced residual). The
// consumer kernel's CTAs each read seq, then the last of them (arrive
// counter) advances it.
struct ArIn {
    const uint64_t *base;         // this rank's receive buffer
    unsigned *seq;
    unsigned *arrive;             // consumer CTAs that have read seq (local, zero between calls)
    int64_t n_max, n;
    int world;
    unsigned n_ctas;              // CTAs of the consumer launch
    int on;
};

// The ranks' words for one token's row (rank s at p0 + s * stride), read
// and summed in rank order.
struct ArRows {
    const uint64_t *p0;
    int64_t stride;
    int n;
    unsigned seq;
};

// ---- flagged words between the CTAs of one grid ----------------------------
//
// A 64-bit word (flag << 32 | 32-bit payload) is stored and loaded whole, so a
// reader that sees the flag also sees the payload: nothing has to be fenced
// before the word is published.

__device__ __forceinline__ void st_relaxed_gpu_u64(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_gpu_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// Counter increment without ordering: its result is only used to elect the
// last arriver, whose reads wait on flagged words instead of on a fence.
__device__ __forceinline__ int atom_add_relaxed_gpu(int *p, int v) {
    int old;
    asm volatile("atom.relaxed.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
    return old;
}

// The word at p once its high half equals flag (bounded wait; on give-up the
// device error word is set and flag << 32 is returned, a payload of 0). Once a
// wait on this device has given up, later words are not waited for.
__device__ __forceinline__ uint64_t flagged_word_gpu(const uint64_t *p, uint32_t flag) {
    uint64_t w = ld_relaxed_gpu_u64(p);
    if (uint32_t(w >> 32) == flag) return w;
    const uint64_t t0 = global_timer_ns();
    for (uint32_t it = 1;; ++it) {
        w = ld_relaxed_gpu_u64(p);
        if (uint32_t(w >> 32) == flag) return w;
        if ((it & 63u) == 0 && ((*reinterpret_cast<volatile uint32_t *>(&g_dev_error) & kDevErrWaitTimeout) ||
                                global_timer_ns() - t0 > wait_limit_ns())) {
            atomicOr(&g_dev_error, kDevErrWaitTimeout);
            return uint64_t(flag) << 32;
        }
    }
}

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t *p, uint64_t v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t *p) {
    uint64_t v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// The value of one LL word once it carries sequence number seq (bounded wait;
// on give-up the device error word is set and 0 is returned). Once any wait
// on this device has given up, later words are not waited for at all, so a
// broken peer costs one timeout, not one per word.
__device__ __forceinline__ float ar_word(const uint64_t *p, unsigned seq) {
    uint64_t w = ld_relaxed_sys_u64(p);
    if (unsigned(w >> 32) != seq) {
        const uint64_t t0 = global_timer_ns();
        for (uint32_t it = 1;; ++it) {
            w = ld_relaxed_sys_u64(p);
            if (unsigned(w >> 32) == seq) break;
            if ((it & 63u) == 0 && ((*reinterpret_cast<volatile uint32_t *>(&g_dev_error) & kDevErrWaitTimeout) ||
                                    global_timer_ns() - t0 > wait_limit_ns())) {
                atomicOr(&g_dev_error, kDevErrWaitTimeout);
                return 0.0f;
            }
        }
    }
    return __uint_as_float(unsigned(w));
}

__device__ __forceinline__ void ld_relaxed_sys_v2u64(const uint64_t *p, uint64_t &a, uint64_t &b) {
    asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}

// The sum over ranks 0..n-1, in rank order, of eight consecutive LL words
// (rank s at p + s * stride, 16-byte aligned). The loads of kArRound ranks
// are issued before any is looked at, so n ranks cost ceil(n / kArRound)
// memory round trips, not n; a word without the expected sequence number is
// then waited for on its own.
#ifndef CPQ_AR_ROUND
#define CPQ_AR_ROUND 2
#endif
constexpr int kArRound = CPQ_AR_ROUND;
__device__ __forceinline__ void ar_sum8(const uint64_t *p, int64_t stride, int n, unsigned seq, float (&v)[8]) {
    for (int s0 = 0; s0 < n; s0 += kArRound) {
        uint64_t w[kArRound][8];
#pragma unroll
        for (int s = 0; s < kArRound; s++)
            if (s0 + s < n) {
#pragma unroll
                for (int i = 0; i < 4; i++)
                    ld_relaxed_sys_v2u64(p + (s0 + s) * stride + 2 * i, w[s][2 * i], w[s][2 * i + 1]);
            }
#pragma unroll
        for (int s = 0; s < kArRound; s++)
            if (s0 + s < n) {
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const float q = unsigned(w[s][i] >> 32) == seq ? __uint_as_float(unsigned(w[s][i]))
                                                                   : ar_word(p + (s0 + s) * stride + i, seq);
                    v[i] = s0 + s == 0 ? q : __fadd_rn(v[i], q);
                }
            }
    }
}

// Thread 0 of every consumer CTA, first: this call's sequence number. The
// load is an acquire, so the arrival after it cannot overtake it; the
// arrival's result (ticket) is only looked at by ar_consumer_end, so its
// round trip overlaps the CTA's reads of the words.
__device__ __forceinline__ unsigned ar_consumer_begin(const ArIn &ar, unsigned &ticket) {
    unsigned s;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(s) : "l"(ar.seq) : "memory");
    ticket = atomicAdd(ar.arrive, 1u);
    return s + 1u;
}

// Thread 0 of every consumer CTA, last: the CTA that arrived last (every other
// CTA has read the sequence number by then) advances the rank's count for the
// next all-reduce.
__device__ __forceinline__ void ar_consumer_end(const ArIn &ar, unsigned ticket, unsigned s) {
    if (ticket == ar.n_ctas - 1) {
        *ar.arrive = 0u;
        *reinterpret_cast<volatile unsigned *>(ar.seq) = s;
    }
}

// ---- activation views ------------------------------------------------------

// Quantized activations (structure of arrays) for M rows of K elements.
//   qs:    int8 [M][K]            (row stride K bytes, 16-byte aligned)
//   d:     f32  [M][K/blk]        (Q8_K: 1/iscale; Q8_0: the fp16 d widened)
//   bsums: i16  [M][K/16]         (Q8_K only)
struct ActQ {
    const int8_t *qs;
    const float *d;
    const int16_t *bsums;
};

// Workspace carve-up for quantized activations.
struct ActLayout {
    size_t qs_off, d_off, bs_off, bytes;
};

__host__ __device__ constexpr size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

inline ActLayout act_layout(int vec_type, int64_t k, int64_t m) {
    ActLayout l;
    const int64_t blk = vec_type == CPQ_TYPE_Q8_K ? kQK_K : kQK8_0;
    l.qs_off = 0;
    l.d_off = align_up(size_t(m) * size_t(k), 256);
    l.bs_off = align_up(l.d_off + size_t(m) * size_t(k / blk) * 4, 256);
    l.bytes = align_up(l.bs_off + (vec_type == CPQ_TYPE_Q8_K ? size_t(m) * size_t(k / 16) * 2 : 0), 256);
    return l;
}

}  // namespace cpq
