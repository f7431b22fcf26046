/*
 * cpq.h — C ABI of codpiece-b200's quantized mul_mat (libcpq.so).
 *
 * Drop-in target: the ggml_mul_mat node that codpiece's graph builder issues
 * for every projection (crates/codpiece-model/src/qwen35.rs:2575-2583, 2758,
 * 2779-2782, 2797, 3029, 3047, 3051, 3197; mtp_graph.rs:184-230; dflash.rs:
 * 449-847). codpiece reaches ggml through bindgen over
 * crates/codpiece-ggml-sys/wrapper.h:1-9 (build.rs:108-127); this header is
 * written to be consumed the same way (plain C, no CUDA or torch types: the
 * stream is a void*).
 *
 * Conventions follow ggml (crates/codpiece-ggml-sys/tests/smoke.rs:29-54):
 *   W: ne = [K, N], type Q4_K / Q6_K / Q8_0, rows of K contiguous blocks
 *   X: ne = [K, M], F32
 *   Y: ne = [N, M], F32, Y[m*N + n] = dot(W row n, X row m)
 * with X re-quantized on the device to W's vec_dot_type (Q8_K for Q4_K/Q6_K,
 * Q8_0 for Q8_0) exactly as ggml-cpu does before its integer block dots.
 *
 * All pointers in cpq_tensor.data are device pointers owned by the caller.
 * Every call is asynchronous on the given stream. No call aborts: failures
 * return a cpq_status and cpq_last_error() describes the last one on the
 * calling thread.
 */
#ifndef CPQ_H
#define CPQ_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define CPQ_ABI_VERSION 1

/* ggml_type ids as serialized in GGUF (crates/codpiece-gguf/src/lib.rs:170-205). */
typedef enum {
    CPQ_TYPE_F32 = 0,
    CPQ_TYPE_F16 = 1,
    CPQ_TYPE_Q8_0 = 8,
    CPQ_TYPE_Q4_K = 12,
    CPQ_TYPE_Q6_K = 14,
    CPQ_TYPE_Q8_K = 15,
} cpq_type;

/* Status codes. 0 matches GGML_STATUS_SUCCESS; a non-zero status is what the
 * caller maps to its own error (codpiece: qwen35.rs:3617-3619 maps a
 * non-SUCCESS compute status to ModelError). */
typedef enum {
    CPQ_SUCCESS = 0,
    CPQ_ERR_INVALID_ARG = 1,     /* null pointer, shape mismatch, bad size */
    CPQ_ERR_UNSUPPORTED = 2,     /* type/layout outside the fast path */
    CPQ_ERR_NOT_INITIALIZED = 3, /* no workspace on the current device */
    CPQ_ERR_WORKSPACE = 4,       /* workspace too small for this call */
    CPQ_ERR_CUDA = 5,            /* a CUDA runtime call failed */
    CPQ_ERR_NCCL = 6,            /* NCCL missing or a collective failed */
    CPQ_ERR_DEVICE = 7,          /* a kernel reported a device-side error */
} cpq_status;

/* Tensor descriptor: the subset of ggml_tensor (ggml.h: type, ne[4], nb[4],
 * data) the operator reads. ne[0] is the contiguous dimension; nb are byte
 * strides. */
typedef struct cpq_tensor {
    int32_t type;
    int64_t ne[4];
    size_t nb[4];
    void *data;
} cpq_tensor;

/* ---- library / device set-up ------------------------------------------- */

/* Allocates the per-device workspace the hot calls use (activation blocks and
 * split partials) so that cpq_mul_mat never allocates. Replaces the pool that
 * ggml-cuda's backend context owns for its mul_mat scratch. Calling it again
 * with a larger size grows the workspace (not during stream capture). */
cpq_status cpq_init(int device, size_t workspace_bytes);
/* Frees the workspace of one device. */
cpq_status cpq_release(int device);

/* Workspace bytes cpq_mul_mat/cpq_mul_mat_ws need for this W/X pair. */
size_t cpq_mul_mat_workspace_size(const cpq_tensor *w, const cpq_tensor *x);

/* ---- the operator -------------------------------------------------------- */

/* Y = W x quantize(X): the execution of ggml_mul_mat(ctx, W, X)
 * (ggml.h ggml_mul_mat; call sites listed at the top of this file) for
 * W in {Q4_K, Q6_K, Q8_0}, X/Y F32, any M >= 1, ne[2] = ne[3] = 1.
 * Other types or layouts return CPQ_ERR_UNSUPPORTED without launching
 * anything. Uses the workspace from cpq_init on the current device. */
cpq_status cpq_mul_mat(const cpq_tensor *w, const cpq_tensor *x, cpq_tensor *y, void *stream);

/* Same, with a caller-provided device workspace: one persistent buffer per
 * device (at least cpq_mul_mat_workspace_size bytes, 256-byte aligned),
 * zeroed once before its first use and used by no one else. It keeps the
 * stream-K counters and the decode GEMV's hand-off words between calls (both
 * zero whenever no call is running), so it must not be a fresh allocation
 * from a shared memory pool on every call. */
cpq_status cpq_mul_mat_ws(const cpq_tensor *w, const cpq_tensor *x, cpq_tensor *y, void *workspace,
                          size_t workspace_bytes, void *stream);

/* Several weights that share one input X (q/k/v at qwen35.rs:3029-3051,
 * gate/up at qwen35.rs:2779-2780): X is quantized once and all n_w products
 * run in one launch. Every w[i] must have the same type and K. */
cpq_status cpq_mul_mat_multi(const cpq_tensor *const *w, cpq_tensor *const *y, int n_w, const cpq_tensor *x,
                             void *stream);

/* Fused prologue applied to X before it is quantized, mirroring the ops that
 * precede the projections in codpiece's layer (qwen35.rs:2534-2537 rms(),
 * 2777 residual add, 2781 silu*mul):
 *   CPQ_PRO_NONE     X
 *   CPQ_PRO_RMS      rms_norm(X + r) * g     r, g optional (NULL); when h_out is
 *                                            non-NULL, X + r is also stored there
 *                                            (the residual stream; must not alias X/r)
 *   CPQ_PRO_SWIGLU   silu(X) * r             X = gate, r = up
 * r and h_out have X's shape and row stride; g has K floats. */
typedef enum { CPQ_PRO_NONE = 0, CPQ_PRO_RMS = 1, CPQ_PRO_SWIGLU = 2 } cpq_prologue_mode;

typedef struct cpq_prologue {
    int32_t mode;
    const float *r;
    const float *g;
    float *h_out;
    float eps;
} cpq_prologue;

/* cpq_mul_mat_multi with a fused prologue: Y_i = W_i x quantize(f(X)). The
 * prologue runs once per call (inside the quantizer on the decode path), so a
 * decode layer is four of these calls (q/k/v, o, gate/up, down). */
cpq_status cpq_mul_mat_fused(const cpq_tensor *const *w, cpq_tensor *const *y, int n_w, const cpq_tensor *x,
                             const cpq_prologue *pro, void *stream);

/* No counterpart in the reference: an entry point for callers that cannot
 * allocate device memory when they run the product (under a host engine that
 * owns every device allocation, or on a thread that must not take the
 * implicit device synchronization of cudaMalloc/cudaFree). Same result as
 * cpq_mul_mat, but all scratch lives in one static device array of about
 * 1.3 MB that every GPU using the library holds until the process exits;
 * no cudaMalloc, no cudaFree, no cpq_init needed. Limits: Q4_K weights only,
 * M <= 3 tokens, K <= 32768, N <= 262144 rows; anything larger returns
 * CPQ_ERR_UNSUPPORTED without launching. CUDA sets up the library's module
 * (and so the array) on a device at the library's first use there, and the
 * first call of this entry point on a device also looks up the array's
 * device address (cudaGetSymbolAddress): both may allocate or synchronize,
 * so make the first call at start-up, before any stream capture and away from
 * latency-critical threads. All calls share the array: calls whose
 * executions overlap on the GPU race. */
cpq_status cpq_mul_mat_noalloc(const cpq_tensor *w, const cpq_tensor *x, cpq_tensor *y, void *stream);

/* Activation re-quantization as ggml-cpu's from_float for the vec_dot_type of
 * wtype (Q8_K for Q4_K/Q6_K, Q8_0 for Q8_0): m rows of k floats (row stride k)
 * into m*k/blck ggml blocks (block_q8_K 292 B, block_q8_0 34 B) at out. */
cpq_status cpq_quantize_act(int32_t wtype, const float *x, void *out, int64_t k, int64_t m, void *stream);

/* Fused decode prologue: out = rmsnorm(x) * g (g may be NULL for unit weight),
 * as codpiece's rms() (qwen35.rs:2534-2537: ggml_rms_norm then ggml_mul).
 * m rows of k floats. */
cpq_status cpq_rms_norm(const float *x, const float *g, float *out, int64_t k, int64_t m, float eps,
                        void *stream);

/* act = silu(gate) * up, elementwise over n floats (qwen35.rs:2781). */
cpq_status cpq_swiglu(const float *gate, const float *up, float *act, int64_t n, void *stream);

/* y += x, elementwise over n floats (the residual adds, qwen35.rs:2777, 2783). */
cpq_status cpq_add_inplace(float *y, const float *x, int64_t n, void *stream);

/* Per-row argmax of m rows of n floats (first index on ties), the in-graph
 * greedy pick after the LM head (qwen35.rs:2800-2818). */
cpq_status cpq_argmax(const float *x, int64_t n, int64_t m, int32_t *out, void *stream);

/* ---- decode plans: a whole chain of decode projections in one launch -------
 *
 * A decode step (M = 1) is a chain of projections in which each one's input
 * comes from the previous ones (codpiece's qwen35 trunk, qwen35.rs:2554-2786:
 * rms -> q/k/v, o, rms -> gate/up, swiglu -> down, per layer). Issued as
 * separate cpq_mul_mat_fused calls, the weight stream stops at every kernel
 * boundary. A plan runs the chain as one persistent kernel in which each
 * SM keeps prefetching the next projections' weights while the current
 * one's input is being produced. No reference counterpart: this is a graph-
 * level fusion of consecutive ggml_mul_mat nodes (each phase has exactly the
 * semantics of one cpq_mul_mat_fused call with M = 1). */

/* One phase: up to three Q4_K weights (same K and row stride) applied to one
 * input vector through the prologue of cpq_mul_mat_fused. x, r, g, h_out and
 * the y vectors are device pointers, 16-byte aligned; x and r hold K floats,
 * y[i] holds N_i = w[i]->ne[1] floats. An input may be the output of an
 * earlier phase of the same plan; a phase must not write what it reads. */
typedef struct cpq_decode_phase {
    int32_t mode;            /* CPQ_PRO_NONE / CPQ_PRO_RMS / CPQ_PRO_SWIGLU */
    int32_t n_w;             /* 1..3 */
    const float *x;          /* input [K] */
    const float *r;          /* RMS: residual added to x (or NULL); SWIGLU: up */
    const float *g;          /* RMS weight [K] (or NULL) */
    float *h_out;            /* RMS with r: x + r stored here (or NULL) */
    float eps;
    const cpq_tensor *w[3];  /* Q4_K weights */
    float *y[3];             /* outputs */
} cpq_decode_phase;

typedef struct cpq_decode_plan cpq_decode_plan;

/* Validates the phases and builds the device-side tables (allocates device
 * memory: call outside stream capture) for `device`. The pointers are baked
 * in: the plan is valid while the weights and buffers live. */
cpq_status cpq_decode_plan_create(const cpq_decode_phase *phases, int n_phases, int device, cpq_decode_plan **plan);
/* Enqueues the chain on `stream` (capturable; one CTA per SM, cooperative).
 * Consecutive runs of plans on one device must not overlap on the GPU. */
cpq_status cpq_decode_plan_run(cpq_decode_plan *plan, void *stream);
/* Frees the plan (after its last run has completed). NULL is ignored. */
void cpq_decode_plan_destroy(cpq_decode_plan *plan);

/* ---- tensor parallel ------------------------------------------------------ */

/* Split axis values (crates/codpiece-model/src/split.rs:17-31). */
typedef enum {
    CPQ_SPLIT_AXIS_0 = 0,    /* split ne[0] (K): row-parallel, ends in an allreduce */
    CPQ_SPLIT_AXIS_1 = 1,    /* split ne[1] (N): column-parallel */
    CPQ_SPLIT_AXIS_2 = 2,
    CPQ_SPLIT_MIRRORED = 3,
    CPQ_SPLIT_PARTIAL = 4,
} cpq_split_axis;

/* Model hyper-parameters the split rules read (qwen35.rs:45-148 Hparams).
 * q_has_gate = 1 for the real qwen35 attn_q (Q and gate interleaved, 2x the
 * q width); 0 for a plain q projection of n_head*head_k rows. */
typedef struct cpq_hparams {
    int64_t n_layer, n_embd, n_head, n_head_kv, head_k, head_v, n_ff;
    int64_t n_k_heads, n_v_heads, d_state, d_inner, full_attn_interval, n_vocab;
    int32_t q_has_gate;
    int32_t split_output; /* CODPIECE_SPLIT_OUTPUT: column-split the LM head */
} cpq_hparams;

/* The per-device split of one tensor: the C-facing SplitState
 * (split.rs:285-294) in the shape of ggml's meta-backend callback result
 * (meta.rs:50-121): ne[segment * n_devices + device], nr[segment]. */
typedef struct cpq_split_state {
    int32_t axis;
    uint32_t n_segments;
    int64_t ne[256];
    uint32_t nr[16];
} cpq_split_state;

/* split.rs:298-333 split_state(): classify the tensor by name, honour its
 * segments, granularity (blck = block size of the axis-0 reference tensor's
 * type) and per-layer rotation. Never fails: unknown names, bad arguments and
 * too many devices fall back to MIRRORED, like meta.rs:47-64. */
cpq_split_state cpq_tp_split_state(const char *name, const cpq_hparams *hp, int64_t extent, int64_t blck,
                                   int n_devices);

/* NCCL communicator for one rank of a tensor-parallel group (one process per
 * GPU). NCCL is loaded on first use (libnccl.so.2). The 128-byte unique id is
 * produced by rank 0 and shared by the caller (e.g. a torch.distributed
 * store). timeout_ms bounds every blocking wait in this API. */
typedef struct cpq_comm cpq_comm;
cpq_status cpq_tp_unique_id(void *id128);
cpq_status cpq_tp_comm_init(cpq_comm **comm, int nranks, int rank, const void *id128, int device,
                            int timeout_ms);
/* In-place sum of n floats across the group (the allreduce ggml's meta
 * backend inserts after every row-parallel product, docs/OPTIMIZATION-IDEAS.md:
 * 21-29). Enqueued on stream; asynchronous. */
cpq_status cpq_tp_allreduce_f32(cpq_comm *comm, float *buf, size_t n, void *stream);
/* Polls the communicator for an asynchronous error (ncclCommGetAsyncError). */
cpq_status cpq_tp_comm_check(cpq_comm *comm);
/* Destroys (or, with abort != 0, aborts) the communicator. */
cpq_status cpq_tp_comm_destroy(cpq_comm *comm, int abort);

/* ---- fused allreduce over NVLink peer memory --------------------------------
 *
 * For the row-parallel projections (attn_output, ffn_down) of the decode
 * step (M <= 3): the GEMV's row-block finalizers store their fp32 partial
 * sums straight into every rank's receive buffer (P2P stores over NVLink,
 * buffers shared through CUDA IPC), and the next fused call's RMS prologue
 * sums the ranks' partials (in rank order) while it reads its residual
 * input. This replaces cpq_tp_allreduce_f32 on the decode path. No reference
 * counterpart: codpiece sums these partials with ggml's meta-backend
 * allreduce (split.rs PARTIAL outputs, meta.rs).
 *
 * Protocol (LL, as in NCCL's LL): each value travels with the all-reduce's
 * sequence number s in one 64-bit word written by a single store, so a
 * reader that sees s in a word also sees its value; nothing else is
 * published. All ranks run the same sequence of all-reduces; s selects one
 * of four buffer slots (s % 4). A rank cannot produce s + 2 before every
 * rank that contributes to s + 1 has consumed s, so four slots also stay
 * safe when some ranks contribute nothing to an all-reduce (the persistent
 * trunk below). A consumer waits for each word at most 2 s (then the device
 * error word is set).
 */
typedef struct cpq_tp_ar cpq_tp_ar;

/* Allocates this rank's receive buffer (n_max floats per rank and slot,
 * n_max >= M * N of the projections) on `device` and writes its CUDA IPC
 * handle (64 bytes) to handle64. world <= 8. */
cpq_status cpq_tp_ar_create(int device, int world, int rank, int64_t n_max, cpq_tp_ar **ar, void *handle64);
/* Opens the other ranks' buffers from world x 64 bytes of handles in rank order. */
cpq_status cpq_tp_ar_connect(cpq_tp_ar *ar, const void *handles);
/* Closes the peers' mappings and frees the buffer (all ranks' calls must
 * have completed). NULL is ignored. */
void cpq_tp_ar_destroy(cpq_tp_ar *ar);

/* out = x + the sum over ranks of the channel's last all-reduced value, m
 * rows of k floats (waits, bounded, for every rank's partial). For the
 * consumers outside the Q4_K decode GEMV (e.g. the Q6_K LM head's residual). */
cpq_status cpq_tp_ar_add(cpq_tp_ar *ar, const float *x, float *out, int64_t k, int64_t m, void *stream);

/* A zero contribution of n floats per token (m tokens) to the next all-reduce:
 * for a rank that owns no part of a row-parallel projection in this layer
 * (at TP8 the attention split leaves half of the ranks without attention
 * rows), so every rank still produces into every all-reduce. */
cpq_status cpq_tp_ar_zero(cpq_tp_ar *ar, int64_t n, int64_t m, void *stream);
/* The greedy token of each of m rows when the LM head's rows (the vocabulary)
 * are split across the ranks (split.rs's optional N split of output.weight):
 * every rank passes its logits [m][ld] (n of them per row, global indices
 * row0 .. row0 + n - 1) and gets out[m] = the index of the largest logit of
 * the whole row, the lowest index on ties: each rank's (max, index) pair
 * crosses NVLink as LL words through the channel, one exchange, no NCCL. */
cpq_status cpq_tp_ar_argmax(cpq_tp_ar *ar, const float *logits, int64_t n, int64_t m, int64_t ld, int64_t row0,
                            int32_t *out, void *stream);

/* cpq_mul_mat_fused with a channel at either end (either may be NULL):
 *  y_ar  Y_0 (n_w must be 1) is all-reduced through the channel instead of
 *        being stored in y[0] (y[0] still gives the shape);
 *  r_ar  the RMS prologue's residual r is the sum over ranks of the last
 *        value all-reduced through the channel (pro->mode CPQ_PRO_RMS,
 *        pro->r NULL, h_out as usual).
 * Q4_K weights and M <= 3 (the decode GEMV) only; anything else returns
 * CPQ_ERR_UNSUPPORTED. */
cpq_status cpq_mul_mat_fused_ar(const cpq_tensor *const *w, cpq_tensor *const *y, int n_w, const cpq_tensor *x,
                                const cpq_prologue *pro, cpq_tp_ar *r_ar, cpq_tp_ar *y_ar, void *stream);

/* ---- the decode trunk: every layer of a decode step in one launch -----------
 *
 * The batch-1 decode trunk of one rank (codpiece's qwen35 layer,
 * qwen35.rs:2554-2786: rms -> q/k/v, o, rms -> gate/up, swiglu -> down, with
 * the residual adds) as one persistent kernel: every projection's weights
 * stream through TMA rings that run ahead across projection boundaries, the
 * hand-offs between projections are flagged words instead of kernel
 * boundaries, and under tensor parallelism the row-parallel partial sums
 * (o, down) cross NVLink inside the same kernel (the channel of
 * cpq_tp_ar_*). No reference counterpart: it fuses the consecutive
 * ggml_mul_mat nodes of a decode graph, each with the semantics of one
 * cpq_mul_mat_fused call at M = 1 (Q8_K re-quantization, integer block dots).
 * The attention core is not part of it: q stands in for the attention output
 * that feeds o (the benchmark's attention-free stack). */
typedef struct cpq_trunk_layer {
    const cpq_tensor *q, *k, *v; /* Q4_K [n_embd -> this rank's rows]; q (and o) NULL: no attention rows
                                    on this rank in this layer (tensor parallel only); k, v may be NULL */
    const cpq_tensor *o;         /* Q4_K [q rows -> n_embd]: this rank's K slice (row-parallel) */
    const cpq_tensor *gate, *up; /* Q4_K [n_embd -> this rank's ffn rows] */
    const cpq_tensor *down;      /* Q4_K [ffn rows -> n_embd]: this rank's K slice (row-parallel) */
    const float *attn_norm;      /* RMS weight [n_embd] before q/k/v, or NULL */
    const float *ffn_norm;       /* RMS weight [n_embd] before gate/up, or NULL */
    uint32_t o_ranks;            /* ranks holding attention rows in this layer (bit mask); 0 = all */
} cpq_trunk_layer;

typedef struct cpq_trunk cpq_trunk;

/* Validates the layers and builds the device-side phase table for `device`
 * (allocates device memory: call outside stream capture). ar is NULL on a
 * single GPU, else this rank's connected channel (n_max >= n_embd); every
 * rank of the group must create its trunk with the same layer count and
 * o_ranks. n_embd is a multiple of 256 up to 6144; q and ffn row counts are
 * multiples of 256. The weight pointers are baked in. */
cpq_status cpq_trunk_create(const cpq_trunk_layer *layers, int n_layers, int64_t n_embd, float eps, cpq_tp_ar *ar,
                            int device, cpq_trunk **trunk);
/* One decode step: h_out = the residual stream after the last layer for the
 * input h_in (n_embd floats each, device pointers, distinct). Capturable; one
 * cooperative launch of one CTA per SM. Runs of one trunk must not overlap
 * on the GPU; under tensor parallelism every rank runs its trunk once per
 * step. A bounded wait that gives up sets the device error word
 * (cpq_device_status). */
cpq_status cpq_trunk_run(cpq_trunk *trunk, const float *h_in, float *h_out, void *stream);
/* Phases in the trunk's table (4 per layer, plus a final fold under tensor
 * parallelism). */
int cpq_trunk_phases(const cpq_trunk *trunk);
/* Frees the trunk (after its last run has completed). NULL is ignored. */
void cpq_trunk_destroy(cpq_trunk *trunk);

/* ---- gated delta-net recurrence ---------------------------------------------
 *
 * ggml_gated_delta_net as codpiece's GDN layers call it (qwen35.rs:2719;
 * ggml-cuda gated_delta_net.cu:4-167, replacing ggml_cuda_op_gated_delta_net
 * and ggml_cuda_op_gated_delta_net_fused_cache, gated_delta_net.cuh:10-14).
 * Shapes (ggml ne order, F32; q, k, v rows contiguous, the rest contiguous):
 *   q, k   [S_v, H_qk, T, n_seqs / r]   v head h reads q/k head h % H_qk,
 *                                       sequence s reads q/k sequence s / r
 *   v      [S_v, H, T, n_seqs]          S_v = 16, 32, 64 or 128
 *   g      [1, H, T, n_seqs] (log decay per head) or [S_v, H, T, n_seqs] (per row)
 *   beta   [1, H, T, n_seqs]
 *   state  S_v * S_v * H * n_seqs       element (i, col) of head h, sequence s at
 *                                       ((s * H + h) * S_v + col) * S_v + i
 * dst: the attention rows [S_v, H, T, n_seqs] (scaled by 1/sqrt(S_v)), then the
 * state output: with n_snap (the op's K) <= 1 the state after the last token;
 * with n_snap > 1 slot j (j < min(n_snap, T)) holds the state j tokens before
 * the last, slots one state set (S_v * S_v * H * n_seqs floats) apart. With
 * cache non-NULL the state output goes there instead, slots cache_slot_stride
 * floats apart, and dst needs only the attention rows. state and the state
 * output may be the same memory. */
cpq_status cpq_gated_delta_net(const cpq_tensor *q, const cpq_tensor *k, const cpq_tensor *v, const cpq_tensor *g,
                               const cpq_tensor *beta, const cpq_tensor *state, cpq_tensor *dst, int32_t n_snap,
                               float *cache, int64_t cache_slot_stride, void *stream);

/* ---- GGUF files: tensor directory and tensor-parallel shards ---------------
 *
 * The reader of crates/codpiece-gguf/src/lib.rs:346-460 (GGUF v1-v3 header,
 * metadata, tensor directory; no tensor data at open; the same validity
 * checks: magic, version, count/length caps, power-of-two alignment, every
 * tensor aligned, in order, non-overlapping and inside the data section) and
 * the upload half of Weights::load (crates/codpiece-model/src/lib.rs:128-311),
 * with the tensor-parallel slicing done here on the host: a shard is the part
 * of a tensor that cpq_tp_split_state assigns to one device (Axis1: whole
 * rows; Axis0: K ranges of whole quant blocks in every row; MIRRORED or NULL:
 * the whole tensor), written once as dense rows. */
typedef struct cpq_gguf cpq_gguf;

typedef struct cpq_gguf_tensor {
    const char *name;  /* valid while the file handle lives */
    int32_t type;      /* ggml type id */
    int32_t n_dims;
    int64_t ne[4];     /* ne[0] contiguous; unused dimensions 1 */
    uint64_t offset;   /* absolute byte offset of the data in the file */
    uint64_t bytes;    /* 0 for a type whose size this library does not know */
} cpq_gguf_tensor;

cpq_status cpq_gguf_open(const char *path, cpq_gguf **gguf);
void cpq_gguf_close(cpq_gguf *gguf);
int64_t cpq_gguf_n_tensors(const cpq_gguf *gguf);
/* Index of the tensor called name, or -1. */
int64_t cpq_gguf_find_tensor(const cpq_gguf *gguf, const char *name);
cpq_status cpq_gguf_tensor_at(const cpq_gguf *gguf, int64_t index, cpq_gguf_tensor *tensor);
/* Metadata: a non-negative integer value, or a string (valid while the handle lives). */
cpq_status cpq_gguf_get_u64(const cpq_gguf *gguf, const char *key, uint64_t *value);
cpq_status cpq_gguf_get_str(const cpq_gguf *gguf, const char *key, const char **value);
/* Device device_index's shard of a 2-D tensor under split (NULL: the whole
 * tensor): its ne[0] x ne[1] and byte size, dense rows. */
cpq_status cpq_gguf_shard_shape(const cpq_gguf *gguf, int64_t index, const cpq_split_state *split, int n_devices,
                                int device_index, int64_t *ne0, int64_t *ne1, size_t *bytes);
/* The shard's bytes into host memory, or into device memory (synchronous copy). */
cpq_status cpq_gguf_read_shard(const cpq_gguf *gguf, int64_t index, const cpq_split_state *split, int n_devices,
                               int device_index, void *host_dst, size_t dst_bytes);
cpq_status cpq_gguf_load_shard(const cpq_gguf *gguf, int64_t index, const cpq_split_state *split, int n_devices,
                               int device_index, void *device_dst, size_t dst_bytes);

/* ---- synthetic weights ----------------------------------------------------- */

/* Fills rows [row0, row0+n_rows) x blocks [blk0, blk0+n_blk) of a tensor of
 * the given type with seeded synthetic blocks (the value distributions of the
 * benchmark configs: fp16 scales |N(0,sigma)|, uniform quants/scales), as a
 * pure function of (seed, global row, global block, byte). dst holds n_rows
 * rows of row_stride bytes. Used for random-init weights of the 27B-shaped
 * stack; a shard generated this way equals the same slice of the whole. */
cpq_status cpq_synth_weights(int32_t type, void *dst, int64_t n_rows, int64_t n_blk, size_t row_stride,
                             uint64_t seed, int64_t row0, int64_t blk0, void *stream);

/* ---- diagnostics ------------------------------------------------------------ */

/* Reads (and with clear != 0 resets) the device-side error word that kernels
 * set when a bounded wait gives up. Synchronizes the device. Clearing also
 * zeroes the stream-K scratch (counters, piece words) of the device's
 * workspace and of cpq_mul_mat_noalloc, which a call that gave up may have
 * left set; a caller-provided workspace (cpq_mul_mat_ws) must be re-zeroed
 * by its owner. */
cpq_status cpq_device_status(int device, uint32_t *err_word, int clear);
/* Sets how long any device-side wait of the library (a copy's completion, a
 * neighbouring CTA's words, a peer rank's all-reduce words) may spin before
 * it gives up and sets the device error word: 2 s by default, here 1 us to
 * 60 s, for `device` (not while its kernels run). No reference counterpart:
 * ggml's CUDA backend has no bounded waits; this bounds a stalled or dead
 * peer. */
cpq_status cpq_set_wait_limit_ns(int device, uint64_t ns);
const char *cpq_last_error(void);
const char *cpq_status_string(cpq_status s);
int cpq_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif
