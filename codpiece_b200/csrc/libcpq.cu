// libcpq.cu — single translation unit of libcpq.so (sm_100a only).
//
// One TU keeps the per-device error word a plain __device__ variable without
// relocatable device code. Parts:
//   quantize.cuh     activation re-quantization (Q8_K, Q8_0), bit-exact
//   gemv.cuh         small-M fused dequant GEMV/GEMM, dp4a (Q6_K, Q8_0)
//   gemv_q6k.cuh     Q6_K and Q8_0 small-M GEMVs over whole row pairs (LM head, Q8_0 trunk)
//   gemv_q6k_mma.cuh Q6_K for M <= 16 on int8 MMA tiles of 8 rows (the head in verify)
//   q8k_block.cuh    the Q8_K block quantizer shared by every Q8_K producer
//   gemv_mma.cuh     Q4_K verify GEMM (M 4..16) on int8 mma tiles, stream-K
//   act_prep.cuh     decode activation image: fused rms/swiglu prologue + Q8_K
//   gemv_row.cuh     Q4_K decode GEMV (M 1..3), lane per row
//   gemm_tc.cuh      chunked-prefill GEMM (M > 16) on tcgen05 tensor cores: Q4_K, Q8_0, Q6_K
//   decode.cuh       persistent decode step: a chain of Q4_K GEMV phases in one launch
//   trunk.cuh        persistent decode trunk: every layer of a rank's step in one launch
//   gdn.cuh          gated delta-net recurrence (the GDN layers' per-token state update)
//   elementwise.cuh  rms norm, SwiGLU, residual add, argmax
//   synth.cuh        seeded synthetic weights
//   split.inl        tensor-parallel partition rules (host)
//   tp.inl           NCCL communicator (host)
//   api.inl          extern "C" entry points declared in include/cpq.h
//   noalloc.inl      cpq_mul_mat_noalloc: decode GEMV on static device scratch
//   plan.inl         cpq_decode_plan_*: host side of the persistent decode kernel
//   tp_ar.inl        cpq_tp_ar_*: the fused allreduce channel over NVLink peer memory
//   trunk.inl        cpq_trunk_*: host side of the persistent decode trunk
//   gguf.inl         cpq_gguf_*: GGUF reader and tensor-parallel shard loader (host)
//   gdn.inl          cpq_gated_delta_net: host side of gdn.cuh
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ < 1000
#error "libcpq targets sm_100a (B200) only"
#endif

#include <algorithm>
#include <cstring>
#include <memory>
#include <utility>
#include <vector>

#include "common.cuh"
#include "elementwise.cuh"
#include "gemv.cuh"
#include "gemv_q6k.cuh"
#include "gemv_q6k_mma.cuh"
#include "gemv_mma.cuh"
#include "act_prep.cuh"
#include "gemv_row.cuh"
#include "gemm_tc.cuh"
#include "decode.cuh"
#include "trunk.cuh"
#include "gdn.cuh"
#include "quantize.cuh"
#include "synth.cuh"
#include "split.inl"
#include "tp.inl"
#include "api.inl"
#include "noalloc.inl"
#include "plan.inl"
#include "tp_ar.inl"
#include "trunk.inl"
#include "gguf.inl"
#include "gdn.inl"
