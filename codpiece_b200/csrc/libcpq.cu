// libcpq.cu — single translation unit of libcpq.so (sm_100a only).
//
// One TU keeps the per-device error word a plain __device__ variable without
// relocatable device code. Parts:
//   quantize.cuh     activation re-quantization (Q8_K, Q8_0), bit-exact
//   gemv.cuh         small-M fused dequant GEMV/GEMM (TMA bulk-copy ring)
//   elementwise.cuh  rms norm, SwiGLU, residual add, argmax
//   synth.cuh        seeded synthetic weights
//   split.inl        tensor-parallel partition rules (host)
//   tp.inl           NCCL communicator (host)
//   api.inl          extern "C" entry points declared in include/cpq.h
#if defined(__CUDA_ARCH__) && __CUDA_ARCH__ < 1000
#error "libcpq targets sm_100a (B200) only"
#endif

#include <algorithm>
#include <cstring>
#include <memory>
#include <utility>

#include "common.cuh"
#include "elementwise.cuh"
#include "gemv.cuh"
#include "quantize.cuh"
#include "synth.cuh"
#include "split.inl"
#include "tp.inl"
#include "api.inl"
