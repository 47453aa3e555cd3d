// Host/device utilities of the B200 attention library. Same names as the
// reference's include/cuda_utils.cuh:9-31,41-61 for the pieces user code touches
// (CUDA_CHECK, WARP_SIZE, FULL_MASK, warp reductions); written for this build.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cstdio>
#include <cstdlib>

#ifndef WARP_SIZE
#define WARP_SIZE 32
#endif
#ifndef FULL_MASK
#define FULL_MASK 0xffffffffu
#endif

// Aborts the process on a failed CUDA runtime call (host utilities and tests only;
// the launchers return their status instead).
#define CUDA_CHECK(call)                                                          \
  do {                                                                            \
    cudaError_t fe_err_ = (call);                                                 \
    if (fe_err_ != cudaSuccess) {                                                 \
      std::fprintf(stderr, "CUDA error at %s:%d: %s\n", __FILE__, __LINE__,       \
                   cudaGetErrorString(fe_err_));                                  \
      std::exit(EXIT_FAILURE);                                                    \
    }                                                                             \
  } while (0)

#define CUDA_CHECK_LAST_ERROR() CUDA_CHECK(cudaGetLastError())

namespace flash_engine {
namespace cuda {

// Butterfly reductions: the result is valid in every lane.
__device__ __forceinline__ float warp_reduce_sum(float v) {
#pragma unroll
  for (int o = WARP_SIZE / 2; o > 0; o >>= 1) v += __shfl_xor_sync(FULL_MASK, v, o);
  return v;
}
__device__ __forceinline__ float warp_reduce_max(float v) {
#pragma unroll
  for (int o = WARP_SIZE / 2; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(FULL_MASK, v, o));
  return v;
}
__device__ __forceinline__ float warp_broadcast(float v, int src_lane = 0) {
  return __shfl_sync(FULL_MASK, v, src_lane);
}

constexpr float NEG_INFINITY = -1e30f;  // the reference's mask constant

}  // namespace cuda
}  // namespace flash_engine
