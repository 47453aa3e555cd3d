// Umbrella header of the B200 inference-attention library -- drop-in for the
// hot-path part of the reference's include/flash_engine.h:1-31: the attention
// headers, the rotary embedding that feeds attention (fused_rope.cuh) and the CUDA
// graph runner used to capture decode steps. The reference's other kernels (RMSNorm,
// activations, speculative decoding, quantized GEMM, cross-entropy) and its memory pool
// are not part of this library.
#pragma once

#include "cuda_graph_runner.h"
#include "cuda_utils.cuh"
#include "flash_attention.cuh"
#include "flash_decoding.cuh"
#include "paged_attention.cuh"
#include "flash_engine_c.h"
#include "fused_rope.cuh"

namespace flash_engine {

constexpr int VERSION_MAJOR = 1;
constexpr int VERSION_MINOR = 2;
constexpr int VERSION_PATCH = 0;

inline const char* get_version() { return "1.2.0"; }

// Prints the device's name, SM count, warp size and shared-memory limits.
void print_device_info(int device_id = 0);

}  // namespace flash_engine
