// Internal interface of the tcgen05 prefill kernels (prefill_sm100.cu).
#pragma once

#include <cuda_runtime.h>

namespace fe {
namespace prefill {

// bf16 (is_bf16) or fp16 Q/K/V/O [B, H, N|M, d]; fp32 accumulation. rope_cos / rope_sin
// (NULL = off): fp32 tables [rope_max_pos, d/2], 16-byte aligned; query row i and key
// row j are rotated at positions i and j before Q K^T.
cudaError_t launch_prefill(const void* q, const void* k, const void* v, void* o, int B, int H,
                           int N, int M, int d, int causal, float scale, bool is_bf16,
                           const float* rope_cos, const float* rope_sin, int rope_max_pos,
                           cudaStream_t stream);

}  // namespace prefill
}  // namespace fe
