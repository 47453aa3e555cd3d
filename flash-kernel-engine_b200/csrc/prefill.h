// Internal interface of the tcgen05 prefill kernels (prefill_sm100.cu).
#pragma once

#include <cuda_runtime.h>

namespace fe {
namespace prefill {

// bf16 (is_bf16) or fp16 Q/K/V/O [B, H, N|M, d]; fp32 accumulation.
cudaError_t launch_prefill(const void* q, const void* k, const void* v, void* o, int B, int H,
                           int N, int M, int d, int causal, float scale, bool is_bf16,
                           cudaStream_t stream);

}  // namespace prefill
}  // namespace fe
