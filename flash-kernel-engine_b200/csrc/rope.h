// Internal interface of the dense RoPE kernel (rope.cu).
#pragma once

#include <cuda_runtime.h>

namespace fe {
namespace rope {

// in/out [B, H, seq, d] (dtype 0 bf16, 1 fp16, 2 fp32; out may be in); cos/sin fp32
// [>= seq, d/2]; row r of B*H*seq is rotated at position r % seq.
cudaError_t launch_rope(const void* in, const float* cos_table, const float* sin_table,
                        void* out, int B, int H, int seq, int d, int dtype, cudaStream_t stream);

// Q [B, H, N, d] and K [B, H, M, d] rotated by one launch where the row path applies
// (two otherwise): row i of each at position i % N (Q) or i % M (K).
cudaError_t launch_rope_qk(const void* q, const void* k, const float* cos_table,
                           const float* sin_table, void* q_out, void* k_out, int B, int H, int N,
                           int M, int d, int dtype, cudaStream_t stream);

}  // namespace rope
}  // namespace fe
