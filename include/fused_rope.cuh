// Rotary position embedding -- drop-in for the reference's include/fused_rope.cuh
// (namespace, RoPEConfig and launcher signature as in :7-30). Input [B, H, seq_len,
// head_dim]; row r of B*H*seq_len has position r % seq_len; pair (2i, 2i+1) becomes
// (x0 c - x1 s, x0 s + x1 c) with c, s = cos/sin[pos][i] of fp32 tables [seq_len,
// head_dim/2] (src/fused_rope.cu:13-45). d_out may be d_in. The bf16 and fp16 siblings
// are new.
#pragma once

#include "cuda_utils.cuh"

namespace flash_engine {
namespace rope {

// include/fused_rope.cuh:9-18
struct RoPEConfig {
  int batch_size;
  int num_heads;
  int seq_len;
  int head_dim;
  float theta_base;  // informational: the tables are the caller's

  RoPEConfig(int b, int h, int s, int d, float base = 10000.0f)
      : batch_size(b), num_heads(h), seq_len(s), head_dim(d), theta_base(base) {}
};

cudaError_t launch_fused_rope_fp32(const float* d_in, const float* d_cos, const float* d_sin,
                                   float* d_out, const RoPEConfig& config,
                                   cudaStream_t stream = nullptr);
cudaError_t launch_fused_rope_bf16(const __nv_bfloat16* d_in, const float* d_cos,
                                   const float* d_sin, __nv_bfloat16* d_out,
                                   const RoPEConfig& config, cudaStream_t stream = nullptr);
cudaError_t launch_fused_rope_fp16(const half* d_in, const float* d_cos, const float* d_sin,
                                   half* d_out, const RoPEConfig& config,
                                   cudaStream_t stream = nullptr);

}  // namespace rope
}  // namespace flash_engine
