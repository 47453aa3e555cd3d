// Split-KV flash decoding -- drop-in for the reference's include/flash_decoding.cuh
// (namespace, FlashDecodingConfig and launcher signature as in :5-31).
#pragma once

#include <cmath>

#include "cuda_utils.cuh"

namespace flash_engine {
namespace decoding {

// include/flash_decoding.cuh:8-19
struct FlashDecodingConfig {
  int batch_size;
  int num_heads;
  int seq_len_kv;
  int head_dim;
  int num_splits;
  float scale;

  FlashDecodingConfig(int b, int h, int m, int d, int splits = 8)
      : batch_size(b), num_heads(h), seq_len_kv(m), head_dim(d), num_splits(splits),
        scale(1.0f / std::sqrt(static_cast<float>(d))) {}
};

// q [B,H,1,d], k/v [B,H,M,d], out [B,H,1,d]; scratch_out [B,H,S,d] and
// scratch_stats [B,H,S,2] are caller-owned. The stats hold (m, l) with m in
// log2 units of the scaled score (the reference stores natural-log m; the
// buffer is scratch, only `out` is the result).
cudaError_t launch_flash_decoding_forward_fp32(const float* d_query, const float* d_key,
                                               const float* d_value, float* d_output,
                                               float* d_scratch_out, float* d_scratch_stats,
                                               const FlashDecodingConfig& config,
                                               cudaStream_t stream = nullptr);

}  // namespace decoding
}  // namespace flash_engine
