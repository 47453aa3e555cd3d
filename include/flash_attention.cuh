// FA2 prefill forward -- drop-in for the reference's include/flash_attention.cuh
// (namespaces, AttentionConfig and launcher signatures as in :7-86).
#pragma once

#include <cmath>

#include "cuda_utils.cuh"

namespace flash_engine {
namespace attention {

// include/flash_attention.cuh:10-22
struct AttentionConfig {
  int batch_size;       // B
  int num_heads;        // H
  int seq_len_q;        // N
  int seq_len_kv;       // M
  int head_dim;         // d
  bool is_causal;       // top-left aligned causal mask (query i sees keys j <= i)
  float softmax_scale;  // 1 / sqrt(d)

  AttentionConfig(int b, int h, int sq, int skv, int d, bool causal = false)
      : batch_size(b), num_heads(h), seq_len_q(sq), seq_len_kv(skv), head_dim(d),
        is_causal(causal), softmax_scale(1.0f / std::sqrt(static_cast<float>(d))) {}
};

// Tile shapes of this build's kernels (the reference's TilingConfig, :24-57,
// describes its own SIMT tiles; these describe the B200 ones).
template <int HEAD_DIM>
struct TilingConfig {
  static constexpr int BLOCK_M = 128;  // query rows per tcgen05 tile (M of the UMMA)
  static constexpr int BLOCK_N = 128;  // keys per KV tile
  static constexpr int HEAD_DIM_ = HEAD_DIM;
};

// fp32, d <= 128. d = 32, 64, 128 with 16-byte aligned tensors: tcgen05 tensor cores
// with 3xTF32 products (each fp32 product split into TF32 high and low parts), which
// hold the 1e-3 relative tolerance; other shapes: a CUDA-core FA2 kernel.
cudaError_t launch_flash_attention_forward_fp32(const float* d_Q, const float* d_K,
                                                const float* d_V, float* d_O,
                                                const AttentionConfig& config,
                                                cudaStream_t stream = nullptr);

// fp16 in/out, fp32 accumulate: tcgen05 tensor cores. d in {32, 64, 128}.
cudaError_t launch_flash_attention_forward_fp16(const half* d_Q, const half* d_K, const half* d_V,
                                                half* d_O, const AttentionConfig& config,
                                                cudaStream_t stream = nullptr);

// bf16 in/out, fp32 accumulate: tcgen05 tensor cores. d in {32, 64, 128}. New.
cudaError_t launch_flash_attention_forward_bf16(const __nv_bfloat16* d_Q,
                                                const __nv_bfloat16* d_K,
                                                const __nv_bfloat16* d_V, __nv_bfloat16* d_O,
                                                const AttentionConfig& config,
                                                cudaStream_t stream = nullptr);

// Row-per-thread baseline (reads M keys; the reference's kernel reads N).
cudaError_t launch_naive_attention_forward_fp32(const float* d_Q, const float* d_K,
                                                const float* d_V, float* d_O,
                                                const AttentionConfig& config,
                                                cudaStream_t stream = nullptr);

}  // namespace attention
}  // namespace flash_engine
