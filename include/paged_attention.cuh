// Paged-KV decode -- drop-in for the reference's include/paged_attention.cuh
// (namespaces, PagedAttentionConfig and v1 launcher signatures as in :7-48).
// Cache layouts as the reference declares them: fp32 (and the new bf16 entries)
// [num_blocks, num_kv_heads, block_size, head_dim]; fp16 vLLM x-packed
// K [num_blocks, num_kv_heads, head_dim/8, block_size, 8], V [num_blocks,
// num_kv_heads, head_dim, block_size].
#pragma once
// The NCCL communicator handle, declared as nccl.h does (no NCCL headers needed).
typedef struct ncclComm* ncclComm_t;

#include <cmath>

#include "cuda_utils.cuh"

namespace flash_engine {
namespace paged_attention {

// include/paged_attention.cuh:10-24
struct PagedAttentionConfig {
  int num_seqs;
  int num_heads;
  int num_kv_heads;
  int head_dim;
  int block_size;
  int max_context_len;
  int max_num_blocks_per_seq;
  float scale;

  PagedAttentionConfig(int seqs, int heads, int kv_heads, int dim, int blk_size, int max_len,
                       int max_blks)
      : num_seqs(seqs), num_heads(heads), num_kv_heads(kv_heads), head_dim(dim),
        block_size(blk_size), max_context_len(max_len), max_num_blocks_per_seq(max_blks),
        scale(1.0f / std::sqrt(static_cast<float>(dim))) {}
};

// fp16 cache, vLLM layout (the reference's entry is a stub that launches nothing).
cudaError_t launch_paged_attention_v1_fp16(const half* d_query, const half* d_key_cache,
                                           const half* d_value_cache, half* d_output,
                                           const int* d_block_tables, const int* d_context_lens,
                                           const PagedAttentionConfig& config,
                                           cudaStream_t stream = nullptr);

cudaError_t launch_paged_attention_v1_fp32(const float* d_query, const float* d_key_cache,
                                           const float* d_value_cache, float* d_output,
                                           const int* d_block_tables, const int* d_context_lens,
                                           const PagedAttentionConfig& config,
                                           cudaStream_t stream = nullptr);

// New: bf16 cache, no scratch.
cudaError_t launch_paged_attention_v1_bf16(const __nv_bfloat16* d_query,
                                           const __nv_bfloat16* d_key_cache,
                                           const __nv_bfloat16* d_value_cache,
                                           __nv_bfloat16* d_output, const int* d_block_tables,
                                           const int* d_context_lens,
                                           const PagedAttentionConfig& config,
                                           cudaStream_t stream = nullptr);

// New: bf16 cache, split-KV with a caller-owned workspace of
// fe_paged_attention_v2_workspace_floats(...) floats (see flash_engine_c.h).
cudaError_t launch_paged_attention_v2_bf16(const __nv_bfloat16* d_query,
                                           const __nv_bfloat16* d_key_cache,
                                           const __nv_bfloat16* d_value_cache,
                                           __nv_bfloat16* d_output, const int* d_block_tables,
                                           const int* d_context_lens,
                                           const PagedAttentionConfig& config,
                                           float* d_workspace, size_t workspace_floats,
                                           cudaStream_t stream = nullptr);

// New: the KV-range-sharded bf16 decode step on `world` GPUs (this process is `rank`),
// decode of this rank's token window + ncclAllGather of the partials on `comm` + the
// log-sum-exp merge into the full [S, H, d] output (fe_paged_decode_kv_range_nccl_bf16).
cudaError_t launch_paged_decode_kv_range_bf16(
    const __nv_bfloat16* d_query, const __nv_bfloat16* d_key_cache,
    const __nv_bfloat16* d_value_cache, __nv_bfloat16* d_output, const int* d_block_tables,
    const int* d_context_lens, const PagedAttentionConfig& config, ncclComm_t comm, int rank,
    int world, float* d_workspace, size_t workspace_floats, float* d_scratch,
    size_t scratch_floats, cudaStream_t stream = nullptr);

}  // namespace paged_attention
}  // namespace flash_engine
