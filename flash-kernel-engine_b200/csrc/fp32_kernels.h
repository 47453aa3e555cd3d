// Internal interface of the fp32 kernels (attention_fp32.cu, prefill_tf32.cu).
#pragma once

#include <cuda_runtime.h>

namespace fe {
namespace simt {

cudaError_t launch_fa2_fp32(const float* q, const float* k, const float* v, float* o, int B, int H,
                            int N, int M, int d, float scale, int causal, cudaStream_t st);
// fp32 FA2 forward on the tensor core with 3xTF32 products (prefill_tf32.cu), used by
// launch_fa2_fp32 for head dims 32, 64 and 128 with 16-byte aligned tensors.
bool fa2_tf32_eligible(const float* q, const float* k, const float* v, const float* o, int B,
                       int H, int N, int M, int d);
cudaError_t launch_fa2_tf32(const float* q, const float* k, const float* v, float* o, int B, int H,
                            int N, int M, int d, float scale, int causal, cudaStream_t st);
cudaError_t launch_naive_fp32(const float* q, const float* k, const float* v, float* o, int B,
                              int H, int N, int M, int d, float scale, int causal, cudaStream_t st);
cudaError_t launch_paged_fp32(const float* q, const float* kc, const float* vc, float* out,
                              const int* bt, const int* lens, int S, int H, int Hkv, int d, int bs,
                              int maxb, int num_blocks, float scale, cudaStream_t st);
cudaError_t launch_decode_split_fp32(const float* q, const float* k, const float* v,
                                     float* part_o, float* part_ml, int BH, int M, int d,
                                     int splits, float scale, cudaStream_t st);

}  // namespace simt
}  // namespace fe
