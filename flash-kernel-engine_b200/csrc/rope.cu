// Rotary position embedding of a dense [B, H, seq_len, d] tensor: row r (of B*H*seq_len)
// has position r % seq_len and pair (2i, 2i+1) becomes (x0 c - x1 s, x0 s + x1 c) with
// c, s = cos/sin[pos][i] of fp32 tables [>= seq_len, d/2] -- the computation of the
// reference's fused_rope_kernel_fp32 (src/fused_rope.cu:13-45), here also for bf16 and
// fp16 (fp32 arithmetic, rounded to the element type). out may be in (in place).
// Vector path: one thread per 8 elements (4 pairs) with 128-bit loads of the element
// chunk and of the 4 cos / 4 sin entries; needs d % 8 == 0 and 16-byte aligned
// pointers. Otherwise one thread per pair.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <type_traits>

#include "internal.h"
#include "rope.h"

namespace fe {
namespace rope {

template <typename T>
__device__ __forceinline__ float ld_f(const T* p) {
  return static_cast<float>(*p);
}
template <typename T>
__device__ __forceinline__ T to_t(float x) {
  if constexpr (std::is_same<T, __nv_bfloat16>::value) return __float2bfloat16_rn(x);
  else if constexpr (std::is_same<T, half>::value) return __float2half_rn(x);
  else return x;
}

template <typename T>
__global__ void __launch_bounds__(256) rope_vec_kernel(const T* __restrict__ in,
                                                       const float* __restrict__ cs,
                                                       const float* __restrict__ sn,
                                                       T* __restrict__ out, long long rows,
                                                       int seq, int d) {
  const int cpr = d / 8;  // chunks of 8 elements per row
  const long long total = rows * cpr;
  for (long long c = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c < total;
       c += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = c / cpr;
    const int ch = static_cast<int>(c - row * cpr);
    const long long pos = row % seq;
    const float4 c4 = __ldg(reinterpret_cast<const float4*>(cs + pos * (d / 2) + ch * 4));
    const float4 s4 = __ldg(reinterpret_cast<const float4*>(sn + pos * (d / 2) + ch * 4));
    const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
    const T* src = in + row * d + ch * 8;
    T* dst = out + row * d + ch * 8;
    if constexpr (sizeof(T) == 4) {
      const float4 a = *reinterpret_cast<const float4*>(src);
      const float4 b = *reinterpret_cast<const float4*>(src + 4);
      const float x[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      float y[8];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        y[2 * k] = x[2 * k] * cc[k] - x[2 * k + 1] * ss[k];
        y[2 * k + 1] = x[2 * k] * ss[k] + x[2 * k + 1] * cc[k];
      }
      *reinterpret_cast<float4*>(dst) = make_float4(y[0], y[1], y[2], y[3]);
      *reinterpret_cast<float4*>(dst + 4) = make_float4(y[4], y[5], y[6], y[7]);
    } else {
      const uint4 v = *reinterpret_cast<const uint4*>(src);
      uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        // element 2k in the low half-word, 2k + 1 in the high one
        T lo, hi;
        const uint16_t ul = static_cast<uint16_t>(w[k] & 0xffffu), uh = static_cast<uint16_t>(w[k] >> 16);
        memcpy(&lo, &ul, 2);
        memcpy(&hi, &uh, 2);
        const float x0 = static_cast<float>(lo), x1 = static_cast<float>(hi);
        const T y0 = to_t<T>(x0 * cc[k] - x1 * ss[k]), y1 = to_t<T>(x0 * ss[k] + x1 * cc[k]);
        uint16_t b0, b1;
        memcpy(&b0, &y0, 2);
        memcpy(&b1, &y1, 2);
        w[k] = static_cast<uint32_t>(b0) | (static_cast<uint32_t>(b1) << 16);
      }
      *reinterpret_cast<uint4*>(dst) = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) rope_pair_kernel(const T* __restrict__ in,
                                                        const float* __restrict__ cs,
                                                        const float* __restrict__ sn,
                                                        T* __restrict__ out, long long rows,
                                                        int seq, int d) {
  const int half_d = d / 2;
  const long long total = rows * half_d;
  for (long long c = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; c < total;
       c += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long row = c / half_d;
    const int i = static_cast<int>(c - row * half_d);
    const long long pos = row % seq;
    const float cc = __ldg(cs + pos * half_d + i), ss = __ldg(sn + pos * half_d + i);
    const float x0 = ld_f(in + row * d + 2 * i), x1 = ld_f(in + row * d + 2 * i + 1);
    out[row * d + 2 * i] = to_t<T>(x0 * cc - x1 * ss);
    out[row * d + 2 * i + 1] = to_t<T>(x0 * ss + x1 * cc);
  }
}

template <typename T>
static cudaError_t launch_t(const void* in, const float* cs, const float* sn, void* out,
                            long long rows, int seq, int d, cudaStream_t st) {
  const bool vec = d % 8 == 0 &&
                   ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out) |
                     reinterpret_cast<uintptr_t>(cs) | reinterpret_cast<uintptr_t>(sn)) & 15) == 0;
  const long long work = rows * (vec ? d / 8 : d / 2);
  const int blocks = static_cast<int>(std::min<long long>((work + 255) / 256, 148LL * 16));
  if (vec)
    rope_vec_kernel<T><<<blocks, 256, 0, st>>>(static_cast<const T*>(in), cs, sn,
                                               static_cast<T*>(out), rows, seq, d);
  else
    rope_pair_kernel<T><<<blocks, 256, 0, st>>>(static_cast<const T*>(in), cs, sn,
                                                static_cast<T*>(out), rows, seq, d);
  return cudaGetLastError();
}

cudaError_t launch_rope(const void* in, const float* cs, const float* sn, void* out, int B,
                        int H, int seq, int d, int dtype, cudaStream_t st) {
  if (B < 0 || H < 0 || seq < 1 || d < 2 || d % 2 || !cs || !sn) return cudaErrorInvalidValue;
  const long long rows = static_cast<long long>(B) * H * seq;
  if (rows == 0) return cudaSuccess;
  if (dtype == 0) return launch_t<__nv_bfloat16>(in, cs, sn, out, rows, seq, d, st);
  if (dtype == 1) return launch_t<half>(in, cs, sn, out, rows, seq, d, st);
  if (dtype == 2) return launch_t<float>(in, cs, sn, out, rows, seq, d, st);
  return cudaErrorInvalidValue;
}

}  // namespace rope
}  // namespace fe
