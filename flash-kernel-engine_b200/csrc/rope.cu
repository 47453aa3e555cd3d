// Rotary position embedding of a dense [B, H, seq_len, d] tensor: row r (of B*H*seq_len)
// has position r % seq_len and pair (2i, 2i+1) becomes (x0 c - x1 s, x0 s + x1 c) with
// c, s = cos/sin[pos][i] of fp32 tables [>= seq_len, d/2] -- the computation of the
// reference's fused_rope_kernel_fp32 (src/fused_rope.cu:13-45), here also for bf16 and
// fp16 (fp32 arithmetic, rounded to the element type). out may be in (in place).
// Row path (bf16 / fp16, d / 8 a power of two up to 256, 16-byte aligned pointers): a
// 256-thread block covers 256 / (d / 8) rows per pass, one thread per 8 elements (4 pairs)
// with 128-bit loads of the element chunk and of its 4 cos / 4 sin entries, U rows a
// thread in flight; the position is stepped per pass instead of divided per chunk, and the
// grid is one resident wave. blockIdx.y selects the tensor, so Q and K are rotated by one
// launch. Vector path (fp32, or d % 8 == 0 otherwise): one thread per chunk (32 bytes of
// fp32, which amortise the index division: 94% of the copy rate against 82% through the
// row path), indices divided per chunk. Otherwise one thread per pair.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <initializer_list>
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

// One tensor of a row-path launch.
template <typename T>
struct RowJob {
  const T* in;
  T* out;
  long long rows;
  int seq;
};

// A chunk: 8 consecutive elements of a row (4 pairs), 16 bytes of bf16 / fp16 or 32 of fp32.
template <typename T>
struct Chunk {
  uint4 v;
};
template <>
struct Chunk<float> {
  float4 a, b;
};
template <typename T>
__device__ __forceinline__ Chunk<T> load_chunk(const T* p) {
  if constexpr (sizeof(T) == 4)
    return Chunk<T>{*reinterpret_cast<const float4*>(p), *reinterpret_cast<const float4*>(p + 4)};
  else
    return Chunk<T>{*reinterpret_cast<const uint4*>(p)};
}
template <typename T>
__device__ __forceinline__ void store_chunk(T* p, const Chunk<T>& c) {
  if constexpr (sizeof(T) == 4) {
    *reinterpret_cast<float4*>(p) = c.a;
    *reinterpret_cast<float4*>(p + 4) = c.b;
  } else {
    *reinterpret_cast<uint4*>(p) = c.v;
  }
}

// Rotates the 4 pairs of a chunk with their cos / sin entries (fp32 arithmetic, rounded
// to the element type).
template <typename T>
__device__ __forceinline__ Chunk<T> rotate_chunk(const Chunk<T>& x, float4 c4, float4 s4) {
  const float cc[4] = {c4.x, c4.y, c4.z, c4.w}, ss[4] = {s4.x, s4.y, s4.z, s4.w};
  if constexpr (sizeof(T) == 4) {
    const float e[8] = {x.a.x, x.a.y, x.a.z, x.a.w, x.b.x, x.b.y, x.b.z, x.b.w};
    float y[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      y[2 * k] = e[2 * k] * cc[k] - e[2 * k + 1] * ss[k];
      y[2 * k + 1] = e[2 * k] * ss[k] + e[2 * k + 1] * cc[k];
    }
    return Chunk<T>{make_float4(y[0], y[1], y[2], y[3]), make_float4(y[4], y[5], y[6], y[7])};
  } else {
    uint32_t w[4] = {x.v.x, x.v.y, x.v.z, x.v.w};
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
    return Chunk<T>{make_uint4(w[0], w[1], w[2], w[3])};
  }
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
    store_chunk<T>(out + row * d + ch * 8, rotate_chunk<T>(load_chunk<T>(in + row * d + ch * 8), c4, s4));
  }
}

// Row path. lg_cpr = log2(d / 8).
template <typename T, int U>
__global__ void __launch_bounds__(256) rope_row_kernel(RowJob<T> j0, RowJob<T> j1,
                                                       const float* __restrict__ cs,
                                                       const float* __restrict__ sn, int d,
                                                       int lg_cpr) {
  const RowJob<T> j = blockIdx.y == 0 ? j0 : j1;
  const int rpb = 256 >> lg_cpr;                    // rows a block covers per pass
  const int ch = threadIdx.x & ((1 << lg_cpr) - 1);  // 8-element chunk of the row
  long long row = static_cast<long long>(blockIdx.x) * rpb + (threadIdx.x >> lg_cpr);
  const long long step = static_cast<long long>(gridDim.x) * rpb;
  if (row >= j.rows) return;
  int pos = static_cast<int>(row % j.seq);
  const int pstep = static_cast<int>(step % j.seq);
  const int half_d = d >> 1;
  for (; row < j.rows; row += U * step) {
    Chunk<T> x[U];
    float4 c4[U], s4[U];
    int pu = pos;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (u > 0) {
        pu += pstep;
        if (pu >= j.seq) pu -= j.seq;
      }
      if (row + u * step < j.rows) {
        x[u] = load_chunk<T>(j.in + (row + u * step) * d + ch * 8);
        c4[u] = __ldg(reinterpret_cast<const float4*>(cs + static_cast<size_t>(pu) * half_d + ch * 4));
        s4[u] = __ldg(reinterpret_cast<const float4*>(sn + static_cast<size_t>(pu) * half_d + ch * 4));
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (row + u * step < j.rows)
        store_chunk<T>(j.out + (row + u * step) * d + ch * 8, rotate_chunk<T>(x[u], c4[u], s4[u]));
    }
    pu += pstep;  // the position of row + U * step
    if (pu >= j.seq) pu -= j.seq;
    pos = pu;
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

// rows a thread has in flight (config 2's K: 46.4 µs with 1 or 2, 47.9 µs with 4)
constexpr int kRowUnroll = 2;

// log2(d / 8) when the row path applies to these pointers, else -1.
static int row_path_lg(int d, std::initializer_list<const void*> ptrs) {
  if (d % 8) return -1;
  uintptr_t a = 0;
  for (const void* q : ptrs) a |= reinterpret_cast<uintptr_t>(q);
  if (a & 15) return -1;
  const int cpr = d / 8;
  if (cpr > 256 || (cpr & (cpr - 1))) return -1;
  int lg = 0;
  while ((1 << lg) < cpr) ++lg;
  return lg;
}

// Blocks a row-path tensor gets: its rows in passes of U rows a thread, at most its share
// of one resident wave.
template <typename T>
static int row_blocks(long long rows, int lg, int tensors) {
  static int occ = 0;
  if (!occ) {
    int o = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, rope_row_kernel<T, kRowUnroll>, 256, 0) !=
            cudaSuccess || o < 1)
      o = 1;
    occ = o;
  }
  const long long need = (rows + (256 >> lg) - 1) / (256 >> lg);
  const long long wave = std::max<long long>(1, static_cast<long long>(sm_count()) * occ / tensors);
  return static_cast<int>(std::max<long long>(1, std::min(need, wave)));
}

template <typename T>
static cudaError_t launch_t(const void* in, const float* cs, const float* sn, void* out,
                            long long rows, int seq, int d, cudaStream_t st) {
  if constexpr (sizeof(T) == 2) {
    const int lg = row_path_lg(d, {in, out, cs, sn});
    if (lg >= 0) {
      const RowJob<T> j{static_cast<const T*>(in), static_cast<T*>(out), rows, seq};
      rope_row_kernel<T, kRowUnroll><<<dim3(row_blocks<T>(rows, lg, 1), 1), 256, 0, st>>>(
          j, j, cs, sn, d, lg);
      return cudaGetLastError();
    }
  }
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

static bool rope_args_ok(int B, int H, int seq, int d, const float* cs, const float* sn) {
  return B >= 0 && H >= 0 && seq >= 1 && d >= 2 && d % 2 == 0 && cs && sn;
}

cudaError_t launch_rope(const void* in, const float* cs, const float* sn, void* out, int B,
                        int H, int seq, int d, int dtype, cudaStream_t st) {
  if (!rope_args_ok(B, H, seq, d, cs, sn)) return cudaErrorInvalidValue;
  const long long rows = static_cast<long long>(B) * H * seq;
  if (rows == 0) return cudaSuccess;
  if (dtype == 0) return launch_t<__nv_bfloat16>(in, cs, sn, out, rows, seq, d, st);
  if (dtype == 1) return launch_t<half>(in, cs, sn, out, rows, seq, d, st);
  if (dtype == 2) return launch_t<float>(in, cs, sn, out, rows, seq, d, st);
  return cudaErrorInvalidValue;
}

template <typename T>
static cudaError_t launch_qk_t(const void* q, const void* k, const float* cs, const float* sn,
                               void* q_out, void* k_out, int B, int H, int N, int M, int d,
                               cudaStream_t st) {
  const long long rq = static_cast<long long>(B) * H * N, rk = static_cast<long long>(B) * H * M;
  if constexpr (sizeof(T) == 2) {
    const int lg = row_path_lg(d, {q, k, q_out, k_out, cs, sn});
    if (lg >= 0) {
      const RowJob<T> jq{static_cast<const T*>(q), static_cast<T*>(q_out), rq, N};
      const RowJob<T> jk{static_cast<const T*>(k), static_cast<T*>(k_out), rk, M};
      const int blocks = std::max(row_blocks<T>(rq, lg, 2), row_blocks<T>(rk, lg, 2));
      rope_row_kernel<T, kRowUnroll><<<dim3(blocks, 2), 256, 0, st>>>(jq, jk, cs, sn, d, lg);
      return cudaGetLastError();
    }
  }
  cudaError_t e = launch_t<T>(q, cs, sn, q_out, rq, N, d, st);
  if (e == cudaSuccess) e = launch_t<T>(k, cs, sn, k_out, rk, M, d, st);
  return e;
}

cudaError_t launch_rope_qk(const void* q, const void* k, const float* cs, const float* sn,
                           void* q_out, void* k_out, int B, int H, int N, int M, int d, int dtype,
                           cudaStream_t st) {
  if (!rope_args_ok(B, H, N, d, cs, sn) || M < 1) return cudaErrorInvalidValue;
  if (static_cast<long long>(B) * H == 0) return cudaSuccess;
  if (dtype == 0) return launch_qk_t<__nv_bfloat16>(q, k, cs, sn, q_out, k_out, B, H, N, M, d, st);
  if (dtype == 1) return launch_qk_t<half>(q, k, cs, sn, q_out, k_out, B, H, N, M, d, st);
  if (dtype == 2) return launch_qk_t<float>(q, k, cs, sn, q_out, k_out, B, H, N, M, d, st);
  return cudaErrorInvalidValue;
}

}  // namespace rope
}  // namespace fe
