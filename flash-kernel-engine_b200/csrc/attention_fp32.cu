// fp32 (CUDA-core) kernels behind the reference's fp32 entry points:
//  * FA2 forward          (launch_flash_attention_forward_fp32, src/flash_attention.cu:111-345)
//  * naive forward        (launch_naive_attention_forward_fp32, src/flash_attention.cu:12-104)
//  * paged decode, GQA    (launch_paged_attention_v1_fp32, src/paged_attention.cu:14-215)
//  * dense split-KV stage 1 (launch_flash_decoding_forward_fp32, src/flash_decoding.cu:14-142)
// fp32 inputs need fp32 products to hold the 1e-3 relative tolerance, so these run
// on the FMA pipes; the bf16/fp16 paths use tensor cores.
//
// All softmax arithmetic is done in the log2 domain: s2 = (q.k) * scale * log2(e),
// p = 2^(s2 - m2); this is the same softmax as exp(s - m) (2^(x log2 e) = e^x).
#include <limits.h>

#include "fp32_kernels.h"
#include "internal.h"
#include "ptx.cuh"

namespace fe {
namespace simt {

constexpr float NEG_INF = -__builtin_huge_valf();

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Asynchronous 4-byte global -> shared copies (cp.async), completed per group.
__device__ __forceinline__ void cp_async4(float* dst, const float* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// =========================================================================
// FA2 forward, fp32. CTA = 64 query rows of one (b, h); 8 warps x 8 rows. The K/V
// tiles are double-buffered: tile t+1 is copied in (cp.async) while tile t is used.
// Per 64-key tile: lane j scores keys j and j+32 for its warp's 8 rows, the warp
// does the online-softmax update per row, then every lane accumulates P V for
// its D/32 output columns. D is the padded head dim (multiple of 32).
template <int D>
__global__ void __launch_bounds__(256) fa2_fp32_kernel(const float* __restrict__ Q,
                                                       const float* __restrict__ K,
                                                       const float* __restrict__ V,
                                                       float* __restrict__ O, int N, int M, int d,
                                                       float sl, int causal) {
  constexpr int BM = 64, BN = 64, KS = D + 1, E = D / 32;
  extern __shared__ float sm[];
  float* sQ = sm;                 // [BM][KS]
  float* sKb = sQ + BM * KS;      // [2][BN][KS]
  float* sVb = sKb + 2 * BN * KS; // [2][BN][D]
  float* sP = sVb + 2 * BN * D;   // [8 warps][8 rows][BN]
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const size_t bh = blockIdx.y;
  const int r0 = blockIdx.x * BM;
  const float* Qb = Q + bh * N * d;
  const float* Kb = K + bh * M * d;
  const float* Vb = V + bh * M * d;

  for (int i = tid; i < BM * D; i += 256) {
    const int r = i / D, c = i - r * D;
    sQ[r * KS + c] = (r0 + r < N && c < d) ? Qb[static_cast<size_t>(r0 + r) * d + c] : 0.f;
  }
  float m[8], l[8], acc[8][E];
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    m[r] = NEG_INF;
    l[r] = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) acc[r][e] = 0.f;
  }
  int ntiles = (M + BN - 1) / BN;
  if (causal) ntiles = min(ntiles, (r0 + BM + BN - 1) / BN);
  float* myP = sP + warp * 8 * BN;
  // copies of key tile t into buffer t & 1 (rows past M are zeroed)
  auto issue_tile = [&](int t) {
    const int c0 = t * BN;
    float* sK = sKb + (t & 1) * BN * KS;
    float* sV = sVb + (t & 1) * BN * D;
    for (int i = tid; i < BN * D; i += 256) {
      const int r = i / D, c = i - r * D;
      if (c0 + r < M && c < d) {
        const size_t gi = static_cast<size_t>(c0 + r) * d + c;
        cp_async4(sK + r * KS + c, Kb + gi);
        cp_async4(sV + r * D + c, Vb + gi);
      } else {
        sK[r * KS + c] = 0.f;
        sV[r * D + c] = 0.f;
      }
    }
    cp_async_commit();
  };
  if (ntiles > 0) issue_tile(0);
  for (int t = 0; t < ntiles; ++t) {
    const int c0 = t * BN;
    const float* sK = sKb + (t & 1) * BN * KS;
    const float* sV = sVb + (t & 1) * BN * D;
    // the buffer of tile t+1 was last read in iteration t-1, which ended in a barrier
    if (t + 1 < ntiles) {
      issue_tile(t + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    float s[8][2];
#pragma unroll
    for (int r = 0; r < 8; ++r) s[r][0] = s[r][1] = 0.f;
    const float* k0 = sK + lane * KS;
    const float* k1 = sK + (lane + 32) * KS;
    const float* qw = sQ + warp * 8 * KS;
#pragma unroll 4
    for (int c = 0; c < D; ++c) {
      const float a0 = k0[c], a1 = k1[c];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float qv = qw[r * KS + c];
        s[r][0] = fmaf(qv, a0, s[r][0]);
        s[r][1] = fmaf(qv, a1, s[r][1]);
      }
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int row = r0 + warp * 8 + r;
#pragma unroll
      for (int jj = 0; jj < 2; ++jj) {
        const int col = c0 + lane + 32 * jj;
        const bool valid = col < M && (!causal || col <= row);
        s[r][jj] = valid ? s[r][jj] * sl : NEG_INF;
      }
      const float tmax = warp_max(fmaxf(s[r][0], s[r][1]));
      const float mn = fmaxf(m[r], tmax);
      const float mu = mn == NEG_INF ? 0.f : mn;
      const float corr = ex2(m[r] - mu);
      m[r] = mn;
      const float p0 = ex2(s[r][0] - mu), p1 = ex2(s[r][1] - mu);
      l[r] = l[r] * corr + p0 + p1;  // per-lane partial; reduced at the end
#pragma unroll
      for (int e = 0; e < E; ++e) acc[r][e] *= corr;
      myP[r * BN + lane] = p0;
      myP[r * BN + lane + 32] = p1;
    }
    __syncwarp();
#pragma unroll 2
    for (int j = 0; j < BN; ++j) {
      float vv[E];
#pragma unroll
      for (int e = 0; e < E; ++e) vv[e] = sV[j * D + lane + 32 * e];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const float pr = myP[r * BN + j];
#pragma unroll
        for (int e = 0; e < E; ++e) acc[r][e] = fmaf(pr, vv[e], acc[r][e]);
      }
    }
    __syncthreads();  // every warp is done with this buffer before it is refilled
  }
#pragma unroll
  for (int r = 0; r < 8; ++r) {
    const int row = r0 + warp * 8 + r;
    const float L = warp_sum(l[r]);
    if (row >= N) continue;
    const float inv = L > 0.f ? 1.f / L : 0.f;
    float* orow = O + bh * N * d + static_cast<size_t>(row) * d;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int c = lane + 32 * e;
      if (c < d) orow[c] = acc[r][e] * inv;
    }
  }
}

template <int D>
static cudaError_t launch_fa2_fp32_d(const float* q, const float* k, const float* v, float* o,
                                     int B, int H, int N, int M, int d, float sl, int causal,
                                     cudaStream_t st) {
  const int smem = (64 * (D + 1) * 3 + 2 * 64 * D + 8 * 8 * 64) * 4;
  cudaError_t e = ensure_smem_optin(reinterpret_cast<const void*>(fa2_fp32_kernel<D>), smem);
  if (e != cudaSuccess) return e;
  dim3 grid((N + 63) / 64, B * H);
  fa2_fp32_kernel<D><<<grid, 256, smem, st>>>(q, k, v, o, N, M, d, sl, causal);
  return cudaGetLastError();
}

cudaError_t launch_fa2_fp32(const float* q, const float* k, const float* v, float* o, int B, int H,
                            int N, int M, int d, float scale, int causal, cudaStream_t st) {
  const float sl = scale * kLog2e;
  if (d <= 32) return launch_fa2_fp32_d<32>(q, k, v, o, B, H, N, M, d, sl, causal, st);
  if (d <= 64) return launch_fa2_fp32_d<64>(q, k, v, o, B, H, N, M, d, sl, causal, st);
  if (d <= 128) return launch_fa2_fp32_d<128>(q, k, v, o, B, H, N, M, d, sl, causal, st);
  return cudaErrorInvalidValue;
}

// =========================================================================
// Naive attention: one thread per query row, online softmax over all M keys
// (the reference's kernel reads N keys instead of M, src/flash_attention.cu:28-31,50;
// this one uses M). Accumulator in local memory, like the reference (d <= 256).
__global__ void __launch_bounds__(128) naive_fp32_kernel(const float* __restrict__ Q,
                                                         const float* __restrict__ K,
                                                         const float* __restrict__ V,
                                                         float* __restrict__ O, int N, int M, int d,
                                                         float sl, int causal) {
  const size_t bh = blockIdx.z;
  const int row = blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= N) return;
  const float* q = Q + (bh * N + row) * d;
  const float* Kb = K + bh * M * d;
  const float* Vb = V + bh * M * d;
  float acc[256];
  for (int c = 0; c < d; ++c) acc[c] = 0.f;
  float m = NEG_INF, l = 0.f;
  const int kend = causal ? min(M, row + 1) : M;
  for (int j = 0; j < kend; ++j) {
    float s = 0.f;
    for (int c = 0; c < d; ++c) s = fmaf(q[c], Kb[static_cast<size_t>(j) * d + c], s);
    s *= sl;
    const float mn = fmaxf(m, s);
    const float corr = ex2(m - mn), p = ex2(s - mn);
    l = l * corr + p;
    for (int c = 0; c < d; ++c) acc[c] = fmaf(p, Vb[static_cast<size_t>(j) * d + c], acc[c] * corr);
    m = mn;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
  float* o = O + (bh * N + row) * d;
  for (int c = 0; c < d; ++c) o[c] = acc[c] * inv;
}

cudaError_t launch_naive_fp32(const float* q, const float* k, const float* v, float* o, int B,
                              int H, int N, int M, int d, float scale, int causal,
                              cudaStream_t st) {
  if (d < 1 || d > 256) return cudaErrorInvalidValue;
  dim3 grid((N + 127) / 128, 1, B * H);
  naive_fp32_kernel<<<grid, 128, 0, st>>>(q, k, v, o, N, M, d, scale * kLog2e, causal);
  return cudaGetLastError();
}

// =========================================================================
// Warp-per-token decode core shared by the paged and dense fp32 decoders.
// CTA = 4 warps working on up to HG query heads that read the same KV head.
// Each warp takes tokens round-robin; lanes own D/32 dims; per token and head the
// warp reduces the dot product with shuffles and updates its own (m, l, acc);
// the four warp states are merged through shared memory at the end.
template <int D, int HG>
struct WarpDecode {
  static constexpr int E = D / 32;
  float m[HG], l[HG], acc[HG][E];
  __device__ __forceinline__ void init() {
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      m[h] = NEG_INF;
      l[h] = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[h][e] = 0.f;
    }
  }
  // q: [HG][D] in shared memory (zero padded); k, v: token rows (d valid floats).
  __device__ __forceinline__ void token(const float* q, const float* k, const float* v, int d,
                                        int nh, float sl, int lane) {
    float kv[E], vv[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int c = lane + 32 * e;
      kv[e] = c < d ? __ldg(k + c) : 0.f;
      vv[e] = c < d ? __ldg(v + c) : 0.f;
    }
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      if (h >= nh) break;
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) s = fmaf(q[h * D + lane + 32 * e], kv[e], s);
      s = warp_sum(s) * sl;
      const float mn = fmaxf(m[h], s);
      const float corr = ex2(m[h] - mn), p = ex2(s - mn);
      l[h] = l[h] * corr + p;
#pragma unroll
      for (int e = 0; e < E; ++e) acc[h][e] = fmaf(p, vv[e], acc[h][e] * corr);
      m[h] = mn;
    }
  }
  // Merge 4 warp states through smem (cm/cl: [4][HG], co: [4][HG][D]); returns the
  // merged (M, L, O) for (h, c) pairs handled by the calling thread via `emit`.
  template <typename Emit>
  __device__ __forceinline__ void merge(float* cm, float* cl, float* co, int nh, int d, int warp,
                                        int lane, Emit emit) {
    if (lane == 0) {
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        cm[warp * HG + h] = m[h];
        cl[warp * HG + h] = l[h];
      }
    }
#pragma unroll
    for (int h = 0; h < HG; ++h)
#pragma unroll
      for (int e = 0; e < E; ++e) co[(warp * HG + h) * D + lane + 32 * e] = acc[h][e];
    __syncthreads();
    for (int i = threadIdx.x; i < nh * D; i += blockDim.x) {
      const int h = i / D, c = i - h * D;
      if (c >= d) continue;
      float Mx = NEG_INF;
      for (int w = 0; w < 4; ++w) Mx = fmaxf(Mx, cm[w * HG + h]);
      float L = 0.f, Ov = 0.f;
      for (int w = 0; w < 4; ++w) {
        const float mw = cm[w * HG + h];
        const float wt = mw == NEG_INF ? 0.f : ex2(mw - Mx);
        L += cl[w * HG + h] * wt;
        Ov += co[(w * HG + h) * D + c] * wt;
      }
      emit(h, c, Mx, L, Ov);
    }
  }
};

// Paged fp32 decode: grid (Hkv * head_chunks, S); the chunk's query heads share
// every K/V row read.
template <int D, int HG>
__global__ void __launch_bounds__(128) paged_fp32_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    float* __restrict__ out, const int* __restrict__ bt, const int* __restrict__ lens, int H,
    int Hkv, int d, int bs, int maxb, int num_blocks, float sl, unsigned* err) {
  __shared__ float sq[HG * D];
  __shared__ float cm[4 * HG], cl[4 * HG];
  __shared__ float co[4 * HG * D];
  const int G = H / Hkv, chunks = (G + HG - 1) / HG;
  const int kvh = blockIdx.x / chunks, ch = blockIdx.x - kvh * chunks;
  const int seq = blockIdx.y;
  const int h0 = kvh * G + ch * HG;
  const int nh = min(HG, G - ch * HG);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < HG * D; i += 128) {
    const int h = i / D, c = i - h * D;
    sq[i] = (h < nh && c < d) ? q[(static_cast<size_t>(seq) * H + h0 + h) * d + c] : 0.f;
  }
  __syncthreads();
  const int ctx = lens[seq];
  WarpDecode<D, HG> st;
  st.init();
  for (int t = warp; t < ctx; t += 4) {
    const int phys = __ldg(bt + static_cast<size_t>(seq) * maxb + t / bs);
    if (phys < 0 || (num_blocks > 0 && phys >= num_blocks)) {
      if (lane == 0) atomicOr(err, kErrBadBlock);
      continue;
    }
    const size_t off = ((static_cast<size_t>(phys) * Hkv + kvh) * bs + t % bs) * d;
    st.token(sq, kc + off, vc + off, d, nh, sl, lane);
  }
  st.merge(cm, cl, co, nh, d, warp, lane, [&](int h, int c, float, float L, float Ov) {
    out[(static_cast<size_t>(seq) * H + h0 + h) * d + c] = L > 0.f ? Ov / L : 0.f;
  });
}

cudaError_t launch_paged_fp32(const float* q, const float* kc, const float* vc, float* out,
                              const int* bt, const int* lens, int S, int H, int Hkv, int d, int bs,
                              int maxb, int num_blocks, float scale, cudaStream_t st) {
  if (S <= 0) return cudaSuccess;
  const int G = H / Hkv;
  const int HG = G >= 8 ? 8 : G >= 4 ? 4 : G >= 2 ? 2 : 1;
  const int chunks = (G + HG - 1) / HG;
  dim3 grid(Hkv * chunks, S);
  const float sl = scale * kLog2e;
  unsigned* err = device_error_word();
#define FE_P(D_, HG_)                                                                      \
  if (d <= D_ && HG == HG_) {                                                              \
    paged_fp32_kernel<D_, HG_><<<grid, 128, 0, st>>>(q, kc, vc, out, bt, lens, H, Hkv, d, bs, \
                                                     maxb, num_blocks, sl, err);           \
    return cudaGetLastError();                                                             \
  }
  FE_P(64, 1) FE_P(64, 2) FE_P(64, 4) FE_P(64, 8)
  FE_P(128, 1) FE_P(128, 2) FE_P(128, 4) FE_P(128, 8)
  FE_P(256, 1) FE_P(256, 2) FE_P(256, 4)
#undef FE_P
  return cudaErrorInvalidValue;
}

// Dense split-KV stage 1 (fp32): grid (splits, B*H). Writes the unnormalised O,
// m (log2 units) and l of split s of row bh; an empty split writes (-inf, 0).
template <int D>
__global__ void __launch_bounds__(128) decode_split_fp32_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    float* __restrict__ part_o, float* __restrict__ part_ml, int M, int d, int splits, float sl) {
  __shared__ float sq[D];
  __shared__ float cm[4], cl[4];
  __shared__ float co[4 * D];
  const int s = blockIdx.x;
  const size_t bh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = (M + splits - 1) / splits;
  const int t0 = s * per, t1 = min(M, t0 + per);
  for (int c = threadIdx.x; c < D; c += 128) sq[c] = c < d ? q[bh * d + c] : 0.f;
  __syncthreads();
  WarpDecode<D, 1> st;
  st.init();
  for (int t = t0 + warp; t < t1; t += 4) {
    const size_t off = (bh * M + t) * d;
    st.token(sq, k + off, v + off, d, 1, sl, lane);
  }
  const size_t slot = bh * splits + s;
  st.merge(cm, cl, co, 1, d, warp, lane, [&](int, int c, float Mx, float L, float Ov) {
    part_o[slot * d + c] = Ov;
    if (c == 0) {
      part_ml[slot * 2] = Mx;
      part_ml[slot * 2 + 1] = L;
    }
  });
}

cudaError_t launch_decode_split_fp32(const float* q, const float* k, const float* v,
                                     float* part_o, float* part_ml, int BH, int M, int d,
                                     int splits, float scale, cudaStream_t st) {
  if (BH <= 0) return cudaSuccess;
  dim3 grid(splits, BH);
  const float sl = scale * kLog2e;
  if (d <= 64)
    decode_split_fp32_kernel<64><<<grid, 128, 0, st>>>(q, k, v, part_o, part_ml, M, d, splits, sl);
  else if (d <= 128)
    decode_split_fp32_kernel<128><<<grid, 128, 0, st>>>(q, k, v, part_o, part_ml, M, d, splits, sl);
  else if (d <= 256)
    decode_split_fp32_kernel<256><<<grid, 128, 0, st>>>(q, k, v, part_o, part_ml, M, d, splits, sl);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace simt
}  // namespace fe
