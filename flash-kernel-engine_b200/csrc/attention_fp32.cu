// fp32 (CUDA-core) kernels behind the reference's fp32 entry points:
//  * FA2 forward          (launch_flash_attention_forward_fp32, src/flash_attention.cu:111-345)
//  * naive forward        (launch_naive_attention_forward_fp32, src/flash_attention.cu:12-104)
//  * paged decode, GQA, single pass, for the shapes the persistent decode of
//    paged_decode.cu does not take (launch_paged_attention_v1_fp32,
//    src/paged_attention.cu:14-215)
//  * dense split-KV stage 1 (launch_flash_decoding_forward_fp32, src/flash_decoding.cu:14-142)
// fp32 inputs need fp32 products to hold the 1e-3 relative tolerance, so these run
// on the FMA pipes; the bf16/fp16 paths use tensor cores.
//
// All softmax arithmetic is done in the log2 domain: s2 = (q.k) * scale * log2(e),
// p = 2^(s2 - m2); this is the same softmax as exp(s - m) (2^(x log2 e) = e^x).
#include <limits.h>
#include <stdlib.h>

#include <type_traits>

#include "../../include/cuda_utils.cuh"
#include "fp32_kernels.h"
#include "internal.h"
#include "ptx.cuh"

namespace fe {
namespace simt {

constexpr float NEG_INF = -__builtin_huge_valf();

// Butterfly warp reductions of include/cuda_utils.cuh (result in every lane).
using flash_engine::cuda::warp_reduce_max;
using flash_engine::cuda::warp_reduce_sum;
__device__ __forceinline__ float warp_sum(float v) { return warp_reduce_sum(v); }
__device__ __forceinline__ float warp_max(float v) { return warp_reduce_max(v); }

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
// FA2 forward, fp32. A CTA owns 64 query rows of one (b, h) and a share of their key
// tiles; the `nsplit` CTAs of one row tile form a thread-block cluster and take the
// 64-key tiles t = split, split + nsplit, ... of the row tile. Eight warps each own 8
// rows. Lane (tr = lane / 16, tc = lane % 16) of warp w scores rows w*8 + tr*4 + i
// (i < 4) against keys tc + 16 j (j < 4) of the tile: per 4 head dims it loads four
// 128-bit Q words and four 128-bit K words from shared memory and issues 64 FMAs.
// The softmax row max and sum reduce over the 16 lanes of the row group with shuffles.
// P goes to shared memory transposed ([key][row]), so that the P V product reads one
// 128-bit word of P (4 rows) and D/64 128-bit words of V (4 head dims each) for 4 D/16
// FMAs. K/V tiles are double-buffered with cp.async.
// With nsplit > 1 the CTAs of the cluster exchange (m, l, O) partials through
// distributed shared memory: CTA c merges rows [c*64/nsplit, (c+1)*64/nsplit) of every
// partner (the log-sum-exp combine of src/flash_decoding.cu:151-223) and writes them.
constexpr int kFaBM = 64, kFaBN = 64;

template <int D>
struct FaSmem {
  static constexpr int QS = D + 4;          // row stride of Q and K tiles (floats)
  static constexpr int PS = kFaBM + 4;      // row stride of the transposed P tile
  static constexpr int kQ = kFaBM * QS;
  static constexpr int kK = kFaBN * QS;
  static constexpr int kV = kFaBN * D;
  static constexpr int kP = kFaBN * PS;
  static constexpr int floats = kQ + 2 * kK + 2 * kV + kP;
  static constexpr int bytes = floats * 4;
  // the cluster combine reuses the K buffers: O [64][D], then m [64], l [64]
  static_assert(kFaBM * D + 2 * kFaBM <= 2 * kK, "combine buffer does not fit");
};

__device__ __forceinline__ void cp_async16(float* dst, const float* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared-memory offset in CTA `rank` of this cluster.
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_v2(uint32_t addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b)
               : "memory");
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b),
               "f"(c), "f"(d)
               : "memory");
}
// Every thread of every CTA of the cluster arrives; shared-memory writes before it
// (local and remote) are visible to the whole cluster after it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Copies rows [r_begin, r_begin + 64) of a [rows, d] fp32 matrix into a [64][stride]
// shared tile (columns up to D); rows past `rows` and columns past d read as zeros.
template <int D>
__device__ __forceinline__ void fa_load_tile(float* dst, int stride, const float* src, int r_begin,
                                             int rows, int d, bool vec, int tid) {
  if (vec) {
    constexpr int C4 = D / 4;
    for (int i = tid; i < kFaBN * C4; i += 256) {
      const int r = i / C4, c = (i - r * C4) * 4;
      float* s = dst + r * stride + c;
      if (r_begin + r < rows && c < d)
        cp_async16(s, src + static_cast<size_t>(r_begin + r) * d + c);
      else
        *reinterpret_cast<float4*>(s) = make_float4(0.f, 0.f, 0.f, 0.f);
    }
  } else {
    for (int i = tid; i < kFaBN * D; i += 256) {
      const int r = i / D, c = i - r * D;
      float* s = dst + r * stride + c;
      if (r_begin + r < rows && c < d)
        cp_async4(s, src + static_cast<size_t>(r_begin + r) * d + c);
      else
        *s = 0.f;
    }
  }
}

template <int D>
__global__ void __launch_bounds__(256, D <= 64 ? 2 : 1)
    fa2_fp32_kernel(const float* __restrict__ Q, const float* __restrict__ K,
                    const float* __restrict__ V, float* __restrict__ O, int N, int M, int d,
                    float sl, int causal, int nsplit, int vec) {
  using L = FaSmem<D>;
  constexpr int QS = L::QS, PS = L::PS;
  constexpr int G = D >= 64 ? 4 : 2;   // consecutive head dims a lane owns per group
  constexpr int NG = D / (16 * G);     // groups: head dims e*16*G + tc*G + [0, G)
  constexpr int CW = NG * G;           // head dims per lane = D / 16
  extern __shared__ __align__(16) float sm[];
  float* sQ = sm;
  float* sKb = sQ + L::kQ;
  float* sVb = sKb + 2 * L::kK;
  float* sPT = sVb + 2 * L::kV;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tr = lane >> 4, tc = lane & 15;
  const int rb = warp * 8 + tr * 4;   // first of this lane's 4 rows within the tile
  const size_t bh = blockIdx.y;
  const int split = nsplit > 1 ? static_cast<int>(cluster_rank()) : 0;
  const int r0 = (blockIdx.x / nsplit) * kFaBM;
  const float* Qb = Q + bh * N * d;
  const float* Kb = K + bh * M * d;
  const float* Vb = V + bh * M * d;

  int ntiles = (M + kFaBN - 1) / kFaBN;
  if (causal) ntiles = min(ntiles, (r0 + kFaBM + kFaBN - 1) / kFaBN);
  const int nloc = ntiles > split ? (ntiles - split + nsplit - 1) / nsplit : 0;

  fa_load_tile<D>(sQ, QS, Qb, r0, N, d, vec, tid);
  auto issue_tile = [&](int it) {
    const int c0 = (split + it * nsplit) * kFaBN;
    fa_load_tile<D>(sKb + (it & 1) * L::kK, QS, Kb, c0, M, d, vec, tid);
    fa_load_tile<D>(sVb + (it & 1) * L::kV, D, Vb, c0, M, d, vec, tid);
    cp_async_commit();
  };
  if (nloc > 0) issue_tile(0);
  else cp_async_commit();

  float m[4], l[4], acc[4][CW];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = NEG_INF;
    l[i] = 0.f;
#pragma unroll
    for (int c = 0; c < CW; ++c) acc[i][c] = 0.f;
  }

  for (int it = 0; it < nloc; ++it) {
    const int c0 = (split + it * nsplit) * kFaBN;
    const float* sK = sKb + (it & 1) * L::kK;
    const float* sV = sVb + (it & 1) * L::kV;
    // the buffer of tile it+1 was last read in iteration it-1, which ended in a barrier
    if (it + 1 < nloc) {
      issue_tile(it + 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    float s[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] = 0.f;
    const float* qrow = sQ + rb * QS;
    const float* krow = sK + tc * QS;
#pragma unroll 4
    for (int k = 0; k < D; k += 4) {
      float4 qv[4], kv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) qv[i] = *reinterpret_cast<const float4*>(qrow + i * QS + k);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        kv[j] = *reinterpret_cast<const float4*>(krow + j * 16 * QS + k);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s[i][j] = fmaf(qv[i].x, kv[j].x, s[i][j]);
          s[i][j] = fmaf(qv[i].y, kv[j].y, s[i][j]);
          s[i][j] = fmaf(qv[i].z, kv[j].z, s[i][j]);
          s[i][j] = fmaf(qv[i].w, kv[j].w, s[i][j]);
        }
    }

    // online softmax per row over the 16 lanes of the row group
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = r0 + rb + i;
      float tmax = NEG_INF;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = c0 + tc + 16 * j;
        const bool valid = col < M && (!causal || col <= row);
        s[i][j] = valid ? s[i][j] * sl : NEG_INF;
        tmax = fmaxf(tmax, s[i][j]);
      }
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float mn = fmaxf(m[i], tmax);
      const float mu = mn == NEG_INF ? 0.f : mn;
      const float corr = ex2(m[i] - mu);
      m[i] = mn;
      float ps = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[i][j] = ex2(s[i][j] - mu);
        ps += s[i][j];
      }
      l[i] = l[i] * corr + ps;   // this lane's share; reduced over the row group at the end
#pragma unroll
      for (int c = 0; c < CW; ++c) acc[i][c] *= corr;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      *reinterpret_cast<float4*>(sPT + (tc + 16 * j) * PS + rb) =
          make_float4(s[0][j], s[1][j], s[2][j], s[3][j]);
    __syncwarp();   // the warp reads back only its own 8 rows of P

#pragma unroll 4
    for (int j = 0; j < kFaBN; ++j) {
      const float4 p = *reinterpret_cast<const float4*>(sPT + j * PS + rb);
      const float pr[4] = {p.x, p.y, p.z, p.w};
      float vv[CW];
#pragma unroll
      for (int e = 0; e < NG; ++e) {
        const float* vp = sV + j * D + e * 16 * G + tc * G;
        if constexpr (G == 4) {
          const float4 t = *reinterpret_cast<const float4*>(vp);
          vv[e * 4 + 0] = t.x;
          vv[e * 4 + 1] = t.y;
          vv[e * 4 + 2] = t.z;
          vv[e * 4 + 3] = t.w;
        } else {
          const float2 t = *reinterpret_cast<const float2*>(vp);
          vv[e * 2 + 0] = t.x;
          vv[e * 2 + 1] = t.y;
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < CW; ++c) acc[i][c] = fmaf(pr[i], vv[c], acc[i][c]);
    }
    __syncthreads();   // every warp is done with this K/V buffer before it is refilled
  }
  cp_async_wait<0>();

#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) l[i] += __shfl_xor_sync(0xffffffffu, l[i], o);

  float* Ob = O + bh * N * d;
  if (nsplit == 1) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int row = r0 + rb + i;
      if (row >= N) continue;
      const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
      float* orow = Ob + static_cast<size_t>(row) * d;
#pragma unroll
      for (int e = 0; e < NG; ++e)
#pragma unroll
        for (int g = 0; g < G; ++g) {
          const int c = e * 16 * G + tc * G + g;
          if (c < d) orow[c] = acc[i][e * G + g] * inv;
        }
    }
    return;
  }

  // ---- cluster combine. Rows of slice c = [c*SR, (c+1)*SR) go to CTA c; a lane's 4 rows
  // lie in one slice (SR >= 8 for nsplit <= 8).
  const int SR = kFaBM / nsplit;
  float* rO = sKb;                    // [nsplit][SR][D]
  float* rM = rO + kFaBM * D;         // [nsplit][SR]
  float* rL = rM + kFaBM;             // [nsplit][SR]
  cluster_sync_all();                 // every CTA of the cluster is done with its K buffers
  {
    const int dst = rb / SR;
    const int rr = (split * SR + rb - dst * SR);   // row index in dst's [nsplit*SR] rows
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint32_t orow = cluster_map(smem_u32(rO + (rr + i) * D), dst);
#pragma unroll
      for (int e = 0; e < NG; ++e) {
        const uint32_t a = orow + (e * 16 * G + tc * G) * 4;
        if constexpr (G == 4)
          st_cluster_v4(a, acc[i][e * 4 + 0], acc[i][e * 4 + 1], acc[i][e * 4 + 2],
                        acc[i][e * 4 + 3]);
        else
          st_cluster_v2(a, acc[i][e * 2 + 0], acc[i][e * 2 + 1]);
      }
      if (tc == 0) {
        st_cluster_f32(cluster_map(smem_u32(rM + rr + i), dst), m[i]);
        st_cluster_f32(cluster_map(smem_u32(rL + rr + i), dst), l[i]);
      }
    }
  }
  cluster_sync_all();                 // all partials of this CTA's slice have landed
  constexpr int C4 = D / 4;
  for (int idx = tid; idx < SR * C4; idx += 256) {
    const int rr = idx / C4, c = (idx - rr * C4) * 4;
    const int row = r0 + split * SR + rr;
    if (row >= N || c >= d) continue;
    float mx = NEG_INF;
    for (int s2 = 0; s2 < nsplit; ++s2) mx = fmaxf(mx, rM[s2 * SR + rr]);
    float tot = 0.f;
    float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (mx != NEG_INF) {
      for (int s2 = 0; s2 < nsplit; ++s2) {
        const float w = ex2(rM[s2 * SR + rr] - mx);
        tot += rL[s2 * SR + rr] * w;
        const float4 t = *reinterpret_cast<const float4*>(rO + (s2 * SR + rr) * D + c);
        o4.x = fmaf(w, t.x, o4.x);
        o4.y = fmaf(w, t.y, o4.y);
        o4.z = fmaf(w, t.z, o4.z);
        o4.w = fmaf(w, t.w, o4.w);
      }
    }
    const float inv = tot > 0.f ? 1.f / tot : 0.f;
    float* op = Ob + static_cast<size_t>(row) * d + c;
    if (vec) {
      *reinterpret_cast<float4*>(op) = make_float4(o4.x * inv, o4.y * inv, o4.z * inv, o4.w * inv);
    } else {
      const float ov[4] = {o4.x, o4.y, o4.z, o4.w};
      for (int g = 0; g < 4 && c + g < d; ++g) op[g] = ov[g] * inv;
    }
  }
}

// Number of CTAs (one cluster) that share a row tile's key tiles: the most (up to 8 and
// up to the key-tile count) that still fit the grid in one wave of resident CTAs (two
// per SM at D <= 64, one at D = 128). Config 1 ([1, 8, 512, 64]) takes 4: 256 CTAs.
// FE_FP32_SPLIT=1,2,4,8 overrides the choice (tuning).
static int fa2_fp32_split(int row_tiles, int bh, int M, int d) {
  static const int forced = [] {
    const char* s = getenv("FE_FP32_SPLIT");
    const int v = s ? atoi(s) : 0;
    return (v == 1 || v == 2 || v == 4 || v == 8) ? v : 0;
  }();
  const int ktiles = (M + kFaBN - 1) / kFaBN;
  int n = 1;
  if (forced) {
    n = forced;
  } else {
    const long long slots = static_cast<long long>(sm_count()) * (d <= 64 ? 2 : 1);
    const long long base = static_cast<long long>(row_tiles) * bh;
    while (n < 8 && base * n * 2 <= slots) n *= 2;
  }
  while (n > 1 && n > ktiles) n /= 2;
  return n;
}

template <int D>
static cudaError_t launch_fa2_fp32_d(const float* q, const float* k, const float* v, float* o,
                                     int B, int H, int N, int M, int d, float sl, int causal,
                                     cudaStream_t st) {
  const int smem = FaSmem<D>::bytes;
  cudaError_t e = ensure_smem_optin(reinterpret_cast<const void*>(fa2_fp32_kernel<D>), smem);
  if (e != cudaSuccess) return e;
  const int row_tiles = (N + kFaBM - 1) / kFaBM;
  const int nsplit = fa2_fp32_split(row_tiles, B * H, M, d);
  const auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  const int vec = (d % 4 == 0) && al(q) && al(k) && al(v) && al(o);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(row_tiles * nsplit, B * H);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = nsplit;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = nsplit > 1 ? 1 : 0;
  e = cudaLaunchKernelEx(&cfg, fa2_fp32_kernel<D>, q, k, v, o, N, M, d, sl, causal, nsplit, vec);
  if (e != cudaSuccess) return e;
  return cudaGetLastError();
}

cudaError_t launch_fa2_fp32(const float* q, const float* k, const float* v, float* o, int B, int H,
                            int N, int M, int d, float scale, int causal, cudaStream_t st) {
  if (fa2_tf32_eligible(q, k, v, o, B, H, N, M, d))
    return launch_fa2_tf32(q, k, v, o, B, H, N, M, d, scale, causal, st);
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
// Warp decode core shared by the paged and dense fp32 decoders. A CTA of NW warps
// works on up to HG query heads that read the same KV head. Each warp takes groups of
// TB consecutive tokens round-robin.
//  * It loads the K and V rows of all TB tokens before it uses the first, so TB rows
//    per warp are in flight.
//  * It forms all TB x HG partial dot products, then reduces them together (each
//    butterfly step over every value, so the shuffles overlap).
//  * It updates the online softmax once per head per group: one rescale and TB
//    exponentials.
// One row at a time, with a reduction and a rescale per token and head, left these
// HBM-bound kernels latency-bound at 14% of the copy bandwidth. Lanes own D/32 dims,
// and q lives in registers. The NW warp states are merged through shared memory at
// the end.
template <int D, int HG>
constexpr int decode_tb() { return (D <= 128 && HG <= 4) ? 8 : 4; }

template <int D, int HG>
struct WarpDecode {
  static constexpr int E = D / 32;
  static constexpr int TB = decode_tb<D, HG>();
  float m[HG], l[HG], acc[HG][E], qr[HG][E];
  // q: [HG][D] in shared memory (zero padded), read into registers once.
  __device__ __forceinline__ void init(const float* q, int lane) {
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      m[h] = NEG_INF;
      l[h] = 0.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        acc[h][e] = 0.f;
        qr[h][e] = q[h * D + lane + 32 * e];
      }
    }
  }
  // k[j], v[j]: rows of token j of the group (d valid floats), used where valid bit j
  // is set (warp-uniform).
  __device__ __forceinline__ void tokens(const float* const (&k)[TB], const float* const (&v)[TB],
                                         unsigned valid, int d, int nh, float sl, int lane) {
    if (valid == 0) return;
    float kv[TB][E], vv[TB][E];
#pragma unroll
    for (int j = 0; j < TB; ++j)
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const int c = lane + 32 * e;
        const bool in = ((valid >> j) & 1u) && c < d;
        kv[j][e] = in ? __ldg(k[j] + c) : 0.f;
        vv[j][e] = in ? __ldg(v[j] + c) : 0.f;
      }
    float sp[TB][HG];
#pragma unroll
    for (int j = 0; j < TB; ++j)
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        float t = 0.f;
#pragma unroll
        for (int e = 0; e < E; ++e) t = fmaf(qr[h][e], kv[j][e], t);
        sp[j][h] = t;
      }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1)
#pragma unroll
      for (int j = 0; j < TB; ++j)
#pragma unroll
        for (int h = 0; h < HG; ++h) sp[j][h] += __shfl_xor_sync(0xffffffffu, sp[j][h], off);
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      if (h >= nh) break;
      float mx = NEG_INF;
#pragma unroll
      for (int j = 0; j < TB; ++j)
        if ((valid >> j) & 1u) mx = fmaxf(mx, sp[j][h] * sl);
      const float mn = fmaxf(m[h], mx);  // finite: at least one token is valid
      const float corr = ex2(m[h] - mn);
      float psum = 0.f;
      float pv[E];
#pragma unroll
      for (int e = 0; e < E; ++e) pv[e] = 0.f;
#pragma unroll
      for (int j = 0; j < TB; ++j) {
        const float pj = ((valid >> j) & 1u) ? ex2(fmaf(sp[j][h], sl, -mn)) : 0.f;
        psum += pj;
#pragma unroll
        for (int e = 0; e < E; ++e) pv[e] = fmaf(pj, vv[j][e], pv[e]);
      }
      l[h] = fmaf(l[h], corr, psum);
#pragma unroll
      for (int e = 0; e < E; ++e) acc[h][e] = fmaf(acc[h][e], corr, pv[e]);
      m[h] = mn;
    }
  }
  // Merge NW warp states through smem (cm/cl: [NW][HG], co: [NW][HG][D]); returns the
  // merged (M, L, O) for (h, c) pairs handled by the calling thread via `emit`.
  template <int NW, typename Emit>
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
      for (int w = 0; w < NW; ++w) Mx = fmaxf(Mx, cm[w * HG + h]);
      float L = 0.f, Ov = 0.f;
      for (int w = 0; w < NW; ++w) {
        const float mw = cm[w * HG + h];
        const float wt = mw == NEG_INF ? 0.f : ex2(mw - Mx);
        L += cl[w * HG + h] * wt;
        Ov += co[(w * HG + h) * D + c] * wt;
      }
      emit(h, c, Mx, L, Ov);
    }
  }
};

// Vectorised variant of WarpDecode for head dim D = d in {64, 128}, HG in {4, 8} and
// 16-byte aligned rows. TB * HG = 32 (token, head) scores per group.
//  * Lane i owns dims [i*C, (i+1)*C), C = D/32, and loads a row's share as one 64- or
//    128-bit word.
//  * The 32 partial dot products are reduce-scattered: five butterfly steps that halve
//    the set each time, 31 shuffles in all. Lane l then holds the full score of token
//    l / HG, head l % HG.
//  * The softmax of a group takes one exponential per lane, plus one per head for the
//    rescale; the group maxima of the heads are exchanged by shuffles.
//  * P V takes each p by shuffle from the lane that holds it.
// The sum l stays split over the lanes of each head until the end.
template <int D, int HG>
struct WarpDecodeV {
  static constexpr int C = D / 32;
  static constexpr int TB = 32 / HG;
  static_assert((D == 64 || D == 128) && (HG == 4 || HG == 8), "vector decode shape");
  using VecT = typename std::conditional<C == 4, float4, float2>::type;
  float m[HG], acc[HG][C], qr[HG][C];
  float m_own, l_part;  // running max and partial sum of head (lane % HG)
  __device__ __forceinline__ void init(const float* q, int lane) {
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      m[h] = NEG_INF;
#pragma unroll
      for (int c = 0; c < C; ++c) {
        acc[h][c] = 0.f;
        qr[h][c] = q[h * D + lane * C + c];
      }
    }
    m_own = NEG_INF;
    l_part = 0.f;
  }
  __device__ __forceinline__ static void load_row(const float* p, bool in, float (&x)[C]) {
    if (in) {
      const VecT t = __ldg(reinterpret_cast<const VecT*>(p));
      x[0] = t.x;
      x[1] = t.y;
      if constexpr (C == 4) {
        x[2] = t.z;
        x[3] = t.w;
      }
    } else {
#pragma unroll
      for (int c = 0; c < C; ++c) x[c] = 0.f;
    }
  }
  __device__ __forceinline__ void tokens(const float* const (&k)[TB], const float* const (&v)[TB],
                                         unsigned valid, int, int, float sl, int lane) {
    if (valid == 0) return;
    float kv[TB][C], vv[TB][C];
#pragma unroll
    for (int j = 0; j < TB; ++j) {
      const bool in = (valid >> j) & 1u;
      load_row(k[j] + lane * C, in, kv[j]);
      load_row(v[j] + lane * C, in, vv[j]);
    }
    float x[32];  // x[j * HG + h]: this lane's part of q_h . k_j
#pragma unroll
    for (int j = 0; j < TB; ++j)
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        float t = 0.f;
#pragma unroll
        for (int c = 0; c < C; ++c) t = fmaf(qr[h][c], kv[j][c], t);
        x[j * HG + h] = t;
      }
    // reduce-scatter: after the step over lane bit b, the lane keeps the half of the
    // remaining indices selected by its bit b; at the end x[0] is index = lane
#pragma unroll
    for (int half = 16; half >= 1; half >>= 1) {
      const bool up = lane & half;
#pragma unroll
      for (int i = 0; i < half; ++i) {
        const float send = up ? x[i] : x[i + half];
        const float keep = up ? x[i + half] : x[i];
        x[i] = keep + __shfl_xor_sync(0xffffffffu, send, half);
      }
    }
    const int j_own = lane / HG;
    const bool v_own = (valid >> j_own) & 1u;
    const float s_own = v_own ? x[0] * sl : NEG_INF;
    // group max per head over the lanes of that head (lane % HG equal)
    float mx = s_own;
#pragma unroll
    for (int off = HG; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    const float m_new = fmaxf(m_own, mx);  // finite: at least one token is valid
    const float p_own = v_own ? ex2(s_own - m_new) : 0.f;
    l_part = fmaf(l_part, ex2(m_own - m_new), p_own);
    m_own = m_new;
#pragma unroll
    for (int h = 0; h < HG; ++h) {
      const float mh = __shfl_sync(0xffffffffu, m_new, h);  // lane h holds head h
      const float corr = ex2(m[h] - mh);
      m[h] = mh;
#pragma unroll
      for (int c = 0; c < C; ++c) acc[h][c] *= corr;
    }
#pragma unroll
    for (int j = 0; j < TB; ++j)
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        const float pj = __shfl_sync(0xffffffffu, p_own, j * HG + h);
#pragma unroll
        for (int c = 0; c < C; ++c) acc[h][c] = fmaf(pj, vv[j][c], acc[h][c]);
      }
  }
  // Merge NW warp states through smem (cm/cl: [NW][HG], co: [NW][HG][D]), as WarpDecode.
  template <int NW, typename Emit>
  __device__ __forceinline__ void merge(float* cm, float* cl, float* co, int nh, int d, int warp,
                                        int lane, Emit emit) {
    float lsum = l_part;
#pragma unroll
    for (int off = HG; off < 32; off <<= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
    if (lane < HG) {  // lane h holds head h's max and, now, its sum
      cm[warp * HG + lane] = m_own;
      cl[warp * HG + lane] = lsum;
    }
#pragma unroll
    for (int h = 0; h < HG; ++h)
#pragma unroll
      for (int c = 0; c < C; ++c) co[(warp * HG + h) * D + lane * C + c] = acc[h][c];
    __syncthreads();
    for (int i = threadIdx.x; i < nh * D; i += blockDim.x) {
      const int h = i / D, c = i - h * D;
      if (c >= d) continue;
      float Mx = NEG_INF;
      for (int w = 0; w < NW; ++w) Mx = fmaxf(Mx, cm[w * HG + h]);
      float L = 0.f, Ov = 0.f;
      for (int w = 0; w < NW; ++w) {
        const float mw = cm[w * HG + h];
        const float wt = mw == NEG_INF ? 0.f : ex2(mw - Mx);
        L += cl[w * HG + h] * wt;
        Ov += co[(w * HG + h) * D + c] * wt;
      }
      emit(h, c, Mx, L, Ov);
    }
  }
};

// The decoder a paged kernel instantiates: vectorised for the shapes it supports.
template <int D, int HG, bool VEC>
using PagedDecoder = typename std::conditional<VEC, WarpDecodeV<D, HG>, WarpDecode<D, HG>>::type;

// Paged fp32 decode: grid (Hkv * head_chunks, S), 4 warps; the chunk's query heads
// share every K/V row read.
template <int D, int HG, bool VEC>
__global__ void __launch_bounds__(128) paged_fp32_kernel(
    const float* __restrict__ q, const float* __restrict__ kc, const float* __restrict__ vc,
    float* __restrict__ out, const int* __restrict__ bt, const int* __restrict__ lens, int H,
    int Hkv, int d, int bs, int maxb, int num_blocks, float sl, unsigned* err) {
  constexpr int NW = 4;
  using WD = PagedDecoder<D, HG, VEC>;
  constexpr int TB = WD::TB;
  __shared__ float sq[HG * D];
  __shared__ float cm[NW * HG], cl[NW * HG];
  __shared__ float co[NW * HG * D];
  const int G = H / Hkv, chunks = (G + HG - 1) / HG;
  const int kvh = blockIdx.x / chunks, ch = blockIdx.x - kvh * chunks;
  const int seq = blockIdx.y;
  const int h0 = kvh * G + ch * HG;
  const int nh = min(HG, G - ch * HG);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < HG * D; i += NW * 32) {
    const int h = i / D, c = i - h * D;
    sq[i] = (h < nh && c < d) ? q[(static_cast<size_t>(seq) * H + h0 + h) * d + c] : 0.f;
  }
  __syncthreads();
  const int ctx = lens[seq];
  WD st;
  st.init(sq, lane);
  for (int t0 = warp * TB; t0 < ctx; t0 += NW * TB) {
    const float* kp[TB];
    const float* vp[TB];
    unsigned valid = 0;
#pragma unroll
    for (int j = 0; j < TB; ++j) {
      const int t = t0 + j;
      kp[j] = vp[j] = kc;
      if (t >= ctx) continue;
      if (t / bs >= maxb) {  // context longer than the block-table row
        if (lane == 0) atomicOr(err, kErrBadBlock);
        continue;
      }
      const int phys = __ldg(bt + static_cast<size_t>(seq) * maxb + t / bs);
      if (phys < 0 || (num_blocks > 0 && phys >= num_blocks)) {
        if (lane == 0) atomicOr(err, kErrBadBlock);
        continue;
      }
      const size_t off = ((static_cast<size_t>(phys) * Hkv + kvh) * bs + t % bs) * d;
      kp[j] = kc + off;
      vp[j] = vc + off;
      valid |= 1u << j;
    }
    st.tokens(kp, vp, valid, d, nh, sl, lane);
  }
  st.template merge<NW>(cm, cl, co, nh, d, warp, lane,
                        [&](int h, int c, float, float L, float Ov) {
                          out[(static_cast<size_t>(seq) * H + h0 + h) * d + c] =
                              L > 0.f ? Ov / L : 0.f;
                        });
}

// Launches the vectorised decoder where the shape allows it, else the generic one.
template <int D, int HG>
static cudaError_t launch_paged_fp32_v(bool vec, dim3 grid, const float* q, const float* kc,
                                       const float* vc, float* out, const int* bt,
                                       const int* lens, int H, int Hkv, int d, int bs, int maxb,
                                       int num_blocks, float sl, unsigned* err, cudaStream_t st) {
  if constexpr ((D == 64 || D == 128) && (HG == 4 || HG == 8)) {
    if (vec) {
      paged_fp32_kernel<D, HG, true><<<grid, 128, 0, st>>>(q, kc, vc, out, bt, lens, H, Hkv, d,
                                                           bs, maxb, num_blocks, sl, err);
      return cudaGetLastError();
    }
  }
  paged_fp32_kernel<D, HG, false><<<grid, 128, 0, st>>>(q, kc, vc, out, bt, lens, H, Hkv, d, bs,
                                                        maxb, num_blocks, sl, err);
  return cudaGetLastError();
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
  const bool vec = (d == 64 || d == 128) && (HG == 4 || HG == 8) &&
                   ((reinterpret_cast<uintptr_t>(kc) | reinterpret_cast<uintptr_t>(vc)) & 15) == 0;
#define FE_P(D_, HG_)                                                                  \
  if (d <= D_ && HG == HG_)                                                            \
    return launch_paged_fp32_v<D_, HG_>(vec, grid, q, kc, vc, out, bt, lens, H, Hkv, d, bs, \
                                        maxb, num_blocks, sl, err, st);
  FE_P(64, 1) FE_P(64, 2) FE_P(64, 4) FE_P(64, 8)
  FE_P(128, 1) FE_P(128, 2) FE_P(128, 4) FE_P(128, 8)
  FE_P(256, 1) FE_P(256, 2) FE_P(256, 4)
#undef FE_P
  return cudaErrorInvalidValue;
}

// Dense split-KV stage 1 (fp32): grid (splits, B*H), 8 warps. Writes the
// unnormalised O, m (log2 units) and l of split s of row bh; an empty split writes
// (-inf, 0).
template <int D>
__global__ void __launch_bounds__(256) decode_split_fp32_kernel(
    const float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
    float* __restrict__ part_o, float* __restrict__ part_ml, int M, int d, int splits, float sl) {
  constexpr int NW = 8;
  using WD = WarpDecode<D, 1>;
  constexpr int TB = WD::TB;
  __shared__ float sq[D];
  __shared__ float cm[NW], cl[NW];
  __shared__ float co[NW * D];
  const int s = blockIdx.x;
  const size_t bh = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int per = (M + splits - 1) / splits;
  const int t0 = s * per, t1 = min(M, t0 + per);
  for (int c = threadIdx.x; c < D; c += NW * 32) sq[c] = c < d ? q[bh * d + c] : 0.f;
  __syncthreads();
  WD st;
  st.init(sq, lane);
  for (int tb = t0 + warp * TB; tb < t1; tb += NW * TB) {
    const float* kp[TB];
    const float* vp[TB];
    unsigned valid = 0;
#pragma unroll
    for (int j = 0; j < TB; ++j) {
      const int t = min(tb + j, t1 - 1);
      kp[j] = k + (bh * M + t) * d;
      vp[j] = v + (bh * M + t) * d;
      if (tb + j < t1) valid |= 1u << j;
    }
    st.tokens(kp, vp, valid, d, 1, sl, lane);
  }
  const size_t slot = bh * splits + s;
  st.template merge<NW>(cm, cl, co, 1, d, warp, lane,
                        [&](int, int c, float Mx, float L, float Ov) {
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
    decode_split_fp32_kernel<64><<<grid, 256, 0, st>>>(q, k, v, part_o, part_ml, M, d, splits, sl);
  else if (d <= 128)
    decode_split_fp32_kernel<128><<<grid, 256, 0, st>>>(q, k, v, part_o, part_ml, M, d, splits, sl);
  else if (d <= 256)
    decode_split_fp32_kernel<256><<<grid, 256, 0, st>>>(q, k, v, part_o, part_ml, M, d, splits, sl);
  else
    return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace simt
}  // namespace fe
