// Paged-KV decode attention for bf16 / fp16 caches on sm_100a.
//
// Semantics follow the reference's PagedAttention v1 (src/paged_attention.cu:14-178,
// python/flash_engine/ops.py:59-101): for sequence s and query head h,
//   out[s,h] = softmax(q[s,h] . K^T * scale) V over tokens [0, context_lens[s]),
// token t living in row t % BS of physical block block_tables[s, t / BS], KV head
// h / (H / Hkv) (src/paged_attention.cu:33-35, :54-84). Cache layout
// [num_blocks, Hkv, BS, d], the one the reference's fp32 kernel implements.
//
// Design (B200):
//  * Persistent CTAs (SMs x occupancy). Work units are (sequence, split, KV head,
//    head chunk); every CTA builds the compact unit list itself with a block-wide
//    prefix scan of the per-sequence split counts (read from context_lens), so no
//    host synchronisation or scratch is needed to skip empty work.
//  * One producer warp streams each (block, KV head) page of K and V into a ring of
//    shared-memory stages with 2-D TMA bulk-tensor loads (128-byte swizzle, L2
//    evict-first, no multicast), completing on mbarriers. Block-table entries are
//    fetched 32 at a time by the warp.
//  * NCW consumer warps take pages round-robin. Per 16 tokens a warp computes
//    S^T = K Q^T with mma.m16n8k16 (tokens x query heads: all G query heads of the
//    group share every K/V byte fetched), does the online-softmax update in the
//    log2 domain, turns P^T into the B operand with movmatrix, and accumulates
//    O^T += V^T P^T (V^T fragments via ldmatrix.trans from the swizzled tile).
//  * The consumer warps merge their (m, l, O) in shared memory at the end of a
//    unit and write either the final output (single-split sequences) or an fp32
//    partial (O, m, l) for the log-sum-exp merge kernel.
#include <cooperative_groups.h>
#include <limits.h>

#include <type_traits>

#include "internal.h"
#include "paged_decode.h"
#include "ptx.cuh"

namespace fe {
namespace paged {

template <typename T>
struct Elem;
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    mma_bf16_16816(d, a, b0, b1);
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return pack_bf16x2(lo, hi); }
  static __device__ __forceinline__ __nv_bfloat16 cvt(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Elem<half> {
  static __device__ __forceinline__ void mma(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
    mma_f16_16816(d, a, b0, b1);
  }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) { return pack_f16x2(lo, hi); }
  static __device__ __forceinline__ half cvt(float x) { return __float2half_rn(x); }
};

// Page range of split `split` of sequence `ctx` inside the token window.
struct SplitRange {
  int p0, p1;  // pages [p0, p1)
  int lo, hi;  // valid tokens [lo, hi)
};
__device__ __forceinline__ SplitRange split_range(int ctx, int tb, int te, int bs, int pps,
                                                  int split) {
  SplitRange r;
  r.lo = max(tb, 0);
  r.hi = min(te, ctx);
  if (r.hi <= r.lo) {
    r.p0 = r.p1 = 0;
    return r;
  }
  const int pb = r.lo / bs, pe = (r.hi + bs - 1) / bs;
  r.p0 = pb + split * pps;
  r.p1 = min(pe, r.p0 + pps);
  if (r.p1 < r.p0) r.p1 = r.p0;
  return r;
}

__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ int warp_incl_scan(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// Page gi of a CTA (its running page counter) belongs to consumer warp gi % NCW
// and lives in that warp's own ring of DEPTH stages. Every stage therefore has a
// single consumer that takes its pages in order, so a parity wait can never be
// satisfied by an older phase of the same stage.
template <int NCW, int DEPTH>
struct StageOf {
  int s, round;
  __device__ __forceinline__ explicit StageOf(int gi) {
    const int j = gi / NCW;
    s = (j % DEPTH) * NCW + (gi - j * NCW);
    round = j / DEPTH;
  }
};

template <typename T, int D, int BS, int NT, int NCW, int NSTAGE>
struct Cfg {
  static constexpr int HPC = 8 * NT;       // query heads per CTA
  static constexpr int HALVES = D / 64;    // 128-byte swizzle atoms per row
  static constexpr int TILE = BS * D * 2;  // bytes of one page of K (or V)
  static constexpr int STAGE = 2 * TILE;
  static constexpr int CSTRIDE = D + 4;    // padded row of the merge buffer (floats)
  static constexpr int NTHREADS = (NCW + 1) * 32;
  static constexpr int COMB_BYTES = NCW * HPC * (2 + CSTRIDE) * 4;
  static constexpr int FIXED_SMEM = 1024 /*align slack*/ + NSTAGE * STAGE + COMB_BYTES +
                                    NSTAGE * 16 /*bars*/ + NSTAGE * 4 + 64;
  static int smem_bytes(int num_seqs) { return FIXED_SMEM + (num_seqs + 1) * 4; }
};

// Number of work splits of one sequence (0 if its token window is empty; 1 for an
// empty sequence when the final output must still be written).
__device__ __forceinline__ int seq_splits(int ctx, int tb, int te, int bs, int pps,
                                          bool direct_final) {
  const int lo = max(tb, 0), hi = min(te, ctx);
  if (hi <= lo) return direct_final ? 1 : 0;
  const int np = (hi + bs - 1) / bs - lo / bs;
  return (np + pps - 1) / pps;
}

template <typename T, int D, int BS, int NT, int NCW, int NSTAGE>
__global__ void __launch_bounds__((NCW + 1) * 32, 1)
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const Params p) {
  using C = Cfg<T, D, BS, NT, NCW, NSTAGE>;
  constexpr int HPC = C::HPC, HALVES = C::HALVES, TILE = C::TILE, STAGE = C::STAGE;
  constexpr int CSTRIDE = C::CSTRIDE, NTH = C::NTHREADS;
  constexpr float NEG_INF = -__builtin_huge_valf();

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  float* comb_m = reinterpret_cast<float*>(smem + NSTAGE * STAGE);  // [NCW][HPC]
  float* comb_l = comb_m + NCW * HPC;                                // [NCW][HPC]
  float* comb_o = comb_l + NCW * HPC;                                // [NCW][HPC][CSTRIDE]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NSTAGE * STAGE + C::COMB_BYTES);
  uint64_t* empty = full + NSTAGE;
  int* stage_valid = reinterpret_cast<int*>(empty + NSTAGE);
  int* prefix = stage_valid + NSTAGE;  // [num_seqs + 1]
  __shared__ int warp_tot[NCW + 1];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int S = p.num_seqs;
  const int Hkv = p.num_kv_heads, G = p.num_heads / p.num_kv_heads;
  const int HC = p.head_chunks;
  const bool direct_final = p.direct_final != 0;

  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
  }

  // ---- compact unit list: prefix[s] = first compact (sequence, split) index of s.
  {
    const int per = (S + NTH - 1) / NTH;
    const int beg = min(S, tid * per), end = min(S, beg + per);
    int local = 0;
    for (int i = beg; i < end; ++i) {
      const int n = seq_splits(__ldg(p.context_lens + i), p.tok_begin, p.tok_end, BS,
                               p.pages_per_split, direct_final);
      // More splits than partial slots means context_len > max_context_len: the
      // tail is dropped and the error word says so.
      if (n > p.max_splits && blockIdx.x == 0) atomicOr(p.err, kErrBadBlock);
      local += min(n, p.max_splits);
    }
    const int incl = warp_incl_scan(local);
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      int v = lane <= NCW ? warp_tot[lane] : 0;
      v = warp_incl_scan(v);
      if (lane <= NCW) warp_tot[lane] = v;
    }
    __syncthreads();
    int run = incl - local + (warp > 0 ? warp_tot[warp - 1] : 0);
    for (int i = beg; i < end; ++i) {
      prefix[i] = run;
      run += min(seq_splits(__ldg(p.context_lens + i), p.tok_begin, p.tok_end, BS,
                            p.pages_per_split, direct_final),
                 p.max_splits);
    }
    if (tid == 0) prefix[S] = warp_tot[NCW];
    __syncthreads();
  }
  const int units_per_cu = Hkv * HC;
  const int total_units = prefix[S] * units_per_cu;

  // unit -> (seq, split, kvh, hc, page range)
  auto decode_unit = [&](int u, int& seq, int& split, int& kvh, int& hc, SplitRange& r) {
    const int cu = u / units_per_cu, y = u - cu * units_per_cu;
    kvh = y / HC;
    hc = y - kvh * HC;
    int lo = 0, hi = S;  // largest s with prefix[s] <= cu
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (prefix[mid] <= cu) lo = mid; else hi = mid;
    }
    seq = lo;
    split = cu - prefix[lo];
    r = split_range(__ldg(p.context_lens + seq), p.tok_begin, p.tok_end, BS, p.pages_per_split,
                    split);
  };

  if (warp == NCW) {
    // ===================================================== producer warp
    if (lane == 0) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    const uint64_t pol = l2_policy_evict_first();
    int gi = 0;  // pages issued by this CTA so far (identical count on every lane)
    bool ok = true;
    for (int u = blockIdx.x; u < total_units && ok; u += gridDim.x) {
      int seq, split, kvh, hc;
      SplitRange r;
      decode_unit(u, seq, split, kvh, hc, r);
      const int npg = r.p1 - r.p0;
      const int* bt = p.block_tables + static_cast<size_t>(seq) * p.max_blocks_per_seq;
      for (int base = 0; base < npg && ok; base += 32) {
        int phys = 0, valid = 0;
        if (base + lane < npg && r.p0 + base + lane >= p.max_blocks_per_seq) {
          atomicOr(p.err, kErrBadBlock);  // context longer than the block table row
        } else if (base + lane < npg) {
          phys = __ldg(bt + r.p0 + base + lane);
          const long long row = (static_cast<long long>(phys) * Hkv + kvh) * BS;
          valid = phys >= 0 && (p.num_phys_blocks <= 0 || phys < p.num_phys_blocks) &&
                  row + BS <= static_cast<long long>(INT_MAX);
          if (!valid) atomicOr(p.err, kErrBadBlock);
        }
        const int cnt = min(32, npg - base);
        for (int k = 0; k < cnt; ++k) {
          const int ph = __shfl_sync(0xffffffffu, phys, k);
          const int vd = __shfl_sync(0xffffffffu, valid, k);
          int good = 1;
          if (lane == 0) {
            const StageOf<NCW, NSTAGE / NCW> so(gi);
            const int s = so.s, rnd = so.round;
            if (rnd > 0 && !mbar_wait(&empty[s], (rnd - 1) & 1)) {
              atomicOr(p.err, kErrWaitTimeout);
              good = 0;
            } else {
              stage_valid[s] = vd;
              uint8_t* ks = smem + s * STAGE;
              uint8_t* vs = ks + TILE;
              if (vd) {
                mbar_arrive_expect_tx(&full[s], STAGE);
                const int y = (ph * Hkv + kvh) * BS;
#ifdef FE_DEBUG_CHECKS
                if (static_cast<long long>(y) + BS > p.dbg_kv_rows) atomicOr(p.err, 1u << 8);
#endif
#pragma unroll
                for (int h = 0; h < HALVES; ++h) {
                  tma_load_2d(ks + h * BS * 128, &kmap, h * 64, y, &full[s], pol);
                  tma_load_2d(vs + h * BS * 128, &vmap, h * 64, y, &full[s], pol);
                }
              } else {
                mbar_arrive(&full[s]);  // nothing to load; consumers skip the page
              }
            }
          }
          good = __shfl_sync(0xffffffffu, good, 0);
          if (!good) {
            ok = false;
            break;
          }
          ++gi;
        }
      }
    }
    // Drain: no bulk copy of this CTA may still be in flight when it exits.
    if (lane == 0) {
      for (int j = max(0, gi - NSTAGE); j < gi; ++j) {
        const StageOf<NCW, NSTAGE / NCW> so(j);
        if (!mbar_wait(&full[so.s], so.round & 1)) {
          atomicOr(p.err, kErrWaitTimeout);
          break;
        }
      }
    }
    return;
  }

  // ======================================================= consumer warps
  using E = Elem<T>;
  const int g = lane >> 2, c = lane & 3;
  const T* __restrict__ qbase = reinterpret_cast<const T*>(p.q);
  const uint32_t ring = smem_u32(smem);
  const float sl = p.scale_log2;

  uint32_t qf[NT][D / 16][2];
  uint32_t qn[NT][D / 16][2];
  auto load_q = [&](uint32_t (&dst)[NT][D / 16][2], int u) {
    int seq, split, kvh, hc;
    SplitRange r;
    decode_unit(u, seq, split, kvh, hc, r);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int gh = hc * HPC + nt * 8 + g;
      const bool v = gh < G;
      const T* qp = qbase + (static_cast<size_t>(seq) * p.num_heads + kvh * G + (v ? gh : 0)) * D;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        dst[nt][ks][0] = v ? __ldg(reinterpret_cast<const unsigned*>(qp + ks * 16 + 2 * c)) : 0u;
        dst[nt][ks][1] = v ? __ldg(reinterpret_cast<const unsigned*>(qp + ks * 16 + 8 + 2 * c)) : 0u;
      }
    }
  };

  int gbase = 0;  // pages consumed by this CTA before the current unit
  bool ok = true;
  if (blockIdx.x < total_units) load_q(qn, blockIdx.x);
  for (int u = blockIdx.x; u < total_units; u += gridDim.x) {
    int seq, split, kvh, hc;
    SplitRange r;
    decode_unit(u, seq, split, kvh, hc, r);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        qf[nt][ks][0] = qn[nt][ks][0];
        qf[nt][ks][1] = qn[nt][ks][1];
      }
    if (u + gridDim.x < total_units) load_q(qn, u + gridDim.x);  // prefetch the next unit's q

    float m_run[NT][2], l_run[NT][2], o[NT][D / 16][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = NEG_INF;
      l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
    }

    const int npg = r.p1 - r.p0;
    const int first = ((warp - gbase) % NCW + NCW) % NCW;
    for (int i = first; i < npg && ok; i += NCW) {
      const int gi = gbase + i;
      const StageOf<NCW, NSTAGE / NCW> so(gi);
      const int s = so.s;
      const bool waited = mbar_wait(&full[s], so.round & 1);
      if (!__all_sync(0xffffffffu, waited)) {
        if (lane == 0) atomicOr(p.err, kErrWaitTimeout);
        ok = false;
        break;
      }
      const int t0 = (r.p0 + i) * BS;
      const int vlo = max(r.lo - t0, 0), vhi = min(r.hi - t0, BS);
      const uint32_t ks = ring + s * STAGE, vs = ks + TILE;
      bool zeroed = false;
      if (stage_valid[s]) {
        if (vlo > 0 || vhi < BS) {
          // Rows outside the window may hold anything (NaN included); P is 0 there
          // but 0 * NaN is not, so clear those V rows before the PV product.
          uint8_t* vrow = smem + s * STAGE + TILE;
          for (int idx = lane; idx < BS * HALVES * 8; idx += 32) {
            const int row = (idx >> 3) % BS, h = idx / (8 * BS), ch = idx & 7;
            if (row < vlo || row >= vhi)
              *reinterpret_cast<uint4*>(vrow + h * BS * 128 + row * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
          }
          __syncwarp();
          zeroed = true;
        }
#pragma unroll
        for (int t = 0; t < BS / 16; ++t) {
          if (t * 16 >= vhi || t * 16 + 16 <= vlo) continue;
          float sacc[NT][4];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) sacc[nt][0] = sacc[nt][1] = sacc[nt][2] = sacc[nt][3] = 0.f;
          // S^T = K Q^T : A = K tile (16 tokens x 16 dims per k-step)
          {
            const int mq = lane >> 3;
            const int tok = t * 16 + (lane & 7) + 8 * (mq & 1);
#pragma unroll
            for (int kk = 0; kk < D / 16; ++kk) {
              const int ch = 2 * kk + (mq >> 1);
              const uint32_t addr =
                  ks + (ch >> 3) * (BS * 128) + tok * 128 + ((((ch & 7) ^ (tok & 7))) << 4);
              uint32_t a[4];
              ldsm_x4(addr, a[0], a[1], a[2], a[3]);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) E::mma(sacc[nt], a, qf[nt][kk][0], qf[nt][kk][1]);
            }
          }
          // online softmax (log2 domain)
          const int rA = t * 16 + g, rB = rA + 8;
          const bool inA = rA >= vlo && rA < vhi, inB = rB >= vlo && rB < vhi;
          uint32_t pb[NT][2];
#pragma unroll
          for (int nt = 0; nt < NT; ++nt) {
            const float x0 = inA ? sacc[nt][0] * sl : NEG_INF;
            const float x1 = inA ? sacc[nt][1] * sl : NEG_INF;
            const float x2 = inB ? sacc[nt][2] * sl : NEG_INF;
            const float x3 = inB ? sacc[nt][3] * sl : NEG_INF;
            float mx0 = fmaxf(x0, x2), mx1 = fmaxf(x1, x3);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
              mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
              mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
            }
            const float mn0 = fmaxf(m_run[nt][0], mx0), mn1 = fmaxf(m_run[nt][1], mx1);
            const float mu0 = mn0 == NEG_INF ? 0.f : mn0, mu1 = mn1 == NEG_INF ? 0.f : mn1;
            const float corr0 = ex2(m_run[nt][0] - mu0), corr1 = ex2(m_run[nt][1] - mu1);
            m_run[nt][0] = mn0;
            m_run[nt][1] = mn1;
            const float p0 = ex2(x0 - mu0), p1 = ex2(x1 - mu1);
            const float p2 = ex2(x2 - mu0), p3 = ex2(x3 - mu1);
            l_run[nt][0] = l_run[nt][0] * corr0 + (p0 + p2);
            l_run[nt][1] = l_run[nt][1] * corr1 + (p1 + p3);
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
              o[nt][mt][0] *= corr0;
              o[nt][mt][1] *= corr1;
              o[nt][mt][2] *= corr0;
              o[nt][mt][3] *= corr1;
            }
            pb[nt][0] = movmatrix_t(E::pack(p0, p1));
            pb[nt][1] = movmatrix_t(E::pack(p2, p3));
          }
          // O^T += V^T P^T : A = V^T via ldmatrix.trans
          {
            const int mq = lane >> 3;
            const int tok = t * 16 + (lane & 7) + 8 * (mq >> 1);
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
              const int ch = 2 * mt + (mq & 1);
              const uint32_t addr =
                  vs + (ch >> 3) * (BS * 128) + tok * 128 + ((((ch & 7) ^ (tok & 7))) << 4);
              uint32_t a[4];
              ldsm_x4_t(addr, a[0], a[1], a[2], a[3]);
#pragma unroll
              for (int nt = 0; nt < NT; ++nt) E::mma(o[nt][mt], a, pb[nt][0], pb[nt][1]);
            }
          }
        }
      }
      if (zeroed) fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    gbase += npg;

    // ---- merge the NCW warp states of this unit
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        float l = l_run[nt][j];
        l += __shfl_xor_sync(0xffffffffu, l, 4);
        l += __shfl_xor_sync(0xffffffffu, l, 8);
        l += __shfl_xor_sync(0xffffffffu, l, 16);
        l_run[nt][j] = l;
      }
    if (g == 0) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        comb_m[warp * HPC + nt * 8 + 2 * c] = m_run[nt][0];
        comb_m[warp * HPC + nt * 8 + 2 * c + 1] = m_run[nt][1];
        comb_l[warp * HPC + nt * 8 + 2 * c] = l_run[nt][0];
        comb_l[warp * HPC + nt * 8 + 2 * c + 1] = l_run[nt][1];
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) {
        float* r0 = comb_o + (warp * HPC + nt * 8 + 2 * c) * CSTRIDE + mt * 16 + g;
        r0[0] = o[nt][mt][0];
        r0[CSTRIDE] = o[nt][mt][1];
        r0[8] = o[nt][mt][2];
        r0[CSTRIDE + 8] = o[nt][mt][3];
      }
    __syncwarp();
    named_bar(1, NCW * 32);

    const int nsplit_seq =
        min(seq_splits(__ldg(p.context_lens + seq), p.tok_begin, p.tok_end, BS,
                       p.pages_per_split, direct_final),
            p.max_splits);
    const bool final_out = direct_final && nsplit_seq == 1;
    for (int idx = tid; idx < HPC * D; idx += NCW * 32) {
      const int hl = idx / D, dim = idx - hl * D;
      const int gh = hc * HPC + hl;
      if (gh >= G) continue;
      float M = NEG_INF;
#pragma unroll
      for (int w = 0; w < NCW; ++w) M = fmaxf(M, comb_m[w * HPC + hl]);
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int w = 0; w < NCW; ++w) {
        const float mw = comb_m[w * HPC + hl];
        const float wt = mw == NEG_INF ? 0.f : ex2(mw - M);
        L += comb_l[w * HPC + hl] * wt;
        O += comb_o[(w * HPC + hl) * CSTRIDE + dim] * wt;
      }
      const size_t row = static_cast<size_t>(seq) * p.num_heads + kvh * G + gh;
#ifdef FE_DEBUG_CHECKS
      if (row >= static_cast<size_t>(p.num_seqs) * p.num_heads ||
          (!final_out && (split < 0 || split >= p.max_splits || !p.part_o)) ||
          (final_out && !p.out)) {
        atomicOr(p.err, 1u << 9);
        continue;
      }
#endif
      if (final_out) {
        reinterpret_cast<T*>(p.out)[row * D + dim] = E::cvt(L > 0.f ? O / L : 0.f);
      } else {
        const size_t part = row * p.max_splits + split;
        p.part_o[part * D + dim] = O;
        if (dim == 0) {
          p.part_ml[part * 2 + 0] = M;
          p.part_ml[part * 2 + 1] = L;
        }
      }
    }
    __syncwarp();
    named_bar(2, NCW * 32);
  }
}

// ---------------------------------------------------------------------------
// Log-sum-exp merge of split partials. One warp per output row.
//   ctx mode (context_lens != nullptr): row = seq * H + h, its valid partials are the
//     seq_splits(...) first slots of [rows, max_splits]; rows with a single split
//     were already finalised by the decode kernel when skip_single is set.
//   all mode: every (rank, part) slot is a partial (possibly empty: l = 0).
template <int DMAX>
__global__ void __launch_bounds__(128) merge_kernel(const MergeParams mp) {
  constexpr float NEG_INF = -__builtin_huge_valf();
  constexpr int PER = DMAX / 32;
  const int D = mp.head_dim;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * 4 + warp;
  if (row >= mp.rows) return;
  int nparts, ranks;
  if (mp.context_lens) {
    const int seq = row / mp.heads;
    nparts = min(seq_splits(__ldg(mp.context_lens + seq), mp.tok_begin, mp.tok_end,
                            mp.block_size, mp.pages_per_split, false),
                 mp.parts_per_rank);
    if (mp.skip_single && nparts <= 1) return;
    ranks = 1;
  } else {
    nparts = mp.parts_per_rank;
    ranks = mp.ranks;
  }
  // pass 1: global max
  float M = NEG_INF;
  for (int rk = 0; rk < ranks; ++rk)
    for (int j = lane; j < nparts; j += 32) {
      const size_t slot = (static_cast<size_t>(rk) * mp.rows + row) * mp.parts_per_rank + j;
      const float l = mp.part_stats[slot * 2 + 1];
      if (l > 0.f) M = fmaxf(M, mp.part_stats[slot * 2]);
    }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
  float L = 0.f, acc[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) acc[k] = 0.f;
  for (int rk = 0; rk < ranks; ++rk)
    for (int j0 = 0; j0 < nparts; j0 += 32) {
      const int j = j0 + lane;
      float wt = 0.f, l = 0.f;
      size_t slot = 0;
      if (j < nparts) {
        slot = (static_cast<size_t>(rk) * mp.rows + row) * mp.parts_per_rank + j;
        l = mp.part_stats[slot * 2 + 1];
        if (l > 0.f) wt = ex2(mp.part_stats[slot * 2] - M);
      }
      L += l * wt;
      const int cnt = min(32, nparts - j0);
      for (int k = 0; k < cnt; ++k) {
        const float w = __shfl_sync(0xffffffffu, wt, k);
        if (w == 0.f) continue;
        const size_t sl = (static_cast<size_t>(rk) * mp.rows + row) * mp.parts_per_rank + j0 + k;
        const float* po = mp.part_out + sl * D;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          const int dim = lane + 32 * e;
          if (dim < D) acc[e] += po[dim] * w;
        }
      }
    }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
  const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
  for (int e = 0; e < PER; ++e) {
    const int dim = lane + 32 * e;
    if (dim >= D) continue;
    const size_t oi = static_cast<size_t>(row) * D + dim;
    if (mp.out_dtype == 0) {
      reinterpret_cast<float*>(mp.out)[oi] = acc[e] * inv;
    } else if (mp.out_dtype == 1) {
      reinterpret_cast<__nv_bfloat16*>(mp.out)[oi] = __float2bfloat16_rn(acc[e] * inv);
    } else if (mp.out_dtype == 3) {
      reinterpret_cast<half*>(mp.out)[oi] = __float2half_rn(acc[e] * inv);
    } else {
      reinterpret_cast<float*>(mp.out)[oi] = acc[e];
    }
  }
  if (mp.out_dtype == 2 && lane == 0) {
    mp.out_stats[static_cast<size_t>(row) * 2] = L > 0.f ? M : NEG_INF;
    mp.out_stats[static_cast<size_t>(row) * 2 + 1] = L;
  }
}

// ---------------------------------------------------------------------------
// host launch

template <typename T, int D, int BS, int NT>
static cudaError_t launch_cfg(const Params& p, const void* kc, const void* vc, long long kv_rows,
                              cudaStream_t stream) {
  constexpr int NCW = 4;
  // NCW consumer warps x DEPTH private stages each; ~64 KB of stages per CTA.
  constexpr int DEPTH = (D * BS <= 1024) ? 4 : (D * BS <= 2048) ? 2 : 1;
  constexpr int NSTAGE = NCW * DEPTH;
  static_assert(NSTAGE % NCW == 0, "stages must split evenly over the consumer warps");
  using C = Cfg<T, D, BS, NT, NCW, NSTAGE>;
  auto kern = paged_decode_kernel<T, D, BS, NT, NCW, NSTAGE>;
  const int smem = C::smem_bytes(p.num_seqs);
  cudaError_t e = ensure_smem_optin(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  CUtensorMap km, vm;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  e = encode_tma_2d_b16(&km, kc, bf16, D, kv_rows, D, 64, BS);
  if (e != cudaSuccess) return e;
  e = encode_tma_2d_b16(&vm, vc, bf16, D, kv_rows, D, 64, BS);
  if (e != cudaSuccess) return e;
  int occ = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, C::NTHREADS, smem);
  if (e != cudaSuccess) return e;
  if (occ < 1) return cudaErrorInvalidConfiguration;
  const int grid = sm_count() * occ;
  Params pp = p;
  pp.dbg_kv_rows = kv_rows;
  kern<<<grid, C::NTHREADS, smem, stream>>>(km, vm, pp);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_decode(const Params& p, int head_dim, int block_size, const void* kc,
                          const void* vc, long long kv_rows, int nt, cudaStream_t stream) {
#define FE_CASE(D_, BS_, NT_)                                                     \
  if (head_dim == D_ && block_size == BS_ && nt == NT_)                           \
    return launch_cfg<T, D_, BS_, NT_>(p, kc, vc, kv_rows, stream);
  FE_CASE(128, 16, 1)
  FE_CASE(128, 16, 2)
  FE_CASE(64, 16, 1)
  FE_CASE(64, 16, 2)
  FE_CASE(128, 32, 1)
  FE_CASE(128, 32, 2)
  FE_CASE(64, 32, 1)
  FE_CASE(64, 32, 2)
#undef FE_CASE
  return cudaErrorInvalidValue;
}

template cudaError_t launch_decode<__nv_bfloat16>(const Params&, int, int, const void*, const void*,
                                                  long long, int, cudaStream_t);
template cudaError_t launch_decode<half>(const Params&, int, int, const void*, const void*,
                                         long long, int, cudaStream_t);

cudaError_t launch_merge(const MergeParams& mp, int head_dim, cudaStream_t stream) {
  if (mp.rows <= 0) return cudaSuccess;
  const int grid = (mp.rows + 3) / 4;
  MergeParams m2 = mp;
  m2.head_dim = head_dim;
  if (head_dim < 1) return cudaErrorInvalidValue;
  if (head_dim <= 64) merge_kernel<64><<<grid, 128, 0, stream>>>(m2);
  else if (head_dim <= 128) merge_kernel<128><<<grid, 128, 0, stream>>>(m2);
  else if (head_dim <= 256) merge_kernel<256><<<grid, 128, 0, stream>>>(m2);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

}  // namespace paged
}  // namespace fe
