// FA2 online-softmax prefill forward on the 5th-generation tensor core (sm_100a).
//
// O = softmax(Q K^T * scale [+ causal mask]) V for bf16 / fp16 Q, K, V, O of shape
// [B, H, N|M, d] with fp32 accumulation -- the computation of the reference's
// launch_flash_attention_forward_fp16 (src/flash_attention.cu:350-524), causal mask
// top-left aligned (query row i sees keys j <= i, src/flash_attention.cu:224).
//
// One CTA (3 warpgroups) computes two 128-row query tiles (Q0, Q1) of one
// (batch, head). It is launched at 168 registers per thread; setmaxnreg then
// moves registers from warpgroup 2 (56 each) to the softmax warpgroups (224
// each): 384 x 168 = 256 x 224 + 128 x 56.
//  * warp 8 (TMA): loads Q0/Q1 once, then K_j and V_j tiles (128 keys x d) into
//    two-stage rings with 3-D TMA (128-byte swizzle; out-of-range rows zero-fill).
//  * warp 9 (MMA): allocates 512 tensor-memory columns
//    [S0 | S1 | O0 | O1] and, from one elected lane of the warp-wide loop, issues
//      S_t = Q_t K_j^T   (tcgen05.mma, A and B from shared memory)
//      O_t += P_t V_j    (tcgen05.mma, A = P_t from tensor memory, B = V_j)
//    in the order S0(0) S1(0) | PV0(j) S0(j+1) PV1(j) S1(j+1) | ..., so the tensor
//    core works on one tile while the other tile's softmax runs.
//  * warps 0-3 / 4-7 (softmax for Q0 / Q1): thread i owns row i of its tile. It
//    reads its S row from tensor memory, applies mask and scale, and updates the
//    running max m and sum l in the log2 domain. It writes P = 2^(s - m) as 16-bit
//    values over the first half of the S columns. O is rescaled in tensor memory
//    only when the row max grows by more than 2^8 (the stale max is exact for the
//    final O / l). At the end it reads O, divides by l and stores the row.
// Every wait is bounded (mbar_wait); on a timeout the CTA records an error, drains
// its TMA and MMA work, frees tensor memory and exits.
#include <algorithm>
#include <limits.h>

#include <type_traits>

#include "internal.h"
#include "prefill.h"
#include "ptx.cuh"
#include "tcgen05.cuh"

namespace fe {
namespace prefill {

constexpr float NEG_INF = -__builtin_huge_valf();
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when m grows > 2^8
// One exponential pair in every kPolyEvery goes to the FMA-pipe polynomial (0: none).
// With P handed to the MMA warp in two halves, all-MUFU is the fastest at every
// measured shape (config 2 and its 2-, 4- and 8-way head shards), so 0 is the default.
#ifndef FE_PREFILL_POLY_EVERY
#define FE_PREFILL_POLY_EVERY 0
#endif
constexpr int kPolyEvery = FE_PREFILL_POLY_EVERY;
// P of a key tile is handed to the MMA warp in kPChunks pieces (2 or 4; quarters
// measured 2-4% slower than halves on config 2).
#ifndef FE_PREFILL_P_CHUNKS
#define FE_PREFILL_P_CHUNKS 2
#endif
constexpr int kPChunks = FE_PREFILL_P_CHUNKS;
static_assert(kPChunks == 2 || kPChunks == 4, "P is handed over in halves or quarters");

#ifdef FE_PF_TIMELINE
// Per-CTA event times (globaltimer ns) of the last launch, profiling builds only:
// [0] entry, [1] set up (barriers, tensor memory, previous grid complete), [2] first S
// of tile 0 seen by the softmax, [3] softmax 0 done, [4] softmax 1 done, [5] epilogue 0
// done, [6] epilogue 1 done, [7] exit, [8] SM id, [9] query-tile pair, [10] (batch, head).
constexpr int kTimelineCtas = 4096;
__device__ unsigned long long g_pf_timeline[kTimelineCtas][12];
// Steps of the first 148 CTAs: [step][0/1] S of tile 0/1 seen, [2/3] P of tile 0/1 done,
// [4/5] row max of tile 0/1 known.
__device__ unsigned long long g_pf_steps[148][64][16];
#define FE_PST(j, slot) \
  do { if (blockIdx.x < 148 && (j) < 64) g_pf_steps[blockIdx.x][j][slot] = globaltimer_ns(); } while (0)
#define FE_PTL(slot, v) \
  do { if (blockIdx.x < kTimelineCtas) g_pf_timeline[blockIdx.x][slot] = (v); } while (0)
#else
#define FE_PTL(slot, v) do {} while (0)
#define FE_PST(j, slot) do {} while (0)
#endif

template <int D>
struct PCfg {
  static constexpr int BM = 128, BN = 128;
  static constexpr int HALVES = D / 64;
  static constexpr int TILE_BYTES = BM * D * 2;  // one 128-row tile of Q, K or V
  static constexpr int HALF_BYTES = BM * 128;    // one 64-column swizzle atom column
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + 2 * TILE_BYTES;
  static constexpr int V_OFF = K_OFF + 2 * TILE_BYTES;
  static constexpr int BAR_OFF = V_OFF + 2 * TILE_BYTES;
  static constexpr int NBARS = 17 + 2 * (kPChunks - 1);
  static constexpr int SMEM = 1024 + BAR_OFF + NBARS * 8 + 16;
  static constexpr int NTHREADS = 384;
};

struct PParams {
  void* out;
  int N, M, BH;
  int d_out;  // head dim of the tensors: D, or 32 when the D = 64 kernel runs d = 32
  int causal;
  float scale_log2;
  unsigned* err;
  int group;  // (batch, head)s per scheduling group (see the block mapping)
};

// 2^x on the FMA pipe: round x to the nearest integer n with the 1.5 * 2^23 trick,
// evaluate a degree-3 fit of 2^f on f in [-0.5, 0.5] (coefficients fitted for this
// kernel by iteratively reweighted least squares on relative error; max relative
// error 7.5e-5) and add n to the exponent field. x below -126 flushes to ~1e-38.
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;
  const int n = __float_as_int(t) - 0x4B400000;
  const float f = x - (t - 12582912.f);
  float q = fmaf(0.05517157f, f, 0.24261114f);
  q = fmaf(q, f, 0.693261f);
  q = fmaf(q, f, 0.99992806f);
  return __int_as_float(__float_as_int(q) + (n << 23));
}

// Paired fp32 arithmetic of sm_100 (two lanes per instruction) and the 3-input max.
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
#ifndef FE_PREFILL_SCALAR_PAIRS
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
#else  // profiling variant: the same arithmetic as two scalar instructions
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  float a0, a1, b0, b1, c0, c1;
  f2_split(a, a0, a1);
  f2_split(b, b0, b1);
  f2_split(c, c0, c1);
  return f2(fmaf(a0, b0, c0), fmaf(a1, b1, c1));
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  float a0, a1, b0, b1;
  f2_split(a, a0, a1);
  f2_split(b, b0, b1);
  return f2(a0 + b0, a1 + b1);
}
#endif
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

template <typename T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float lo, float hi) {
  return pack_bf16x2(lo, hi);
}
template <>
__device__ __forceinline__ uint32_t pack2<half>(float lo, float hi) {
  return pack_f16x2(lo, hi);
}

template <typename T, int D>
__global__ void __launch_bounds__(384, 1)
    fa_prefill_kernel(const __grid_constant__ CUtensorMap qmap,
                      const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const PParams p) {
  using C = PCfg<D>;
  constexpr int BM = C::BM, BN = C::BN, HALVES = C::HALVES;
  constexpr int TILE = C::TILE_BYTES, HALF = C::HALF_BYTES;
  constexpr bool kBF16 = std::is_same<T, __nv_bfloat16>::value;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2] per query tile
  uint64_t* p_full = bars + 11;  // [2]
  uint64_t* o_done = bars + 13;  // [2]
  uint64_t* drain = bars + 15;
  uint64_t* q_full1 = bars + 16;  // Q1 (Q0 completes on q_full)
  // [kPChunks - 1][2]: chunk c of P_t (keys c * BN / kPChunks ...) is in tensor memory;
  // the last chunk completes on p_full.
  uint64_t* p_part = bars + 17;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBARS);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) FE_PTL(0, globaltimer_ns());
#ifdef FE_PF_TIMELINE
  const long long clk_entry = clock64();
#endif
  // Block mapping: the (batch, head)s are cut into groups of p.group whose K/V fit in
  // L2 together. CTAs are dispatched group by group; inside a group, the query-tile
  // pairs go longest-first across all of its heads, so the causal work is scheduled
  // longest-first (few heads: one group, the whole grid) while the CTAs resident at
  // any time share the K/V of a few heads.
  const int npairs = (p.N + 2 * BM - 1) / (2 * BM);
  const long long L = blockIdx.x;
  const long long per_group = static_cast<long long>(p.group) * npairs;
  const int grp = static_cast<int>(L / per_group);
  const int bh0 = grp * p.group;
  const int gsz = min(p.group, p.BH - bh0);
  const int idx = static_cast<int>(L - grp * per_group);
  const int bh = bh0 + idx % gsz;
  const int pair = npairs - 1 - idx / gsz;
  int m0[2], nkv[2];
  const int kv_tiles = (p.M + BN - 1) / BN;
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    m0[t] = pair * 2 * BM + t * BM;
    if (m0[t] >= p.N) {
      nkv[t] = 0;
    } else if (p.causal) {
      const int last_row = min(p.N - 1, m0[t] + BM - 1);
      const int last_key = min(p.M - 1, last_row);
      nkv[t] = last_key / BN + 1;
    } else {
      nkv[t] = kv_tiles;
    }
  }
  const int nmax = max(nkv[0], nkv[1]);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_full1, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      for (int c = 0; c < kPChunks - 1; ++c) mbar_init(&p_part[c * 2 + i], 128);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == 9) {
    tc::tmem_alloc<512>(tmem_slot);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // Programmatic dependent launch: let the next kernel place its CTAs as ours retire,
  // and wait for the previous kernel's results before the first global access.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) {
    FE_PTL(1, globaltimer_ns());
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    FE_PTL(8, smid);
    FE_PTL(9, pair);
    FE_PTL(10, bh);
  }

  if (warp >= 8) {
   asm volatile("setmaxnreg.dec.sync.aligned.u32 56;\n" ::: "memory");
   if (warp == 8) {
    // ========================================================= TMA producer
    if (lane == 0 && nmax > 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      const uint64_t pol_keep = l2_policy_evict_last();   // K/V are re-read by other CTAs
      const uint64_t pol_once = l2_policy_evict_first();  // Q is read once
      // Q0, then K_0, then Q1: the first product S0(0) needs only Q0 and K_0.
      auto load_q = [&](int t) {
        uint64_t* bar = t == 0 ? q_full : q_full1;
        mbar_arrive_expect_tx(bar, TILE);
        for (int h = 0; h < HALVES; ++h)
          tma_load_3d(smem + C::Q_OFF + t * TILE + h * HALF, &qmap, h * 64, m0[t], bh, bar,
                      pol_once);
      };
      if (nkv[0] > 0) load_q(0);
      bool ok = true;
      int issued_k = 0, issued_v = 0;
      for (int j = 0; j < nmax && ok; ++j) {
        const int st = j & 1, rnd = j >> 1;
        if (rnd > 0 && !mbar_wait(&k_empty[st], (rnd - 1) & 1)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[st], TILE);
        for (int h = 0; h < HALVES; ++h)
          tma_load_3d(smem + C::K_OFF + st * TILE + h * HALF, &kmap, h * 64, j * BN, bh,
                      &k_full[st], pol_keep);
        ++issued_k;
        if (j == 0 && nkv[1] > 0) load_q(1);
        if (rnd > 0 && !mbar_wait(&v_empty[st], (rnd - 1) & 1)) { ok = false; break; }
        mbar_arrive_expect_tx(&v_full[st], TILE);
        for (int h = 0; h < HALVES; ++h)
          tma_load_3d(smem + C::V_OFF + st * TILE + h * HALF, &vmap, h * 64, j * BN, bh,
                      &v_full[st], pol_keep);
        ++issued_v;
      }
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
      // Drain: every bulk copy issued here has landed before the CTA can exit.
      if (nkv[0] > 0) mbar_wait(q_full, 0);
      if (nkv[1] > 0 && issued_k > 0) mbar_wait(q_full1, 0);
      for (int j = max(0, issued_k - 2); j < issued_k; ++j) mbar_wait(&k_full[j & 1], (j >> 1) & 1);
      for (int j = max(0, issued_v - 2); j < issued_v; ++j) mbar_wait(&v_full[j & 1], (j >> 1) & 1);
    }
  } else if (warp == 9) {
    // ========================================================= MMA issuer
    // The whole warp runs the issue loop and its waits, so its state stays warp-uniform;
    // one elected lane issues the MMAs and commits.
    if (nmax > 0) {
      const bool leader = elect_one();
      constexpr uint32_t idesc_qk = tc::idesc_f16(kBF16, BM, BN, false, false);
      constexpr uint32_t idesc_pv = tc::idesc_f16(kBF16, BM, D, false, true);
      const uint32_t sbase = smem_u32(smem);
      auto issue_s = [&](int t, int j) {
        const uint32_t qa = sbase + C::Q_OFF + t * TILE;
        const uint32_t kb = sbase + C::K_OFF + (j & 1) * TILE;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * HALF + (kk & 3) * 32;
          if (leader)
            tc::mma_ss(tmem + t * BN, tc::smem_desc_sw128(qa + off, 16, 1024),
                       tc::smem_desc_sw128(kb + off, 16, 1024), idesc_qk, kk > 0);
        }
        if (leader) tc::commit(&s_full[t]);
      };
      // P V in kPChunks pieces: each starts as soon as the softmax has stored that
      // chunk of P (p_part), while it computes the next ones (the last: p_full).
      auto issue_pv_part = [&](int t, int j, int c) {
        const uint32_t vb = sbase + C::V_OFF + (j & 1) * TILE;
        const uint32_t ptm = tmem + t * BN;              // P_t over the S_t columns
        const uint32_t otm = tmem + 2 * BN + t * D;
        constexpr int KK = BN / 16 / kPChunks;            // 16-key MMAs per chunk
#pragma unroll
        for (int k2 = 0; k2 < KK; ++k2) {
          const int kk = c * KK + k2;
          if (leader)
            tc::mma_ts(otm, ptm + kk * 8, tc::smem_desc_sw128(vb + kk * 16 * 128, HALF, 1024),
                       idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        if (c == kPChunks - 1 && leader) tc::commit(&o_done[t]);
      };
      auto issue_pv = [&](int t, int j) -> bool {
#pragma unroll
        for (int c = 0; c < kPChunks; ++c) {
          uint64_t* bar = c < kPChunks - 1 ? &p_part[c * 2 + t] : &p_full[t];
          if (!__all_sync(0xffffffffu, mbar_wait(bar, j & 1))) return false;
          tc::fence_after_sync();
          issue_pv_part(t, j, c);
        }
        return true;
      };
      // prologue: S0(0) as soon as Q0 and K_0 are in, then S1(0) once Q1 is
      bool ok = __all_sync(0xffffffffu,
                           (nkv[0] == 0 || mbar_wait(q_full, 0)) && mbar_wait(&k_full[0], 0));
      if (ok && nkv[0] > 0) {
        tc::fence_after_sync();
        issue_s(0, 0);
      }
      if (ok && nkv[1] > 0) {
        ok = __all_sync(0xffffffffu, mbar_wait(q_full1, 0));
        if (ok) {
          tc::fence_after_sync();
          issue_s(1, 0);
        }
      }
      if (ok && leader) tc::commit(&k_empty[0]);
      for (int j = 0; j < nmax && ok; ++j) {
        const int st = j & 1;
        if (!__all_sync(0xffffffffu, mbar_wait(&v_full[st], (j >> 1) & 1))) { ok = false; break; }
        const bool next_k = j + 1 < nmax;
        bool k_ready = false;
        if (j < nkv[0]) {
          if (!issue_pv(0, j)) { ok = false; break; }
          if (j + 1 < nkv[0]) {
            if (!__all_sync(0xffffffffu, mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1))) {
              ok = false;
              break;
            }
            k_ready = true;
            issue_s(0, j + 1);
          }
        }
        if (j < nkv[1]) {
          if (!issue_pv(1, j)) { ok = false; break; }
          if (j + 1 < nkv[1]) {
            if (!k_ready &&
                !__all_sync(0xffffffffu, mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1))) {
              ok = false;
              break;
            }
            k_ready = true;
            issue_s(1, j + 1);
          }
        }
        if (next_k) {
          if (!k_ready &&
              !__all_sync(0xffffffffu, mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1))) {
            ok = false;
            break;
          }
          if (leader) tc::commit(&k_empty[(j + 1) & 1]);
        }
        if (leader) tc::commit(&v_empty[st]);
      }
      if (!ok && leader) atomicOr(p.err, kErrWaitTimeout);
      // Drain: all MMAs issued by the leader have completed.
      if (leader) tc::commit(drain);
      mbar_wait(drain, 0);
    }
   }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 224;\n" ::: "memory");
    // ========================================================= softmax warpgroups
    const int t = warp >> 2;            // query tile of this warpgroup
    const int qw = warp & 3;            // lane quarter of tensor memory
    const int row = qw * 32 + lane;     // row within the tile
    const int r = m0[t] + row;          // query row
    const uint32_t lane_off = static_cast<uint32_t>(qw * 32) << 16;
    const uint32_t tS = tmem + lane_off + t * BN;
    const uint32_t tO = tmem + lane_off + 2 * BN + t * D;
    const float sl = p.scale_log2;
    float m_run = NEG_INF, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < nkv[t] && ok; ++j) {
      const bool got = mbar_wait(&s_full[t], j & 1);
      if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
      if (j == 0 && t == 0 && threadIdx.x == 0) FE_PTL(2, globaltimer_ns());
      if ((threadIdx.x & 127) == 0) FE_PST(j, t);
      tc::fence_after_sync();
      uint32_t u[BN];
#pragma unroll
      for (int c4 = 0; c4 < BN / 32; ++c4)
        tc::ld32(tS + c4 * 32, *reinterpret_cast<uint32_t(*)[32]>(&u[c4 * 32]));
      tc::wait_ld();
      if ((threadIdx.x & 127) == 0) FE_PST(j, 6 + t);
      const int c0 = j * BN;
      const bool need_mask = (p.causal && c0 + BN - 1 > m0[t]) || c0 + BN > p.M;
      if (need_mask) {
        const int lim = p.causal ? min(r + 1, p.M) : p.M;  // valid keys: c < lim
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (c0 + i >= lim) u[i] = __float_as_uint(NEG_INF);
      }
      // Row max: 3-input max over pairs, 8 independent chains (sl > 0, so
      // max(s) * sl = max(s * sl)).
      float m8[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) m8[i] = __uint_as_float(u[i]);
#pragma unroll
      for (int i = 8; i < BN; i += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k)
          m8[k] = max3(m8[k], __uint_as_float(u[i + 2 * k]), __uint_as_float(u[i + 2 * k + 1]));
      const float mx = max3(max3(m8[0], m8[1], m8[2]), max3(m8[3], m8[4], m8[5]),
                            fmaxf(m8[6], m8[7])) * sl;
      if ((threadIdx.x & 127) == 0) FE_PST(j, 4 + t);
      const float m_new = fmaxf(m_run, mx);
      const bool need = m_new > m_run + kRescaleThreshold;  // also true while m_run = -inf
      const float m_use = need ? m_new : m_run;
      const float mu = m_use == NEG_INF ? 0.f : m_use;
      const float corr = need ? ex2(m_run - mu) : 1.f;
      if (j > 0 && __any_sync(0xffffffffu, need)) {
        // O_t must hold P V of tile j-1 before it is rescaled, and be rescaled before
        // the first half of P V of tile j accumulates into it.
        const bool got_o = mbar_wait(&o_done[t], (j - 1) & 1);
        if (!__all_sync(0xffffffffu, got_o)) { ok = false; break; }
        tc::fence_after_sync();
#pragma unroll
        for (int c4 = 0; c4 < D / 32; ++c4) {
          uint32_t u[32];
          tc::ld32(tO + c4 * 32, u);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * corr);
          tc::st32(tO + c4 * 32, u);
        }
      }
      // p = 2^(s*sl - m): one FFMA each, then the MUFU ex2 (with kPolyEvery > 0, one
      // pair in every kPolyEvery uses a polynomial on the FMA pipe instead).
      // Each chunk of P is handed to the MMA warp as soon as it is stored.
      uint64_t acc2[4] = {0, 0, 0, 0};  // paired partial sums (0 bits = 0.0f, 0.0f)
      const uint64_t sl2 = f2(sl, sl), nmu2 = f2(-mu, -mu);
      if ((threadIdx.x & 127) == 0) FE_PST(j, 8 + t);
      constexpr int CK = BN / kPChunks;  // keys per chunk
#pragma unroll
      for (int c = 0; c < kPChunks; ++c) {
        uint32_t pk[CK / 2];
#pragma unroll
        for (int i = 0; i < CK / 2; ++i) {
          const uint64_t x2 = fma2(f2(__uint_as_float(u[c * CK + 2 * i]),
                                      __uint_as_float(u[c * CK + 2 * i + 1])),
                                   sl2, nmu2);
          float xa, xb;
          f2_split(x2, xa, xb);
          float a, b;
          if (kPolyEvery > 0 && (i % (kPolyEvery > 0 ? kPolyEvery : 1)) == kPolyEvery - 1) {
            a = ex2_poly(xa);
            b = ex2_poly(xb);
          } else {
            a = ex2(xa);
            b = ex2(xb);
          }
          acc2[i & 3] = add2(acc2[i & 3], f2(a, b));
          pk[i] = pack2<T>(a, b);
        }
        if constexpr (CK == 64) {
          tc::st32(tS + c * 32, pk);
        } else {
          tc::st16(tS + c * 16, pk);
        }
        tc::wait_st();
        if ((threadIdx.x & 127) == 0 && c == 0) FE_PST(j, 12 + t);
        if ((threadIdx.x & 127) == 0 && c == kPChunks - 1) FE_PST(j, 14 + t);
        tc::fence_before_sync();
        mbar_arrive(c < kPChunks - 1 ? &p_part[c * 2 + t] : &p_full[t]);
      }
      float sum = 0.f;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        float lo, hi;
        f2_split(acc2[k], lo, hi);
        sum += lo + hi;
      }
      l_run = l_run * corr + sum;
      m_run = m_use;
      if ((threadIdx.x & 127) == 0) FE_PST(j, 2 + t);
    }
    if ((threadIdx.x & 127) == 0) FE_PTL(3 + t, globaltimer_ns());
    if (!ok) {
      if (lane == 0) atomicOr(p.err, kErrWaitTimeout);
    } else if (nkv[t] > 0) {
      const bool got = mbar_wait(&o_done[t], (nkv[t] - 1) & 1);
      if (__all_sync(0xffffffffu, got)) {
        tc::fence_after_sync();
        const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
        T* orow = reinterpret_cast<T*>(p.out) + (static_cast<size_t>(bh) * p.N + r) * p.d_out;
#pragma unroll
        for (int c4 = 0; c4 < D / 32; ++c4) {
          if (c4 * 32 >= p.d_out) break;  // d = 32 on the D = 64 kernel
          uint32_t u[32];
          tc::ld32(tO + c4 * 32, u);
          tc::wait_ld();
          if (r < p.N) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 v;
              v.x = pack2<T>(__uint_as_float(u[i + 0]) * inv, __uint_as_float(u[i + 1]) * inv);
              v.y = pack2<T>(__uint_as_float(u[i + 2]) * inv, __uint_as_float(u[i + 3]) * inv);
              v.z = pack2<T>(__uint_as_float(u[i + 4]) * inv, __uint_as_float(u[i + 5]) * inv);
              v.w = pack2<T>(__uint_as_float(u[i + 6]) * inv, __uint_as_float(u[i + 7]) * inv);
              *reinterpret_cast<uint4*>(orow + c4 * 32 + i) = v;
            }
          }
        }
      } else if (lane == 0) {
        atomicOr(p.err, kErrWaitTimeout);
      }
    }
    if ((threadIdx.x & 127) == 0) FE_PTL(5 + t, globaltimer_ns());
  }

  tc::fence_before_sync();
  __syncthreads();
  if (threadIdx.x == 0) FE_PTL(7, globaltimer_ns());
#ifdef FE_PF_TIMELINE
  if (threadIdx.x == 0) FE_PTL(11, clock64() - clk_entry);
#endif
  if (warp == 9) {
    tc::fence_after_sync();
    tc::tmem_dealloc<512>(tmem);
  }
}

// ---------------------------------------------------------------------------
// d: the tensors' head dim, D or (D = 64) 32. For d = 32 the tensor maps span the 32
// real columns and load 64-column boxes: TMA fills columns 32..63 with zeros, so Q K^T
// and P V are those of d = 32 (the extra products are zero) and only 32 columns are
// stored.
template <typename T, int D>
static cudaError_t launch_d(const void* q, const void* k, const void* v, void* o, int B, int H,
                            int N, int M, int d, int causal, float scale, cudaStream_t st) {
  using C = PCfg<D>;
  auto kern = fa_prefill_kernel<T, D>;
  cudaError_t e = ensure_smem_optin(reinterpret_cast<const void*>(kern), C::SMEM);
  if (e != cudaSuccess) return e;
  const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
  const long long BH = static_cast<long long>(B) * H;
  CUtensorMap qm, km, vm;
  e = encode_tma_3d_b16(&qm, q, bf16, d, N, BH, 64, 128);
  if (e != cudaSuccess) return e;
  e = encode_tma_3d_b16(&km, k, bf16, d, M, BH, 64, 128);
  if (e != cudaSuccess) return e;
  e = encode_tma_3d_b16(&vm, v, bf16, d, M, BH, 64, 128);
  if (e != cudaSuccess) return e;
  PParams p;
  p.out = o;
  p.N = N;
  p.M = M;
  p.d_out = d;
  p.BH = static_cast<int>(BH);
  p.causal = causal;
  p.scale_log2 = scale * kLog2e;
  p.err = device_error_word();
  if (!p.err) return cudaErrorInitializationError;
  // heads per scheduling group: their K and V together within ~32 MB of L2
  const long long kv_bytes = 2LL * M * d * 2;
  p.group = static_cast<int>(std::max(1LL, std::min<long long>(BH, (32LL << 20) / kv_bytes)));
  const long long blocks = BH * ((N + 255) / 256);
  if (blocks > 0x7fffffffLL) return cudaErrorInvalidValue;
  dim3 grid(static_cast<unsigned>(blocks));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(C::NTHREADS);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, qm, km, vm, p);
}

cudaError_t launch_prefill(const void* q, const void* k, const void* v, void* o, int B, int H,
                           int N, int M, int d, int causal, float scale, bool is_bf16,
                           cudaStream_t stream) {
  if (!(d == 32 || d == 64 || d == 128)) return cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) |
       reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(o)) & 15)
    return cudaErrorInvalidValue;
  if (static_cast<long long>(B) * H > 65535) return cudaErrorInvalidValue;
  if (is_bf16) {
    if (d == 128)
      return launch_d<__nv_bfloat16, 128>(q, k, v, o, B, H, N, M, d, causal, scale, stream);
    return launch_d<__nv_bfloat16, 64>(q, k, v, o, B, H, N, M, d, causal, scale, stream);
  }
  if (d == 128) return launch_d<half, 128>(q, k, v, o, B, H, N, M, d, causal, scale, stream);
  return launch_d<half, 64>(q, k, v, o, B, H, N, M, d, causal, scale, stream);
}

}  // namespace prefill
}  // namespace fe

#ifdef FE_PF_TIMELINE
extern "C" int fe_debug_prefill_steps(unsigned long long* host) {
  return static_cast<int>(cudaMemcpyFromSymbol(host, fe::prefill::g_pf_steps,
                                               sizeof(fe::prefill::g_pf_steps)));
}
extern "C" int fe_debug_prefill_timeline(unsigned long long* host, int ctas) {
  if (ctas > fe::prefill::kTimelineCtas) ctas = fe::prefill::kTimelineCtas;
  return static_cast<int>(cudaMemcpyFromSymbol(host, fe::prefill::g_pf_timeline,
                                               sizeof(unsigned long long) * 12 * ctas));
}
#endif
