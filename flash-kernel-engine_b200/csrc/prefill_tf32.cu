// FA2 forward for fp32 Q, K, V, O on the 5th-generation tensor core (sm_100a), with
// fp32-class accuracy from three TF32 products per fp32 product ("3xTF32"): every
// operand x is split into hi = x with the low 13 mantissa bits cleared (exact in TF32)
// and lo = x - hi (exact in fp32), and a.b is formed as a_hi.b_hi + a_hi.b_lo +
// a_lo.b_hi with fp32 accumulation. The dropped a_lo.b_lo term and the TF32 rounding
// of lo are each about 2^-20 of |a.b|.
//
// It computes the reference's launch_flash_attention_forward_fp32
// (src/flash_attention.cu:111-345): O = softmax(Q K^T * scale [+ causal mask]) V over
// [B, H, N|M, d] fp32 tensors, causal mask top-left aligned (query row i sees keys
// j <= i, src/flash_attention.cu:224). Head dims 32, 64 and 128; the other head dims run
// on the CUDA-core kernel of attention_fp32.cu. Q hi and Q lo sit in tensor memory;
// shared memory holds raw Q and two K/V stages (key tile 64, 32 at d = 128).
//
// A CTA owns one 128-row query tile of one (batch, head) and the 64-key tiles
// t = split, split + nsplit, ... of it. The nsplit CTAs of a row tile form a thread-block
// cluster and merge their (m, l, O) partials through distributed shared memory (the
// log-sum-exp combine of src/flash_decoding.cu:151-223): each CTA stores its partial
// rows into the CTA that owns them, which merges them from its own shared memory.
//  * warp 4 (TMA): Q once, then K_j and V_j (3-D TMA, 128-byte swizzle; rows past N or
//    M read as zeros): tiles 0 and 1 straight into the two stages, later tiles into a
//    landing buffer as soon as the split warps have read the previous one.
//  * warps 6-9 (split): write each landed K / V tile into its stage as hi and lo; V is
//    transposed on the way (V^T hi / lo), the K-major B operand of the P V product.
//    Keys are split first (K_0, K_1, V_0, V_1, then K and V of each later tile), each
//    released on its own barrier, so S_j waits only for K_j.
//    The softmax warps split Q the same way before their first S tile, each its row,
//    into tensor memory.
//  * warp 5 (MMA): allocates tensor memory [S0 | S1 | PL0 | PL1 | O | Qlo | Qhi] and,
//    from one thread, issues
//      S_j = Qhi Khi^T + Qhi Klo^T + Qlo Khi^T   (kind::tf32, A = Q from tensor memory)
//      O  += Phi Vhi + Phi Vlo + Plo Vhi         (A = P from tensor memory, B = V^T)
//    with S double-buffered, so S_{j+1} is computed while the softmax of tile j runs.
//  * warps 0-3 (softmax): thread i owns query row i. It reads S_j, applies mask and
//    scale, updates the running max m and sum l in the log2 domain, and writes
//    P_hi = hi(2^(s - m)) over S_j and P_lo into PL_j. O is rescaled in tensor memory
//    only when the row max grows by more than 2^8 (the stale max is exact for O / l).
// Every wait is bounded (mbar_wait); on a timeout the CTA records an error, drains its
// copies and MMAs, frees tensor memory and exits.
#include <stdlib.h>

#include "fp32_kernels.h"
#include "internal.h"
#include "ptx.cuh"
#include "tcgen05.cuh"

namespace fe {
namespace tf32 {

constexpr float NEG_INF = -__builtin_huge_valf();
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O when m grows > 2^8

#ifdef FE_TF32_TIMELINE
// Per-CTA event times (globaltimer ns) of the last launch, profiling builds only:
// [0] entry, [1] set up, [2] Q landed, [3] K_0 split, [4] S_0 seen, [5] P_0 done,
// [6] S_1 seen, [7] P_1 done, [8] final O, [9] cluster barrier 1 passed, [10] partials
// pushed, [11] cluster barrier 2 passed, [12] rows stored, [13] SM id, [14] clock64
// cycles entry -> [12], [15] MMA thread saw P_0, [16] PV_0 issued, [17] saw P_1, [18] PV_1
// issued, [19] S_1 issued, [20] V_1 split, [21] Q split, [22] drain done.
__device__ unsigned long long g_tf32_timeline[1024][24];
#define FE_TTL(slot, v) \
  do { if (blockIdx.x + blockIdx.y * gridDim.x < 1024) \
         g_tf32_timeline[blockIdx.x + blockIdx.y * gridDim.x][slot] = (v); } while (0)
#else
#define FE_TTL(slot, v) do {} while (0)
#endif

template <int D>
struct TCfg {
  // Q hi and Q lo live in tensor memory (the A operands of the S passes); shared memory
  // holds raw Q as landed and two K/V stages. d = 128: two stages of 64 keys do not fit
  // shared memory (nor tensor memory), so the key tile is 32.
  static constexpr int BM = 128, BN = D > 64 ? 32 : 64;
  static constexpr int HALVES = D / 32;  // 128-byte swizzle atom columns along d
  static constexpr int QH = BM * 128;    // bytes of one Q atom column
  static constexpr int KH = BN * 128;    // bytes of one K or V atom column
  static constexpr int VTH = D * 128;    // bytes of one V^T atom column (D rows)
  static constexpr int Q_BYTES = BM * D * 4;
  static constexpr int KV_BYTES = BN * D * 4;
  static constexpr int Q_RAW = 0;  // raw Q as landed by TMA
  static constexpr int K_HI = 0, K_LO = KV_BYTES, V_HI = 2 * KV_BYTES, V_LO = 3 * KV_BYTES;
  static constexpr int STAGE = 4 * KV_BYTES;
  static constexpr int ST_OFF = Q_BYTES;  // stage s at ST_OFF + s*STAGE
  // Landing buffer of raw K and V for key tiles 2, 3, ...: their copies need only the
  // previous tile's raw data to have been read, not a free stage.
  static constexpr int L_OFF = ST_OFF + 2 * STAGE, L_K = 0, L_V = KV_BYTES;
  static constexpr int BAR_OFF = L_OFF + 2 * KV_BYTES;
  static constexpr int NBARS = 19;
  static constexpr int BAR_END = BAR_OFF + NBARS * 8 + 32;  // + tensor-memory slot, flags
  // Receive buffer of the cluster merge ([BM] rows of D floats, then m and l): a region of
  // its own where it fits (d <= 64), so partners push into it without waiting for this
  // CTA's stage buffers to be free; else (d = 128) the stage buffers.
  static constexpr int RECV_BYTES = (BM * D + 2 * BM) * 4;
  static constexpr int RECV_OWN_OFF = (BAR_END + 127) / 128 * 128;
  static constexpr bool RECV_OWN = 1024 + RECV_OWN_OFF + RECV_BYTES <= 232448;
  static constexpr int RECV_OFF = RECV_OWN ? RECV_OWN_OFF : ST_OFF;
  static_assert(RECV_OWN || RECV_BYTES <= 2 * STAGE, "combine buffer");
  static constexpr int SMEM = 1024 + (RECV_OWN ? RECV_OWN_OFF + RECV_BYTES : BAR_END);
  // Dynamic shared memory requested at launch: enough that two CTAs never share an SM.
  // Each allocates all 512 tensor-memory columns, and two on one SM in one cluster would
  // wait on each other (one in tcgen05.alloc, the other at the cluster barrier).
  static constexpr int SMEM_LAUNCH = SMEM > 120 * 1024 ? SMEM : 120 * 1024;
  static constexpr int NTHREADS = 320;
  // tensor-memory columns: S / P_hi double-buffered, P_lo double-buffered, O, Q lo, Q hi
  static constexpr int T_S = 0, T_PL = 2 * BN, T_O = 4 * BN, T_QL = T_O + D, T_QH = T_QL + D;
  static_assert(T_QH + D <= 512, "tensor memory");
  static_assert(SMEM <= 232448, "shared memory");
};

struct TParams {
  float* out;
  int N, M;
  int causal;
  int nsplit;
  float scale_log2;
  unsigned* err;
};

__device__ __forceinline__ float tf32_hi(float x) {
  return __uint_as_float(__float_as_uint(x) & 0xFFFFE000u);
}

// The hi / lo split of a tile, by NT threads, in two phases: all loads (into registers)
// before the first store, so the source may be the destination (in place) or a buffer
// that is released between the phases. hi = x with the low 13 mantissa bits cleared,
// lo = x - hi; the layout is kept (the transform is elementwise).
template <int BYTES, int NT>
__device__ __forceinline__ void load_tile(const uint8_t* src, float4 (&x)[BYTES / 16 / NT],
                                          int tid) {
  static_assert((BYTES / 16 / NT) * 16 * NT == BYTES, "tile split");
  const float4* h = reinterpret_cast<const float4*>(src);
#pragma unroll
  for (int j = 0; j < BYTES / 16 / NT; ++j) x[j] = h[tid + j * NT];
}
template <int BYTES, int NT>
__device__ __forceinline__ void store_split(const float4 (&x)[BYTES / 16 / NT], uint8_t* hi_base,
                                            uint8_t* lo_base, int tid) {
  float4* h = reinterpret_cast<float4*>(hi_base);
  float4* l = reinterpret_cast<float4*>(lo_base);
#pragma unroll
  for (int j = 0; j < BYTES / 16 / NT; ++j) {
    const float4 a =
        make_float4(tf32_hi(x[j].x), tf32_hi(x[j].y), tf32_hi(x[j].z), tf32_hi(x[j].w));
    h[tid + j * NT] = a;
    l[tid + j * NT] = make_float4(x[j].x - a.x, x[j].y - a.y, x[j].z - a.z, x[j].w - a.w);
  }
}
// hi in place, lo at lo_base.
template <int BYTES, int NT>
__device__ __forceinline__ void split_tile(uint8_t* hi_base, uint8_t* lo_base, int tid) {
  float4 x[BYTES / 16 / NT];
  load_tile<BYTES, NT>(hi_base, x, tid);
  store_split<BYTES, NT>(x, hi_base, lo_base, tid);
}

// V as loaded ([BN keys] rows of 128-byte swizzle atoms, 32 floats of d per atom column)
// -> V^T hi and V^T lo: [D] rows of keys in the same swizzle, the K-major B operand of
// O += P V. (A TF32 B operand in MN-major form, V as loaded, produced no result on this
// hardware.) Lanes take consecutive keys of one 4-float chunk of d.
template <int D, int BN>
constexpr int v_per() { return BN * (D / 4) / 128; }  // float4 chunks per split thread
template <int D, int BN>
__device__ __forceinline__ void load_v(const uint8_t* v, float4 (&x)[v_per<D, BN>()], int tid) {
#pragma unroll
  for (int j = 0; j < v_per<D, BN>(); ++j) {
    const int i = tid + j * 128;
    const int key = i % BN, dc = i / BN;
    x[j] = *reinterpret_cast<const float4*>(v + (dc >> 3) * (BN * 128) + key * 128 +
                                            (((dc & 7) ^ (key & 7)) << 4));
  }
}
template <int D, int BN>
__device__ __forceinline__ void store_vt(const float4 (&x)[v_per<D, BN>()], uint8_t* vt_hi,
                                         uint8_t* vt_lo, int tid) {
#pragma unroll
  for (int j = 0; j < v_per<D, BN>(); ++j) {
    const int i = tid + j * 128;
    const int key = i % BN, dc = i / BN;
    const float xs[4] = {x[j].x, x[j].y, x[j].z, x[j].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = dc * 4 + e;
      const int off = (key >> 5) * (D * 128) + d * 128 + ((((key & 31) >> 2) ^ (d & 7)) << 4) +
                      (key & 3) * 4;
      const float h = tf32_hi(xs[e]);
      *reinterpret_cast<float*>(vt_hi + off) = h;
      *reinterpret_cast<float*>(vt_lo + off) = xs[e] - h;
    }
  }
}
// In place: V^T hi over V, V^T lo at vt_lo. The 128 split threads read all of V into
// registers before any of them overwrites it (named barrier 1).
template <int D, int BN>
__device__ __forceinline__ void split_transpose_v(uint8_t* v, uint8_t* vt_lo, int tid) {
  float4 x[v_per<D, BN>()];
  load_v<D, BN>(v, x, tid);
  asm volatile("bar.sync 1, 128;" ::: "memory");
  store_vt<D, BN>(x, v, vt_lo, tid);
}

// AND of `pred` over the 128 split threads (named barrier 1); every one of them calls it.
__device__ __forceinline__ bool split_group_all(bool pred) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 128, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(pred ? 1 : 0)
      : "memory");
  return r != 0;
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
// Every thread of every CTA of the cluster arrives; shared-memory writes before it
// (local and remote) are visible to the whole cluster after it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_f32(uint32_t addr, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, float x, float y, float z, float w) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(x), "f"(y),
               "f"(z), "f"(w)
               : "memory");
}

template <int D>
__global__ void __launch_bounds__(320, 1)
    fa_tf32_kernel(const __grid_constant__ CUtensorMap qmap,
                   const __grid_constant__ CUtensorMap kmap,
                   const __grid_constant__ CUtensorMap vmap, const TParams p) {
  using C = TCfg<D>;
  constexpr int BM = C::BM, BN = C::BN, HALVES = C::HALVES;
#ifdef FE_TF32_TIMELINE
  const long long clk0 = clock64();
  if (threadIdx.x == 0) {
    FE_TTL(0, globaltimer_ns());
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    FE_TTL(13, smid);
  }
#endif

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* q_ready = bars + 1;
  uint64_t* kv_full = bars + 2;   // [2] TMA landed
  uint64_t* k_ready = bars + 4;   // [2] K_j split into hi / lo (S_j can start)
  uint64_t* kv_empty = bars + 6;  // [2] MMAs done with the stage
  uint64_t* s_full = bars + 8;    // [2] S_j in tensor memory
  uint64_t* p_full = bars + 10;   // [2] P_j in tensor memory
  uint64_t* o_done = bars + 12;   // [2] P_j V_j accumulated
  uint64_t* drain = bars + 14;
  uint64_t* l_full = bars + 15;   // landing buffer holds the next tile's raw K / V
  uint64_t* l_empty = bars + 16;  // the split warps have read it
  uint64_t* v_ready = bars + 17;  // [2] V_j split and transposed (P_j V_j can start)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + C::NBARS);
  int* o_valid = reinterpret_cast<int*>(tmem_slot + 1);  // [4] softmax warp w read its final O

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nsplit = p.nsplit;
  const int split = nsplit > 1 ? static_cast<int>(cluster_rank()) : 0;
  const int bh = blockIdx.y;
  const int m0 = (blockIdx.x / nsplit) * BM;
  int ntiles = (p.M + BN - 1) / BN;
  if (p.causal && p.M > 0) ntiles = min(p.M - 1, min(p.N - 1, m0 + BM - 1)) / BN + 1;
  const int nloc = ntiles > split ? (ntiles - split + nsplit - 1) / nsplit : 0;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_ready, 128);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&k_ready[i], 128);
      mbar_init(&v_ready[i], 128);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(drain, 1);
    mbar_init(l_full, 1);
    mbar_init(l_empty, 128);
    fence_mbar_init();
  }
  if (warp == 5) {
    tc::tmem_alloc<512>(tmem_slot);
    tc::tmem_relinquish();
  }
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *tmem_slot;
  // Cluster merge into a receive buffer of its own: this arrive, waited on just before
  // the first remote store, makes sure every CTA of the cluster is running by then.
  if (C::RECV_OWN && nsplit > 1)
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
  // Programmatic dependent launch: let the next kernel place its CTAs as ours retire,
  // and wait for the previous kernel's results before the first global access.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (threadIdx.x == 0) FE_TTL(1, globaltimer_ns());

  float m_run = NEG_INF, l_run = 0.f;  // softmax threads: this row's running max and sum
  bool have_o = false;                 // softmax threads: O in tensor memory is final

  if (warp == 4) {
    // ========================================================= TMA producer
    if (lane == 0 && nloc > 0) {
      prefetch_tensormap(&qmap);
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
      const uint64_t pol_keep = l2_policy_evict_last();   // K/V are re-read by other CTAs
      const uint64_t pol_once = l2_policy_evict_first();  // Q is read once
      mbar_arrive_expect_tx(q_full, C::Q_BYTES);
      for (int h = 0; h < HALVES; ++h)
        tma_load_3d(smem + C::Q_RAW + h * C::QH, &qmap, h * 32, m0, bh, q_full, pol_once);
      bool ok = true;
      int issued = 0;
      // Tiles 0 and 1 land in their stages; later tiles in the landing buffer, each once
      // the split warps have read the one before (l_empty).
      for (int it = 0; it < nloc; ++it) {
        const int key0 = (split + it * nsplit) * BN;
        uint8_t *kdst, *vdst;
        uint64_t* bar;
        if (it < 2) {
          uint8_t* sb = smem + C::ST_OFF + it * C::STAGE;
          kdst = sb + C::K_HI;
          vdst = sb + C::V_HI;
          bar = &kv_full[it];
        } else {
          if (it > 2 && !mbar_wait(l_empty, (it - 3) & 1)) { ok = false; break; }
          kdst = smem + C::L_OFF + C::L_K;
          vdst = smem + C::L_OFF + C::L_V;
          bar = l_full;
        }
        mbar_arrive_expect_tx(bar, 2 * C::KV_BYTES);
        for (int h = 0; h < HALVES; ++h)
          tma_load_3d(kdst + h * C::KH, &kmap, h * 32, key0, bh, bar, pol_keep);
        for (int h = 0; h < HALVES; ++h)
          tma_load_3d(vdst + h * C::KH, &vmap, h * 32, key0, bh, bar, pol_keep);
        ++issued;
      }
      if (!ok) atomicOr(p.err, kErrWaitTimeout);
      // Drain: every bulk copy issued here has landed before the CTA can exit.
      mbar_wait(q_full, 0);
      for (int it = 0; it < min(issued, 2); ++it) mbar_wait(&kv_full[it], 0);
      if (issued > 2) mbar_wait(l_full, (issued - 3) & 1);
    }
  } else if (warp == 5) {
    // ========================================================= MMA issuer
    // The whole warp runs the issue loop and its waits, so its state stays warp-uniform;
    // one elected lane issues the MMAs and commits.
    if (nloc > 0) {
      const bool leader = elect_one();
      constexpr uint32_t idesc_qk = tc::idesc_tf32(BM, BN, false, false);
      constexpr uint32_t idesc_pv = tc::idesc_tf32(BM, D, false, false);
      const uint32_t sbase = smem_u32(smem);
      auto issue_s = [&](int it) {
        const int b = it & 1;
        const uint32_t kbase = sbase + C::ST_OFF + b * C::STAGE;
#pragma unroll
        for (int pass = 0; pass < 3; ++pass) {
          const uint32_t qa = tmem + (pass == 2 ? C::T_QL : C::T_QH);  // A from tensor memory
          const uint32_t kb = kbase + (pass == 1 ? C::K_LO : C::K_HI);
#pragma unroll
          for (int kk = 0; kk < D / 8; ++kk) {
            const uint32_t koff = (kk >> 2) * C::KH + (kk & 3) * 32;
            if (leader)
              tc::mma_ts_tf32(tmem + C::T_S + b * BN, qa + kk * 8,
                              tc::smem_desc_sw128(kb + koff, 16, 1024), idesc_qk,
                              (pass > 0 || kk > 0) ? 1u : 0u);
          }
        }
        if (leader) tc::commit(&s_full[b]);
      };
      auto issue_pv = [&](int it) {
        const int b = it & 1;
        const uint32_t vbase = sbase + C::ST_OFF + b * C::STAGE;
#pragma unroll
        for (int pass = 0; pass < 3; ++pass) {
          const uint32_t pa = tmem + (pass == 2 ? C::T_PL : C::T_S) + b * BN;
          const uint32_t vb = vbase + (pass == 1 ? C::V_LO : C::V_HI);
#pragma unroll
          for (int kk = 0; kk < BN / 8; ++kk)
            if (leader)
              tc::mma_ts_tf32(tmem + C::T_O, pa + kk * 8,
                              tc::smem_desc_sw128(vb + (kk >> 2) * C::VTH + (kk & 3) * 32, 16,
                                                  1024),
                              idesc_pv, (it > 0 || pass > 0 || kk > 0) ? 1u : 0u);
        }
        if (leader) {
          tc::commit(&o_done[b]);
          tc::commit(&kv_empty[b]);
        }
      };
      // S_{it+1} goes in before P_it V_it, so the tensor core computes it while the
      // softmax of tile it runs. MMAs from this thread execute in issue order, so
      // S_{it+2} overwrites P_it only after P_it V_it has read it.
      bool ok = __all_sync(0xffffffffu, mbar_wait(q_ready, 0) && mbar_wait(&k_ready[0], 0));
      if (ok) {
        tc::fence_after_sync();
        issue_s(0);
      }
      for (int it = 0; it < nloc && ok; ++it) {
        if (it + 1 < nloc) {
          if (!__all_sync(0xffffffffu, mbar_wait(&k_ready[(it + 1) & 1], ((it + 1) >> 1) & 1))) {
            ok = false;
            break;
          }
          tc::fence_after_sync();
          issue_s(it + 1);
          if (it == 0 && leader) FE_TTL(19, globaltimer_ns());
        }
        if (!__all_sync(0xffffffffu, mbar_wait(&p_full[it & 1], (it >> 1) & 1) &&
                                         mbar_wait(&v_ready[it & 1], (it >> 1) & 1))) {
          ok = false;
          break;
        }
        if (it < 2 && leader) FE_TTL(15 + 2 * it, globaltimer_ns());
        tc::fence_after_sync();
        issue_pv(it);
        if (it < 2 && leader) FE_TTL(16 + 2 * it, globaltimer_ns());
      }
      if (!ok && leader) atomicOr(p.err, kErrWaitTimeout);
      // Drain: all MMAs issued by the leader have completed.
      if (leader) tc::commit(drain);
      mbar_wait(drain, 0);
      if (leader) FE_TTL(22, globaltimer_ns());
    }
  } else if (warp >= 6) {
    // ========================================================= hi / lo split
    const int sid = threadIdx.x - 192;
    if (nloc > 0) {
      // The 128 split threads meet on named barrier 1 (inside split_transpose_v), so they
      // take every go / give-up decision together: a wait result is AND-reduced first.
      // Tiles 0 and 1 land in their stages and are split in place, keys first (K_0, K_1,
      // then V_0, V_1): S_0 and S_1 need only the keys, and V_0 is needed only once the
      // softmax of tile 0 is done.
      bool ok = true;
      const int nfirst = min(nloc, 2);
      for (int it = 0; it < nfirst && ok; ++it) {
        uint8_t* sb = smem + C::ST_OFF + it * C::STAGE;
        if (!split_group_all(mbar_wait(&kv_full[it], 0))) { ok = false; break; }
        split_tile<C::KV_BYTES, 128>(sb + C::K_HI, sb + C::K_LO, sid);
        fence_proxy_async_smem();
        mbar_arrive(&k_ready[it]);
        if (sid == 0 && it == 0) FE_TTL(3, globaltimer_ns());
      }
      for (int it = 0; it < nfirst && ok; ++it) {
        uint8_t* sb = smem + C::ST_OFF + it * C::STAGE;
        split_transpose_v<D, BN>(sb + C::V_HI, sb + C::V_LO, sid);
        fence_proxy_async_smem();
        mbar_arrive(&v_ready[it]);
        if (sid == 0 && it == 1) FE_TTL(20, globaltimer_ns());
      }
      for (int it = 2; it < nloc && ok; ++it) {
        // raw tile in the landing buffer; the stage is free once P V of tile it-2 is done
        const int st = it & 1;
        uint8_t* sb = smem + C::ST_OFF + st * C::STAGE;
        const bool got = mbar_wait(l_full, (it - 2) & 1) &&
                         mbar_wait(&kv_empty[st], ((it >> 1) - 1) & 1);
        if (!split_group_all(got)) { ok = false; break; }
        float4 kx[C::KV_BYTES / 16 / 128];
        float4 vx[v_per<D, BN>()];
        load_tile<C::KV_BYTES, 128>(smem + C::L_OFF + C::L_K, kx, sid);
        load_v<D, BN>(smem + C::L_OFF + C::L_V, vx, sid);
        mbar_arrive(l_empty);  // this thread's reads of the landing buffer are done
        store_split<C::KV_BYTES, 128>(kx, sb + C::K_HI, sb + C::K_LO, sid);
        fence_proxy_async_smem();
        mbar_arrive(&k_ready[st]);
        store_vt<D, BN>(vx, sb + C::V_HI, sb + C::V_LO, sid);
        fence_proxy_async_smem();
        mbar_arrive(&v_ready[st]);
      }
      if (!ok && sid == 0) atomicOr(p.err, kErrWaitTimeout);
    }
  } else {
    // ========================================================= softmax (warps 0-3)
    const int row = warp * 32 + lane;  // row within the tile = tensor-memory lane
    const int r = m0 + row;
    const uint32_t lane_off = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t tS = tmem + lane_off + C::T_S;
    const uint32_t tPL = tmem + lane_off + C::T_PL;
    const uint32_t tO = tmem + lane_off + C::T_O;
    const float sl = p.scale_log2;
    const int lim = p.causal ? min(r + 1, p.M) : p.M;  // valid keys: c < lim
    bool ok = true;
    // Q is split here (these warps are idle until S_0) while warps 6-9 split K_0 / V_0.
    if (nloc > 0) {
      ok = __all_sync(0xffffffffu, mbar_wait(q_full, 0));
      if (threadIdx.x == 0) FE_TTL(2, globaltimer_ns());
      if (ok) {
        // this thread's row of raw Q -> hi and lo in tensor-memory columns T_QH / T_QL + d,
        // 32 columns at a time, hi stored before lo is formed (32 values live, not 64)
#pragma unroll
        for (int a = 0; a < HALVES; ++a) {
          uint32_t x[32];
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 v4 = *reinterpret_cast<const float4*>(
                smem + C::Q_RAW + a * C::QH + row * 128 + ((c ^ (row & 7)) << 4));
            x[c * 4 + 0] = __float_as_uint(v4.x);
            x[c * 4 + 1] = __float_as_uint(v4.y);
            x[c * 4 + 2] = __float_as_uint(v4.z);
            x[c * 4 + 3] = __float_as_uint(v4.w);
          }
          uint32_t h[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) h[e] = x[e] & 0xFFFFE000u;  // tf32_hi
          tc::st32(tmem + lane_off + C::T_QH + a * 32, h);
#pragma unroll
          for (int e = 0; e < 32; ++e)
            x[e] = __float_as_uint(__uint_as_float(x[e]) - __uint_as_float(x[e] & 0xFFFFE000u));
          tc::st32(tmem + lane_off + C::T_QL + a * 32, x);
        }
        tc::wait_st();
        tc::fence_before_sync();
        mbar_arrive(q_ready);
        if (threadIdx.x == 0) FE_TTL(21, globaltimer_ns());
      }
    }
    for (int it = 0; it < nloc && ok; ++it) {
      const int b = it & 1;
      const bool got = mbar_wait(&s_full[b], (it >> 1) & 1);
      if (!__all_sync(0xffffffffu, got)) { ok = false; break; }
      if (threadIdx.x == 0 && it < 2) FE_TTL(4 + 2 * it, globaltimer_ns());
      tc::fence_after_sync();
      uint32_t u[BN];
#pragma unroll
      for (int c = 0; c < BN / 32; ++c)
        tc::ld32(tS + b * BN + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&u[c * 32]));
      tc::wait_ld();
      const int c0 = (split + it * nsplit) * BN;
      if (c0 + BN > lim) {
#pragma unroll
        for (int i = 0; i < BN; ++i)
          if (c0 + i >= lim) u[i] = __float_as_uint(NEG_INF);
      }
      float m4[4] = {NEG_INF, NEG_INF, NEG_INF, NEG_INF};
#pragma unroll
      for (int i = 0; i < BN; ++i) m4[i & 3] = fmaxf(m4[i & 3], __uint_as_float(u[i]));
      const float mx = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3])) * sl;
      const float m_new = fmaxf(m_run, mx);
      const bool need = m_new > m_run + kRescaleThreshold;  // also true while m_run = -inf
      const float m_use = need ? m_new : m_run;
      const float mu = m_use == NEG_INF ? 0.f : m_use;
      const float corr = need ? ex2(m_run - mu) : 1.f;
      float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t ph[32], pl[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float x = ex2(fmaf(__uint_as_float(u[c * 32 + i]), sl, -mu));
          s4[i & 3] += x;
          const float h = tf32_hi(x);
          ph[i] = __float_as_uint(h);
          pl[i] = __float_as_uint(x - h);
        }
        tc::st32(tS + b * BN + c * 32, ph);
        tc::st32(tPL + b * BN + c * 32, pl);
      }
      l_run = l_run * corr + ((s4[0] + s4[1]) + (s4[2] + s4[3]));
      m_run = m_use;
      if (it > 0 && __any_sync(0xffffffffu, need)) {
        // O must hold P V of tile it-1 before it is rescaled.
        const bool got_o = mbar_wait(&o_done[(it - 1) & 1], ((it - 1) >> 1) & 1);
        if (!__all_sync(0xffffffffu, got_o)) { ok = false; break; }
        tc::fence_after_sync();
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t w[32];
          tc::ld32(tO + c * 32, w);
          tc::wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = __float_as_uint(__uint_as_float(w[i]) * corr);
          tc::st32(tO + c * 32, w);
        }
      }
      tc::wait_st();
      tc::fence_before_sync();
      mbar_arrive(&p_full[b]);
      if (threadIdx.x == 0 && it < 2) FE_TTL(5 + 2 * it, globaltimer_ns());
    }
    if (!ok) {
      if (lane == 0) atomicOr(p.err, kErrWaitTimeout);
    } else if (nloc > 0) {
      const bool got = mbar_wait(&o_done[(nloc - 1) & 1], ((nloc - 1) >> 1) & 1);
      have_o = __all_sync(0xffffffffu, got);
      if (threadIdx.x == 0) FE_TTL(8, globaltimer_ns());
      if (have_o) {
        tc::fence_after_sync();
      } else if (lane == 0) {
        atomicOr(p.err, kErrWaitTimeout);
      }
    }
    if (!have_o) {
      m_run = NEG_INF;
      l_run = 0.f;
    }
    if (lane == 0) o_valid[warp] = have_o ? 1 : 0;
    if (nsplit == 1) {
      // O / l straight from tensor memory, 32 columns at a time
      const float inv = l_run > 0.f ? 1.f / l_run : 0.f;
      float* orow = p.out + (static_cast<size_t>(bh) * p.N + r) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t w[32];
        if (have_o) {
          tc::ld32(tO + c * 32, w);
          tc::wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) w[i] = 0u;
        }
        if (r < p.N) {
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<float4*>(orow + c * 32 + i) =
                make_float4(__uint_as_float(w[i]) * inv, __uint_as_float(w[i + 1]) * inv,
                            __uint_as_float(w[i + 2]) * inv, __uint_as_float(w[i + 3]) * inv);
        }
      }
    }
  }

  tc::fence_before_sync();
  __syncthreads();
  if (nsplit == 1) {
    if (warp == 5) {
      tc::fence_after_sync();
      tc::tmem_dealloc<512>(tmem);
    }
    return;
  }

  // ---- cluster combine. CTA c owns rows [c*SR, (c+1)*SR) of the tile. Every CTA pushes
  // its partial rows (O unnormalised, m, l) into the owners' receive buffers with
  // distributed-shared-memory stores, then each owner merges its rows from its own
  // shared memory and writes them.
  //  * with a receive buffer of its own (d <= 64) a CTA pushes as soon as its O is final;
  //    with the stage buffers as receive buffer (d = 128) a cluster barrier first makes
  //    sure every CTA's stage buffers are free (copies landed, MMAs drained above);
  //  * a cluster barrier then makes every push visible to its owner. After it no CTA
  //    touches another CTA's shared memory, so a CTA may exit once it has merged its rows.
  // (Signalling with remote mbarrier arrives instead of the cluster barriers measured
  // slower.) Rows are D floats apart, their 16-byte chunks XOR-swizzled by row & 7 so
  // that neither the pushes (a warp stores one chunk of 32 rows) nor the merge reads
  // conflict on banks.
  const int SR = BM / nsplit;
  float* rO = reinterpret_cast<float*>(smem + C::RECV_OFF);  // [nsplit * SR][D]
  float* rM = rO + BM * D;                                   // [nsplit * SR]
  float* rL = rM + BM;                                       // [nsplit * SR]
  if (C::RECV_OWN) {
    asm volatile("barrier.cluster.wait.aligned;" ::: "memory");  // every CTA running
  } else {
    cluster_sync_all();  // every CTA's stage buffers are free
  }
  if (threadIdx.x == 0) FE_TTL(9, globaltimer_ns());
  // Warps 0-7 push: warp w reads tensor-memory lanes 32 (w & 3) .. + 31 (the rows it may
  // access) and, for d >= 64, half of the columns ((w >> 2) selects the half).
  constexpr int PUSH_WARPS = D >= 64 ? 8 : 4;
  constexpr int PCOLS = D / (PUSH_WARPS / 4);
  if (warp < PUSH_WARPS) {
    const int row = (warp & 3) * 32 + lane;
    const int h = warp >> 2;
    const uint32_t owner = static_cast<uint32_t>(row / SR);
    const int slot = split * SR + (row - static_cast<int>(owner) * SR);
    const uint32_t tO = tmem + (static_cast<uint32_t>((warp & 3) * 32) << 16) + C::T_O + h * PCOLS;
    const uint32_t dst = cluster_map(smem_u32(rO + slot * D), owner);
    const bool valid = o_valid[warp & 3] != 0;
    tc::fence_after_sync();  // the MMAs' writes of O (drained before the CTA barrier)
#pragma unroll
    for (int c = 0; c < PCOLS / 32; ++c) {
      uint32_t w[32];
      if (valid) {
        tc::ld32(tO + c * 32, w);
        tc::wait_ld();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) w[i] = 0u;
      }
#pragma unroll
      for (int i = 0; i < 32; i += 4) {
        const int chunk = (h * PCOLS + c * 32 + i) >> 2;
        st_cluster_v4(dst + ((chunk ^ (slot & 7)) << 4), __uint_as_float(w[i]),
                      __uint_as_float(w[i + 1]), __uint_as_float(w[i + 2]),
                      __uint_as_float(w[i + 3]));
      }
    }
    if (h == 0) {
      st_cluster_f32(cluster_map(smem_u32(rM + slot), owner), m_run);
      st_cluster_f32(cluster_map(smem_u32(rL + slot), owner), l_run);
    }
  }
  tc::fence_before_sync();
  if (threadIdx.x == 0) FE_TTL(10, globaltimer_ns());
  cluster_sync_all();  // every push has reached its owner
  if (threadIdx.x == 0) FE_TTL(11, globaltimer_ns());
  if (warp == 5) {     // every tensor-memory read of this CTA is done
    tc::fence_after_sync();
    tc::tmem_dealloc<512>(tmem);
  }
  constexpr int C4 = D / 4;
  for (int idx = threadIdx.x; idx < SR * C4; idx += C::NTHREADS) {
    const int rr = idx / C4, c4 = idx - rr * C4;
    const int row = m0 + split * SR + rr;
    if (row >= p.N) continue;
    float ms[8], ls[8];
    float4 os[8];
    float mx = NEG_INF;
#pragma unroll
    for (int s2 = 0; s2 < 8; ++s2) {
      if (s2 < nsplit) {
        const int slot = s2 * SR + rr;
        ms[s2] = rM[slot];
        ls[s2] = rL[slot];
        os[s2] = *reinterpret_cast<const float4*>(rO + slot * D + ((c4 ^ (slot & 7)) << 2));
        mx = fmaxf(mx, ms[s2]);
      }
    }
    float tot = 0.f;
    float4 o4 = make_float4(0.f, 0.f, 0.f, 0.f);
    if (mx != NEG_INF) {
#pragma unroll
      for (int s2 = 0; s2 < 8; ++s2) {
        if (s2 < nsplit) {
          const float w = ex2(ms[s2] - mx);
          tot = fmaf(ls[s2], w, tot);
          o4.x = fmaf(w, os[s2].x, o4.x);
          o4.y = fmaf(w, os[s2].y, o4.y);
          o4.z = fmaf(w, os[s2].z, o4.z);
          o4.w = fmaf(w, os[s2].w, o4.w);
        }
      }
    }
    const float inv = tot > 0.f ? 1.f / tot : 0.f;
    *reinterpret_cast<float4*>(p.out + (static_cast<size_t>(bh) * p.N + row) * D + c4 * 4) =
        make_float4(o4.x * inv, o4.y * inv, o4.z * inv, o4.w * inv);
  }
#ifdef FE_TF32_TIMELINE
  if (threadIdx.x == 0) {
    FE_TTL(12, globaltimer_ns());
    FE_TTL(14, clock64() - clk0);
  }
#endif
}

// CTAs (one cluster) per 128-row tile: the most (up to 8 and up to the key-tile count)
// that still keep the grid within one CTA per SM, with 8-CTA clusters only while there
// are at most 8 of them (64 CTAs): at 16 of them (the 4-head shard of config 1) a step
// measured 15.5 us against 9.7 us with 4-CTA clusters. FE_TF32_SPLIT=1,2,4,8 overrides the
// choice (tuning).
static int tf32_split(long long row_tiles_bh, int kv_tiles) {
  static const int forced = [] {
    const char* s = getenv("FE_TF32_SPLIT");
    const int v = s ? atoi(s) : 0;
    return (v == 1 || v == 2 || v == 4 || v == 8) ? v : 0;
  }();
  int n = 1;
  if (forced) {
    n = forced;
  } else {
    const long long slots = sm_count();
    while (n < 8 && row_tiles_bh * n * 2 <= slots) n *= 2;
    if (n == 8 && row_tiles_bh > 8) n = 4;
  }
  while (n > 1 && n > kv_tiles) n /= 2;
  return n;
}

}  // namespace tf32

namespace simt {

// True when the fp32 forward of this shape runs on the tensor-core kernel above.
bool fa2_tf32_eligible(const float* q, const float* k, const float* v, const float* o, int B,
                       int H, int N, int M, int d) {
  static const bool off = [] {
    const char* s = getenv("FE_FP32_SIMT");
    return s && atoi(s) != 0;
  }();
  const auto al = [](const void* x) { return (reinterpret_cast<uintptr_t>(x) & 15) == 0; };
  return !off && (d == 32 || d == 64 || d == 128) && N > 0 && M > 0 &&
         static_cast<long long>(B) * H <= 65535 && al(q) && al(k) && al(v) && al(o);
}

template <int D>
static cudaError_t launch_fa2_tf32_d(const float* q, const float* k, const float* v, float* o,
                                     int B, int H, int N, int M, float scale, int causal,
                                     cudaStream_t st) {
  using namespace tf32;
  using C = TCfg<D>;
  auto kern = fa_tf32_kernel<D>;
  cudaError_t e = ensure_smem_optin(reinterpret_cast<const void*>(kern), C::SMEM_LAUNCH);
  if (e != cudaSuccess) return e;
  const long long BH = static_cast<long long>(B) * H;
  CUtensorMap qm, km, vm;
  e = encode_tma_3d_f32(&qm, q, D, N, BH, 32, C::BM);
  if (e != cudaSuccess) return e;
  e = encode_tma_3d_f32(&km, k, D, M, BH, 32, C::BN);
  if (e != cudaSuccess) return e;
  e = encode_tma_3d_f32(&vm, v, D, M, BH, 32, C::BN);
  if (e != cudaSuccess) return e;
  const int row_tiles = (N + C::BM - 1) / C::BM;
  const int kv_tiles = (M + C::BN - 1) / C::BN;
  TParams p;
  p.out = o;
  p.N = N;
  p.M = M;
  p.causal = causal;
  p.nsplit = tf32_split(static_cast<long long>(row_tiles) * BH, kv_tiles);
  p.scale_log2 = scale * kLog2e;
  p.err = device_error_word();
  if (!p.err) return cudaErrorInitializationError;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(row_tiles * p.nsplit), static_cast<unsigned>(BH));
  cfg.blockDim = dim3(C::NTHREADS);
  cfg.dynamicSmemBytes = C::SMEM_LAUNCH;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = p.nsplit;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = p.nsplit > 1 ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kern, qm, km, vm, p);
}

cudaError_t launch_fa2_tf32(const float* q, const float* k, const float* v, float* o, int B, int H,
                            int N, int M, int d, float scale, int causal, cudaStream_t st) {
  if (!fa2_tf32_eligible(q, k, v, o, B, H, N, M, d)) return cudaErrorInvalidValue;
  if (d == 32) return launch_fa2_tf32_d<32>(q, k, v, o, B, H, N, M, scale, causal, st);
  if (d == 128) return launch_fa2_tf32_d<128>(q, k, v, o, B, H, N, M, scale, causal, st);
  return launch_fa2_tf32_d<64>(q, k, v, o, B, H, N, M, scale, causal, st);
}

}  // namespace simt
}  // namespace fe

#ifdef FE_TF32_TIMELINE
extern "C" int fe_debug_tf32_timeline(unsigned long long* host) {
  return static_cast<int>(cudaMemcpyFromSymbol(host, fe::tf32::g_tf32_timeline,
                                               sizeof(fe::tf32::g_tf32_timeline)));
}
#endif
