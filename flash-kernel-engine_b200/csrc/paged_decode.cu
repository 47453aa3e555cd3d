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
//  * Persistent CTAs (SMs x occupancy). Two ways to cut the work into segments
//    (a contiguous page range of one (sequence, KV-head group)):
//      - unit mode (no scratch): one segment per (sequence, KV-head group),
//        dealt round-robin to the CTAs;
//      - flat mode (split-KV with partials): the (KV-head group, sequence, page)
//        space is cut into gridDim.x equal contiguous chunks (stream-K style), one
//        per CTA, so every CTA streams the same number of pages whatever the
//        context-length mix. A sequence inside one chunk is finalised directly. Only
//        the first and the last segment of a chunk can be pieces of a longer
//        sequence, so each CTA owns two fp32 partial slots of a small fixup buffer
//        (slot 0: its first segment, slot 1: its last). After its last segment a
//        CTA bumps the arrival counter of each sequence it holds a piece of
//        (indexed by the chunk the sequence starts in); the CTA whose piece
//        arrives last combines all pieces with the log-sum-exp merge and resets
//        the counter to zero. No second kernel and no waiting; counting at the end
//        keeps the counter updates out of the streaming loop.
//    Both modes read context_lens and build the page prefix with a block-wide scan
//    in every CTA, so no host synchronisation or scratch is needed to skip or
//    place work.
//  * One producer warp streams each (block, KV head) page of K and V into shared
//    memory, completing on mbarriers. Flat cache layout: 2-D TMA bulk-tensor loads
//    with 128-byte swizzle. vLLM layout (K [blocks, Hkv, d/8, 16, 8], V [blocks,
//    Hkv, d, 16]): one contiguous bulk copy per page of K and of V; that layout is
//    already conflict-free for ldmatrix (K chunks of 8 tokens are 128 contiguous
//    bytes, V is stored as V^T rows). L2 evict-first; single-CTA destinations.
//    Block-table entries are fetched 32 at a time, one 32-page group ahead. The
//    whole warp runs the loop and waits for each ring slot; one elected lane issues
//    the copies.
//  * NCW consumer warps, each with a private ring of DEPTH stages (page gi of the
//    CTA belongs to warp gi % NCW). Per 16 tokens a warp computes S^T = K Q^T with
//    mma.m16n8k16 (tokens x query heads: all G query heads of the group share
//    every K/V byte fetched), does the online-softmax update in the log2 domain,
//    turns P^T into the B operand with movmatrix and accumulates O^T += V^T P^T
//    (V^T fragments via ldmatrix.trans from the swizzled tile).
//  * At the end of a segment the consumer warps merge their (m, l, O) in shared
//    memory and write the final row or a partial.
#include <limits.h>

#include <type_traits>

#include "../../include/cuda_utils.cuh"
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

// fp32 cache: the CUDA-core consumer of paged_decode_kernel (no tensor-core product).
template <>
struct Elem<float> {
  static __device__ __forceinline__ float cvt(float x) { return x; }
};

constexpr float NEG_INF = -__builtin_huge_valf();

// The library-owned split-KV scratch of the v1 entry points (see kStreamSlots).
// Zero when the module loads; every launch leaves its slot's counters at zero.
static __device__ __align__(256) float g_stream_scratch[kStreamSlots * kStreamSlotFloats];

__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
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

// Token window of a sequence: [lo, hi) = [tok_begin, min(tok_end, ctx)); its pages
// [lo / bs, ceil(hi / bs)).
struct Window {
  int lo, hi, pb, np;
};
__device__ __forceinline__ Window seq_window(int ctx, int tb, int te, int bs) {
  Window w;
  w.lo = max(tb, 0);
  w.hi = min(te, ctx);
  if (w.hi <= w.lo) {
    w.pb = 0;
    w.np = 0;
  } else {
    w.pb = w.lo / bs;
    w.np = (w.hi + bs - 1) / bs - w.pb;
  }
  return w;
}

// Flat mode keeps, per sequence, its page prefix pre[] and the number of window tokens
// in its last page (tail[], 1..BS) in shared memory, so the segment walk rebuilds a
// window without reading context_lens again. The window starts at tok_begin, a multiple
// of BS.
__device__ __forceinline__ uint8_t last_page_tokens(const Window& w, int bs) {
  return w.np > 0 ? static_cast<uint8_t>(w.hi - (w.pb + w.np - 1) * bs) : 0;
}
__device__ __forceinline__ Window flat_window(const int* pre, const uint8_t* tail, int s, int tb,
                                              int bs) {
  Window w;
  w.np = pre[s + 1] - pre[s];
  w.lo = max(tb, 0);
  w.pb = w.lo / bs;
  w.hi = w.np > 0 ? (w.pb + w.np - 1) * bs + tail[s] : w.lo;
  return w;
}

// Number of unit-mode segments of a sequence: one per pages_per_split pages (at
// least one, so that an empty sequence still gets its zero output row).
__device__ __forceinline__ int unit_splits(const Window& w, int pps) {
  return w.np == 0 ? 1 : (w.np + pps - 1) / pps;
}

// Block-wide exclusive prefix over S per-sequence counts into pre[0..S] (pre[S] =
// total). `count(i)` must be cheap and pure; every thread of the block calls this.
template <int NTH, typename Count>
__device__ __forceinline__ void block_prefix(int* pre, int S, int* warp_tot, Count count) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  constexpr int NW = NTH / 32;
  const int per = (S + NTH - 1) / NTH;
  const int beg = min(S, tid * per), end = min(S, beg + per);
  int local = 0;
  for (int i = beg; i < end; ++i) local += count(i);
  const int incl = warp_incl_scan(local);
  if (lane == 31) warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int v = lane < NW ? warp_tot[lane] : 0;
    v = warp_incl_scan(v);
    if (lane < NW) warp_tot[lane] = v;
  }
  __syncthreads();
  int run = incl - local + (warp > 0 ? warp_tot[warp - 1] : 0);
  for (int i = beg; i < end; ++i) {
    pre[i] = run;
    run += count(i);
  }
  if (tid == 0) pre[S] = warp_tot[NW - 1];
  __syncthreads();
}

// Largest s in [0, S) with pre[s] <= r.
__device__ __forceinline__ int find_seq(const int* pre, int S, long long r) {
  int lo = 0, hi = S;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (pre[mid] <= r) lo = mid; else hi = mid;
  }
  return lo;
}

// Flat-mode partition. The (KV-head group y, sequence s) units are laid out in a cost
// space in which unit (y, s) takes beta virtual pages followed by its np(s) pages:
// unit (y, s) starts at y * (Ptot + beta * S) + pre[s] + beta * s. The cost space is
// cut into gridDim.x equal chunks, one per CTA, and a CTA streams the pages inside its
// chunk. A sequence that starts inside a chunk costs the CTA a segment change (merge of
// the warp states, partial writes, a piece to count in) that takes about as long as
// streaming a few pages, so those beta pages are taken off that CTA's share. A CTA
// whose chunk holds only virtual pages gets no pages; it can never sit between two
// pieces of one unit, whose pages are contiguous. Kept in shared memory, one per CTA.
struct FlatPartition {
  const int* pre;
  int S, Ptot, beta;
  long long Cy;   // cost of one y: Ptot + beta * S
  long long C;    // total cost: Y * Cy
  long long cc;   // cost per CTA chunk
  double inv_cc;  // 1 / cc
  // Largest s in [0, S) with pre[s] + beta * s <= r.
  __device__ __forceinline__ int unit_at(long long r) const {
    int lo = 0, hi = S;
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (pre[mid] + static_cast<long long>(beta) * mid <= r) lo = mid; else hi = mid;
    }
    return lo;
  }
  // Global page index (y * Ptot + page) at cost position c (the first page at or after c).
  __device__ __forceinline__ long long page_at(long long c) const {
    if (c >= C) return static_cast<long long>(C / Cy) * Ptot;
    const long long y = c / Cy;
    const long long r = c - y * Cy;
    const int s = unit_at(r);
    const long long off = r - (pre[s] + static_cast<long long>(beta) * s);
    return y * Ptot + pre[s] + (off > beta ? off - beta : 0);
  }
  // floor(c / cc) for 0 <= c < 2^52: a reciprocal multiply, corrected by one step.
  __device__ __forceinline__ int chunk_of(long long c) const {
    long long q = static_cast<long long>(static_cast<double>(c) * inv_cc);
    if (q * cc > c) --q;
    else if ((q + 1) * cc <= c) ++q;
    return static_cast<int>(q);
  }
  // Cost position of the first page of unit (y, s).
  __device__ __forceinline__ long long unit_cost(int y, int s) const {
    return static_cast<long long>(y) * Cy + pre[s] + static_cast<long long>(beta) * (s + 1);
  }
};

struct Seg {
  int seq, kvh, hc;
  int p0, p1;     // absolute pages [p0, p1)
  int lo, hi;     // valid tokens [lo, hi)
  int slot;       // flat mode: fixup slot of a piece: 1 = the unit's first piece (the
                  // last segment of its CTA), 0 = a continuation (the CTA's first segment)
  int nslots;     // chunks (segments) of this (sequence, head group); 1 = finalise here
  int cfirst;     // flat mode: chunk holding the first page of this (sequence, group)
};

// Walks the segments of one CTA. Producer and consumers run identical copies.
struct SegIter {
  const Params* p;
  const int* pre;
  const uint8_t* tail;  // flat mode
  int S, Y, HC, BS;
  bool flat;
  // unit mode
  int u, total_units;
  // flat mode
  long long P, Pend;
  int Ptot;
  int y;           // KV-head group of page P, and y * Ptot
  long long ybase;
  const FlatPartition* fp;  // in shared memory (keeps the walk's registers few)

  __device__ __forceinline__ bool next(Seg& g) {
    if (!flat) {
      if (u >= total_units) return false;
      const int cu = u / Y, y = u - cu * Y;
      u += gridDim.x;
      const int seq = find_seq(pre, S, cu);
      const Window w = seq_window(__ldg(p->context_lens + seq), p->tok_begin, p->tok_end, BS);
      const int split = cu - pre[seq];
      g.seq = seq;
      g.kvh = y / HC;
      g.hc = y - g.kvh * HC;
      g.p0 = w.pb + split * p->pages_per_split;
      g.p1 = min(w.pb + w.np, g.p0 + p->pages_per_split);
      if (g.p1 < g.p0) g.p1 = g.p0;
      g.lo = w.lo;
      g.hi = w.hi;
      g.slot = split;
      g.nslots = pre[seq + 1] - pre[seq];
      g.cfirst = 0;
      return true;
    }
    if (P >= Pend) return false;
    while (P >= ybase + Ptot) {  // P only grows: no division
      ybase += Ptot;
      ++y;
    }
    const int r = static_cast<int>(P - ybase);
    const int seq = find_seq(pre, S, r);
    const Window w = flat_window(pre, tail, seq, p->tok_begin, BS);
    const int in0 = r - pre[seq];
    const long long left = Pend - P;
    const int n = static_cast<int>(min(static_cast<long long>(w.np - in0), left));
    g.seq = seq;
    g.kvh = y / HC;
    g.hc = y - g.kvh * HC;
    g.p0 = w.pb + in0;
    g.p1 = g.p0 + n;
    g.lo = w.lo;
    g.hi = w.hi;
    // chunks holding the unit's first and last page
    const long long c0 = fp->unit_cost(y, seq);
    const int cfirst = fp->chunk_of(c0);
    g.nslots = fp->chunk_of(c0 + w.np - 1) - cfirst + 1;
    g.cfirst = cfirst;
    g.slot = in0 == 0 ? 1 : 0;
    P += n;
    return true;
  }
};

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

// Log-sum-exp combine of the `total` partials of one output row by one warp
// (src/flash_decoding.cu:151-223: g = max m_p, L = sum l_p 2^(m_p - g),
// O = sum O_p 2^(m_p - g)); part j is slot slot_of(j), its O row (D floats) at
// part_out + o_off(slot) and its (m in log2 units, l) at part_stats + s_off(slot);
// empty parts (l = 0) carry no weight.
// Returns M = g (-inf if every part is empty), L, and acc[e] = O at dim lane + 32e.
// Loads bypass L1: the partials may have been written by other CTAs of this grid.
// Up to BATCH parts take one memory round trip (stats and O rows loaded together);
// more take one for the stats and one per BATCH parts of O rows.
template <int PER, int BATCH, typename SlotOf, typename OOff, typename SOff>
__device__ __forceinline__ void lse_combine_warp(const float* __restrict__ part_out,
                                                 const float* __restrict__ part_stats, int total,
                                                 int D, SlotOf slot_of, OOff o_off, SOff s_off,
                                                 float& M_out, float& L_out, float (&acc)[PER]) {
  const int lane = threadIdx.x & 31;
  if (total <= 32) {
    // Up to 32 parts: lane j loads part j's stats while the O rows of the first BATCH
    // parts load too (one round trip); further O rows follow BATCH at a time.
    float m = NEG_INF, l = 0.f;
    if (lane < total) {
      const size_t slot = slot_of(lane);
      m = __ldcg(part_stats + s_off(slot));
      l = __ldcg(part_stats + s_off(slot) + 1);
    }
    float v[BATCH][PER];
    auto load_rows = [&](int k0) {
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        const bool in = k0 + k < total;
        const float* po = part_out + o_off(in ? slot_of(k0 + k) : slot_of(0));
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          const int dim = lane + 32 * e;
          v[k][e] = (in && dim < D) ? __ldcg(po + dim) : 0.f;
        }
      }
    };
    load_rows(0);
    float M = l > 0.f ? m : NEG_INF;
    M = flash_engine::cuda::warp_reduce_max(M);
    const float w = l > 0.f ? ex2(m - M) : 0.f;
    float L = l * w;
    L = flash_engine::cuda::warp_reduce_sum(L);
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = 0.f;
    for (int k0 = 0; k0 < total; k0 += BATCH) {
      if (k0 > 0) load_rows(k0);
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        const float wk = __shfl_sync(0xffffffffu, w, (k0 + k) & 31);
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[e] += v[k][e] * wk;
      }
    }
    M_out = M;
    L_out = L;
    return;
  }
  float M = NEG_INF;
  for (int j = lane; j < total; j += 32) {
    const size_t slot = slot_of(j);
    const float l = __ldcg(part_stats + s_off(slot) + 1);
    if (l > 0.f) M = fmaxf(M, __ldcg(part_stats + s_off(slot)));
  }
  M = flash_engine::cuda::warp_reduce_max(M);
  float L = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) acc[k] = 0.f;
  for (int j0 = 0; j0 < total; j0 += 32) {
    const int j = j0 + lane;
    float wt = 0.f, l = 0.f;
    size_t myslot = 0;
    if (j < total) {
      myslot = slot_of(j);
      l = __ldcg(part_stats + s_off(myslot) + 1);
      if (l > 0.f) wt = ex2(__ldcg(part_stats + s_off(myslot)) - M);
    }
    L += l * wt;
    const int cnt = min(32, total - j0);
    for (int k0 = 0; k0 < cnt; k0 += BATCH) {
      float v[BATCH][PER];
      float w8[BATCH];
#pragma unroll
      for (int k = 0; k < BATCH; ++k) {
        const int kk = min(k0 + k, cnt - 1);
        w8[k] = k0 + k < cnt ? __shfl_sync(0xffffffffu, wt, kk) : 0.f;
        const size_t sl = __shfl_sync(0xffffffffu, static_cast<unsigned long long>(myslot), kk);
        const float* po = part_out + o_off(sl);
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          const int dim = lane + 32 * e;
          v[k][e] = (dim < D && w8[k] != 0.f) ? __ldcg(po + dim) : 0.f;
        }
      }
#pragma unroll
      for (int k = 0; k < BATCH; ++k)
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[e] += v[k][e] * w8[k];
    }
  }
  L = flash_engine::cuda::warp_reduce_sum(L);
  M_out = M;
  L_out = L;
}

#ifdef FE_TIMELINE
// Per-CTA event times (globaltimer ns) of the last decode launch, for profiling
// builds only: [0] entry, [1] prefix done, [2] first page issued, [3] first page
// ready (consumer warp 0), [4] consumers done, [5] producer done issuing,
// [6] SM id, [7] nanoseconds spent merging split sequences, [8] consumer warp 0 past
// griddepcontrol.wait (the previous grid has completed), [9..11] unused.
__device__ unsigned long long g_timeline[kCounterSlots][12];
#define FE_TL(slot) (g_timeline[blockIdx.x][slot] = globaltimer_ns())
#else
#define FE_TL(slot) ((void)0)
#endif

// A piece of a split (sequence, head group) written by this CTA (flat mode).
struct Pending {
  int cfirst, nslots, seq, kvh, hc, last;
};

template <typename T, int D, int BS, int NT, int NCW, int NSTAGE>
struct Cfg {
  static constexpr bool F32 = std::is_same<T, float>::value;
  static constexpr int HPC = F32 ? 4 * NT : 8 * NT;  // query heads per CTA
  static constexpr int HALVES = D / 64;    // 128-byte swizzle atoms per row (16-bit caches)
  static constexpr int TILE = BS * D * static_cast<int>(sizeof(T));  // one page of K (or V)
  static constexpr int STAGE = 2 * TILE;
  static constexpr int CSTRIDE = D + 4;    // padded row of the merge buffer (floats)
  static constexpr int NTHREADS = (NCW + 1) * 32;
  static constexpr int COMB_BYTES = NCW * HPC * (2 + CSTRIDE) * 4;
  static constexpr int FIXED_SMEM = 1024 /*align slack*/ + NSTAGE * STAGE + COMB_BYTES +
                                    NSTAGE * 16 /*bars*/ + NSTAGE * 4 + 64;
  // + pre[num_seqs + 1] ints and tail[num_seqs] bytes
  static int smem_bytes(int num_seqs) { return FIXED_SMEM + (num_seqs + 1) * 4 + num_seqs + 16; }
};

// Two CTAs of NCW + 1 warps share an SM only if three warps fit one SM sub-partition's
// 16K registers: at most 168 registers a thread (bf16/fp16 NT = 1, and the fp32 decode).
// bf16/fp16 NT = 2 keeps one CTA per SM.
template <typename T, int NT>
struct DecodeRegs {
  static constexpr int value = (NT == 1 || std::is_same<T, float>::value) ? 168 : 255;
};

// Stages of each consumer warp's private ring: about 64 KB of pages per CTA, 1 to 4
// stages a warp.
template <typename T, int D, int BS, int NCW>
constexpr int ring_depth() {
#ifndef FE_DECODE_RING_BYTES
#define FE_DECODE_RING_BYTES 65536
#endif
  constexpr int stage = 2 * BS * D * static_cast<int>(sizeof(T));
  constexpr int dpt = FE_DECODE_RING_BYTES / (NCW * stage);
  return dpt < 1 ? 1 : dpt > 4 ? 4 : dpt;
}

template <typename T, int D, int BS, int NT, int NCW, int NSTAGE, int KVL>
__global__ void __maxnreg__((DecodeRegs<T, NT>::value))
    paged_decode_kernel(const __grid_constant__ CUtensorMap kmap,
                        const __grid_constant__ CUtensorMap vmap, const Params p) {
  using C = Cfg<T, D, BS, NT, NCW, NSTAGE>;
  constexpr int HPC = C::HPC, HALVES = C::HALVES, TILE = C::TILE, STAGE = C::STAGE;
  constexpr int CSTRIDE = C::CSTRIDE, NTH = C::NTHREADS;
  using SO = StageOf<NCW, NSTAGE / NCW>;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  float* comb_m = reinterpret_cast<float*>(smem + NSTAGE * STAGE);  // [NCW][HPC]
  float* comb_l = comb_m + NCW * HPC;                                // [NCW][HPC]
  float* comb_o = comb_l + NCW * HPC;                                // [NCW][HPC][CSTRIDE]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NSTAGE * STAGE + C::COMB_BYTES);
  uint64_t* empty = full + NSTAGE;
  int* stage_valid = reinterpret_cast<int*>(empty + NSTAGE);
  int* pre = stage_valid + NSTAGE;  // [num_seqs + 1]
  uint8_t* tail = reinterpret_cast<uint8_t*>(pre + p.num_seqs + 1);  // [num_seqs] (flat mode)
  __shared__ int warp_tot[NCW + 1];
  __shared__ Pending pend[2];  // flat mode: pieces written as slot 0 / slot 1
  __shared__ FlatPartition fpart;  // flat mode: the partition of the work over the CTAs

  // Programmatic dependent launch, both ways: the next kernel in the stream may start
  // its CTAs as soon as SM room frees up (it waits for this grid's results before
  // reading them), and this grid, launched the same way, waits (griddepcontrol.wait)
  // for the previous kernel's results before it reads anything that kernel may write.
  griddep_launch_dependents();

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) FE_TL(0);
#ifdef FE_TIMELINE
  if (tid == 0) {
    unsigned smid;
    asm volatile("mov.u32 %0, %%smid;" : "=r"(smid));
    g_timeline[blockIdx.x][6] = smid;
    g_timeline[blockIdx.x][7] = 0;
  }
#endif
  const int S = p.num_seqs;
  const int Hkv = p.num_kv_heads, G = p.num_heads / p.num_kv_heads;
  const int HC = p.head_chunks, Y = Hkv * HC;
  const bool flat = p.flat != 0;
  const bool direct_final = p.direct_final != 0;
  // Split-KV scratch: the caller's workspace, or a slot of the library's own.
  float* part_o = p.part_o;
  float* part_ml = p.part_ml;
  int* counters = p.counters;
  if (p.ws_slot >= 0) {
    float* base = g_stream_scratch + static_cast<size_t>(p.ws_slot) * kStreamSlotFloats;
    counters = reinterpret_cast<int*>(base);
    part_o = base + kCounterSlots;
    part_ml = part_o + static_cast<size_t>(gridDim.x) * 2 * HPC * D;
  }

  // Until griddepcontrol.wait below, this grid touches only shared memory and the two
  // inputs that no kernel of this library writes, context_lens and block_tables: the
  // prefix over the sequences and the producer's first block-table group are read
  // while the previous grid (typically the previous decode step) is still finishing.
  // This grid can start before the previous kernel in the stream has completed only if
  // that kernel executed griddepcontrol.launch_dependents, which only this library's
  // kernels do; inputs written by a copy, a host write or any kernel that does not
  // trigger programmatic completion are complete before this grid starts.
  // q, the KV cache, the workspace, the exchange buffers and the outputs are accessed
  // only after the wait.
  if (tid == 0) {
    for (int s = 0; s < NSTAGE; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    fence_mbar_init();
    pend[0].nslots = pend[1].nslots = 0;
  }

  SegIter it;
  it.p = &p;
  it.pre = pre;
  it.tail = tail;
  it.S = S;
  it.Y = Y;
  it.HC = HC;
  it.BS = BS;
  it.flat = flat;
  if (flat) {
    block_prefix<NTH>(pre, S, warp_tot, [&](int i) {
      const Window w = seq_window(__ldg(p.context_lens + i), p.tok_begin, p.tok_end, BS);
      tail[i] = last_page_tokens(w, BS);  // written twice, the same value
      return w.np;
    });
    it.Ptot = pre[S];
    const long long total_pages = static_cast<long long>(Y) * it.Ptot;
    if (tid == 0) {
      FlatPartition& fp = fpart;
      fp.pre = pre;
      fp.S = S;
      fp.Ptot = it.Ptot;
      // beta is halved until it is at most a quarter of a chunk (chunks of little work)
      fp.beta = p.seg_cost_pages;
      for (;;) {
        fp.Cy = it.Ptot + static_cast<long long>(fp.beta) * S;
        fp.C = static_cast<long long>(Y) * fp.Cy;
        fp.cc = (fp.C + gridDim.x - 1) / gridDim.x;
        if (fp.cc < 1) fp.cc = 1;
        if (4LL * fp.beta <= fp.cc || fp.beta == 0) break;
        fp.beta >>= 1;
      }
      fp.inv_cc = 1.0 / static_cast<double>(fp.cc);
    }
    __syncthreads();
    it.fp = &fpart;
    it.P = total_pages == 0 ? 0 : fpart.page_at(static_cast<long long>(blockIdx.x) * fpart.cc);
    it.Pend =
        total_pages == 0 ? 0 : fpart.page_at(static_cast<long long>(blockIdx.x + 1) * fpart.cc);
    it.y = it.Ptot > 0 ? static_cast<int>(it.P / it.Ptot) : 0;
    it.ybase = static_cast<long long>(it.y) * it.Ptot;
    it.u = it.total_units = 0;
  } else {
    block_prefix<NTH>(pre, S, warp_tot, [&](int i) {
      return unit_splits(seq_window(__ldg(p.context_lens + i), p.tok_begin, p.tok_end, BS),
                         p.pages_per_split);
    });
    it.u = blockIdx.x;
    it.total_units = pre[S] * Y;
    it.P = it.Pend = 0;
    it.Ptot = 0;
    it.y = 0;
    it.ybase = 0;
    it.fp = nullptr;
  }
  if (tid == 0) FE_TL(1);

  if (warp == NCW) {
    // ===================================================== producer warp
    if (lane == 0 && KVL == kKvFlat && !C::F32) {
      prefetch_tensormap(&kmap);
      prefetch_tensormap(&vmap);
    }
    const uint64_t pol = l2_policy_evict_first();
    // Block-table entries of one 32-page group of a segment (lane i: page base+i). The
    // loads are only issued here; the entries are checked (check_group) one group later,
    // when they have landed, so the producer never waits on them before issuing the
    // current group's copies.
    constexpr int kNoPage = INT_MIN;      // lane past the segment
    constexpr int kPastRow = INT_MIN + 1; // page past the block-table row
    auto load_group = [&](const Seg& g, int base, int& phys) {
      phys = kNoPage;
      const int page = g.p0 + base + lane;
      if (page < g.p1) {
        phys = page >= p.max_blocks_per_seq
                   ? kPastRow
                   : __ldg(p.block_tables + static_cast<size_t>(g.seq) * p.max_blocks_per_seq +
                           page);
      }
    };
    auto check_group = [&](const Seg& g, int phys) -> int {
      if (phys == kNoPage) return 0;
      if (phys == kPastRow) {
        atomicOr(p.err, kErrBadBlock);  // context longer than the block-table row
        return 0;
      }
      const long long row = (static_cast<long long>(phys) * Hkv + g.kvh) * BS;
      const int valid = phys >= 0 && (p.num_phys_blocks <= 0 || phys < p.num_phys_blocks) &&
                        row + BS <= static_cast<long long>(INT_MAX);
      if (!valid) atomicOr(p.err, kErrBadBlock);
      return valid;
    };
    int gi = 0;
    bool ok = true;
    const bool leader = elect_one();
    Seg cur;
    bool have = it.next(cur);
    int base = 0;
    int ph_cur = kNoPage;
    if (have) load_group(cur, 0, ph_cur);
    griddep_wait();  // the KV cache may have been written by the previous kernel
    while (have && ok) {
      const int vd_cur = check_group(cur, ph_cur);  // loaded one group ago
      // Look one 32-page group ahead and start its block-table loads now.
      Seg ns = cur;
      int nbase = base + 32;
      bool have_n = true;
      if (cur.p0 + nbase >= cur.p1) {
        have_n = it.next(ns);
        nbase = 0;
      }
      int ph_n = kNoPage;
      if (have_n) load_group(ns, nbase, ph_n);
      const int cnt = max(0, min(32, cur.p1 - cur.p0 - base));
      for (int k = 0; k < cnt; ++k) {
        const int ph = __shfl_sync(0xffffffffu, ph_cur, k);
        const int vd = __shfl_sync(0xffffffffu, vd_cur, k);
        // the whole warp waits for the slot; the elected lane issues its copies
        const SO so(gi);
        const int s = so.s;
        int good = so.round == 0 ||
                   __all_sync(0xffffffffu, mbar_wait(&empty[s], (so.round - 1) & 1));
        if (!good && lane == 0) atomicOr(p.err, kErrWaitTimeout);
        if (good && leader) {
          {
            stage_valid[s] = vd;
            uint8_t* ks = smem + s * STAGE;
            uint8_t* vs = ks + TILE;
            if (vd) {
#ifdef FE_TIMELINE
              if (gi == 0) FE_TL(2);
#endif
              mbar_arrive_expect_tx(&full[s], STAGE);
              const int y = (ph * Hkv + cur.kvh) * BS;
#ifdef FE_DEBUG_CHECKS
              if (static_cast<long long>(y) + BS > p.dbg_kv_rows) atomicOr(p.err, 1u << 8);
#endif
              if constexpr (KVL == kKvFlat && !C::F32) {
#pragma unroll
                for (int h = 0; h < HALVES; ++h) {
                  tma_load_2d(ks + h * BS * 128, &kmap, h * 64, y, &full[s], pol);
                  tma_load_2d(vs + h * BS * 128, &vmap, h * 64, y, &full[s], pol);
                }
              } else {
                // vLLM layout, or an fp32 page: one contiguous chunk of K and of V
                const size_t off = static_cast<size_t>(y) * D * sizeof(T);  // page = BS*D elements
                bulk_load(ks, static_cast<const uint8_t*>(p.k_cache) + off, TILE, &full[s], pol);
                bulk_load(vs, static_cast<const uint8_t*>(p.v_cache) + off, TILE, &full[s], pol);
              }
            } else {
              mbar_arrive(&full[s]);  // nothing to load; consumers skip the page
            }
          }
        }
        if (!good) {
          ok = false;
          break;
        }
        ++gi;
      }
      cur = ns;
      base = nbase;
      ph_cur = ph_n;
      have = have_n;
    }
    // Drain: no bulk copy of this CTA may still be in flight when it exits.
    if (lane == 0) FE_TL(5);
    if (lane == 0) {
      for (int j = max(0, gi - NSTAGE); j < gi; ++j) {
        const SO so(j);
        if (!mbar_wait(&full[so.s], so.round & 1)) {
          atomicOr(p.err, kErrWaitTimeout);
          break;
        }
      }
    }
    return;
  }

  // ======================================================= consumer warps
  griddep_wait();
  if (tid == 0) FE_TL(8);
  using E = Elem<T>;
  const int g = lane >> 2, c = lane & 3;
  const T* __restrict__ qbase = reinterpret_cast<const T*>(p.q);
  const uint32_t ring = smem_u32(smem);
  const float sl = p.scale_log2;

  uint32_t qf[NT][D / 16][2];
  uint32_t qn[NT][D / 16][2];
  // q fragments (B operand of S^T = K Q^T): register j of k-step ks holds the
  // dimension pair (2i, 2i+1) with i = ks*8 + 4j + c, so the optional rotary
  // embedding (src/fused_rope.cu:33-43 arithmetic: x0 c - x1 s, x0 s + x1 c) is
  // applied pair by pair in fp32 before the repack.
  // Rotary position of a segment's query token: context_len - 1, clamped to the table.
  auto rope_pos = [&](const Seg& sg) -> int {
    int pos = __ldg(p.context_lens + sg.seq) - 1;
    if (pos < 0) pos = 0;
    if (pos >= p.rope_max_pos) {
      if (lane == 0) atomicOr(p.err, kErrBadBlock);
      pos = p.rope_max_pos - 1;
    }
    return pos;
  };
  auto load_q = [&](uint32_t (&dst)[NT][D / 16][2], const Seg& sg) {
    if constexpr (!C::F32) {
    const bool rope = p.rope_cos != nullptr;
    const int pos = rope ? rope_pos(sg) : 0;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int gh = sg.hc * HPC + nt * 8 + g;
      const bool v = gh < G;
      const T* qp =
          qbase + (static_cast<size_t>(sg.seq) * p.num_heads + sg.kvh * G + (v ? gh : 0)) * D;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          uint32_t w = v ? __ldg(reinterpret_cast<const unsigned*>(qp + ks * 16 + 8 * j + 2 * c))
                         : 0u;
          if (rope && v) {
            const int i = ks * 8 + 4 * j + c;
            const float cs = __ldg(p.rope_cos + static_cast<size_t>(pos) * (D / 2) + i);
            const float sn = __ldg(p.rope_sin + static_cast<size_t>(pos) * (D / 2) + i);
            const T* e = reinterpret_cast<const T*>(&w);
            const float x0 = static_cast<float>(e[0]), x1 = static_cast<float>(e[1]);
            w = E::pack(x0 * cs - x1 * sn, x0 * sn + x1 * cs);
          }
          dst[nt][ks][j] = w;
        }
      }
    }
    }
  };

  // Partials mode: a finished (O, m, l) row goes to merged_o / merged_ml, or, in
  // exchange mode, to this rank's slot of every rank's exchange buffer (generation
  // xstep & 1) as words tagged with xstep -- the all-gather of KV-range sharding done
  // by peer stores.
  // Exchange mode: the step this launch produces. The header is advanced only by the
  // merge of the previous step, which is complete (wait above), so every thread reads
  // the same value.
  const unsigned xstep =
      p.xworld > 0
          ? ld_volatile_u32(&reinterpret_cast<const XHeader*>(p.xbuf[p.xrank])->step) + 1u
          : 0u;
  auto emit_partial = [&](size_t row, int dim, float O, float M, float L) {
    if (p.xworld > 0) {
      const int par = static_cast<int>(xstep & 1u);
#pragma unroll
      for (int r = 0; r < kMaxRanks; ++r) {
        if (r >= p.xworld) break;
        unsigned long long* b =
            reinterpret_cast<unsigned long long*>(p.xbuf[r] + sizeof(XHeader));
        st_volatile_u64(b + x_o_word(par, p.xworld, p.xrank, p.xmax_rows, row, D) + dim,
                        tag_word(O, xstep));
        if (dim == 0) {
          unsigned long long* ml = b + x_ml_word(par, p.xworld, p.xrank, p.xmax_rows, row, D);
          st_volatile_u64(ml, tag_word(M, xstep));
          st_volatile_u64(ml + 1, tag_word(L, xstep));
        }
      }
    } else {
      p.merged_o[row * D + dim] = O;
      if (dim == 0) {
        p.merged_ml[row * 2 + 0] = M;
        p.merged_ml[row * 2 + 1] = L;
      }
    }
  };

  // Flat mode never visits a sequence with no pages in its window: its rows are
  // written here, by one CTA each, as zeros (or empty partials (0, -inf, 0)).
  if (flat) {
    for (int s = blockIdx.x; s < S; s += gridDim.x) {
      if (pre[s + 1] != pre[s]) continue;
      for (int idx = tid; idx < p.num_heads * D; idx += NCW * 32) {
        const size_t row = static_cast<size_t>(s) * p.num_heads + idx / D;
        const int dim = idx % D;
        if (direct_final) {
          reinterpret_cast<T*>(p.out)[row * D + dim] = E::cvt(0.f);
        } else {
          emit_partial(row, dim, 0.f, NEG_INF, 0.f);
        }
      }
    }
  }

  // fp32 consumer (CUDA cores). Lane i owns head dims [i*CW, (i+1)*CW) of every row,
  // CW = D/32; q of the segment's HPC heads sits in registers, pre-scaled by
  // scale*log2(e). Per group of TB = 32/HPC tokens of a page the warp forms the TB x HPC
  // partial dot products, reduce-scatters them (five butterfly steps, 31 shuffles) so
  // that lane l holds the score of token l / HPC, head l % HPC, updates the online
  // softmax with one exponential per lane, and accumulates P V with each p taken by
  // shuffle from the lane that holds it. The sum l stays split over the lanes of a head
  // until the segment ends.
  auto consume_f32 = [&](const Seg& sg, int npg, int first, int gb, bool& okr) {
    if constexpr (C::F32) {
      constexpr int HG = HPC;
      constexpr int TB = 32 / HG;
      constexpr int CW = D / 32;
      using VecT = typename std::conditional<CW == 4, float4, float2>::type;
      float qr[HG][CW];
      {
        const bool rope = p.rope_cos != nullptr;
        const int pos = rope ? rope_pos(sg) : 0;
        const float* qb = static_cast<const float*>(p.q);
#pragma unroll
        for (int h = 0; h < HG; ++h) {
          const int gh = sg.hc * HG + h;
          const bool v = gh < G;
          float x[CW];
          if (v) {
            const VecT t = __ldg(reinterpret_cast<const VecT*>(
                qb + (static_cast<size_t>(sg.seq) * p.num_heads + sg.kvh * G + gh) * D +
                lane * CW));
            x[0] = t.x;
            x[1] = t.y;
            if constexpr (CW == 4) {
              x[2] = t.z;
              x[3] = t.w;
            }
          } else {
#pragma unroll
            for (int cc = 0; cc < CW; ++cc) x[cc] = 0.f;
          }
          if (rope && v) {
#pragma unroll
            for (int cc = 0; cc < CW; cc += 2) {
              const int i = (lane * CW + cc) >> 1;
              const float cs = __ldg(p.rope_cos + static_cast<size_t>(pos) * (D / 2) + i);
              const float sn = __ldg(p.rope_sin + static_cast<size_t>(pos) * (D / 2) + i);
              const float x0 = x[cc], x1 = x[cc + 1];
              x[cc] = x0 * cs - x1 * sn;
              x[cc + 1] = x0 * sn + x1 * cs;
            }
          }
#pragma unroll
          for (int cc = 0; cc < CW; ++cc) qr[h][cc] = x[cc] * sl;
        }
      }
      float acc[HG][CW], mh[HG];
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        mh[h] = NEG_INF;
#pragma unroll
        for (int cc = 0; cc < CW; ++cc) acc[h][cc] = 0.f;
      }
      float m_own = NEG_INF, l_part = 0.f;  // head lane % HG
      for (int i = first; i < npg && okr; i += NCW) {
        const int gi = gb + i;
        const SO so(gi);
        const int s = so.s;
        const bool waited = mbar_wait(&full[s], so.round & 1);
        if (!__all_sync(0xffffffffu, waited)) {
          if (lane == 0) atomicOr(p.err, kErrWaitTimeout);
          okr = false;
          break;
        }
        const int t0 = (sg.p0 + i) * BS;
        const int vlo = max(sg.lo - t0, 0), vhi = min(sg.hi - t0, BS);
        if (stage_valid[s]) {
          const float* kt = reinterpret_cast<const float*>(smem + s * STAGE);
          const float* vt = kt + BS * D;
#pragma unroll 1
          for (int j0 = 0; j0 < BS; j0 += TB) {
            if (j0 >= vhi || j0 + TB <= vlo) continue;  // no token of the window here
            float kv[TB][CW], vv[TB][CW];
#pragma unroll
            for (int j = 0; j < TB; ++j) {
              const VecT a = *reinterpret_cast<const VecT*>(kt + (j0 + j) * D + lane * CW);
              const VecT b = *reinterpret_cast<const VecT*>(vt + (j0 + j) * D + lane * CW);
              kv[j][0] = a.x;
              kv[j][1] = a.y;
              vv[j][0] = b.x;
              vv[j][1] = b.y;
              if constexpr (CW == 4) {
                kv[j][2] = a.z;
                kv[j][3] = a.w;
                vv[j][2] = b.z;
                vv[j][3] = b.w;
              }
            }
            float x[32];  // x[j * HG + h]: this lane's part of q_h . k_j
#pragma unroll
            for (int j = 0; j < TB; ++j)
#pragma unroll
              for (int h = 0; h < HG; ++h) {
                float t = 0.f;
#pragma unroll
                for (int cc = 0; cc < CW; ++cc) t = fmaf(qr[h][cc], kv[j][cc], t);
                x[j * HG + h] = t;
              }
            // reduce-scatter: the step over lane bit `half` keeps the half of the
            // remaining indices selected by that bit; x[0] ends as index = lane
#pragma unroll
            for (int half = 16; half >= 1; half >>= 1) {
              const bool up = lane & half;
#pragma unroll
              for (int k = 0; k < half; ++k) {
                const float send = up ? x[k] : x[k + half];
                const float keep = up ? x[k + half] : x[k];
                x[k] = keep + __shfl_xor_sync(0xffffffffu, send, half);
              }
            }
            const int tok = j0 + lane / HG;
            const bool v_own = tok >= vlo && tok < vhi;
            const float s_own = v_own ? x[0] : NEG_INF;  // rows outside may hold anything
            float mx = s_own;
#pragma unroll
            for (int off = HG; off < 32; off <<= 1)
              mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float m_new = fmaxf(m_own, mx);  // finite: the group has a valid token
            const float p_own = v_own ? ex2(s_own - m_new) : 0.f;
            l_part = fmaf(l_part, ex2(m_own - m_new), p_own);
            m_own = m_new;
#pragma unroll
            for (int h = 0; h < HG; ++h) {
              const float mn = __shfl_sync(0xffffffffu, m_new, h);  // lane h: head h
              const float corr = ex2(mh[h] - mn);
              mh[h] = mn;
#pragma unroll
              for (int cc = 0; cc < CW; ++cc) acc[h][cc] *= corr;
            }
#pragma unroll
            for (int j = 0; j < TB; ++j) {
              if (j0 + j < vlo || j0 + j >= vhi) continue;  // warp-uniform; V may be NaN
#pragma unroll
              for (int h = 0; h < HG; ++h) {
                const float pj = __shfl_sync(0xffffffffu, p_own, j * HG + h);
#pragma unroll
                for (int cc = 0; cc < CW; ++cc) acc[h][cc] = fmaf(pj, vv[j][cc], acc[h][cc]);
              }
            }
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
      // this warp's state of the segment into the merge buffers
      float lsum = l_part;
#pragma unroll
      for (int off = HG; off < 32; off <<= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, off);
      if (lane < HG) {
        comb_m[warp * HPC + lane] = m_own;
        comb_l[warp * HPC + lane] = lsum;
      }
#pragma unroll
      for (int h = 0; h < HG; ++h) {
        VecT o;
        o.x = acc[h][0];
        o.y = acc[h][1];
        if constexpr (CW == 4) {
          o.z = acc[h][2];
          o.w = acc[h][3];
        }
        *reinterpret_cast<VecT*>(comb_o + (warp * HPC + h) * CSTRIDE + lane * CW) = o;
      }
    }
  };

  int gbase = 0;  // pages consumed by this CTA before the current segment
  bool ok = true;
  Seg sg, sn;
  bool have = it.next(sg);
  bool have_n = false;
  if (have) {
    load_q(qn, sg);
    have_n = it.next(sn);
  }
  while (have) {
    const int npg = max(0, sg.p1 - sg.p0);
    const int first = ((warp - gbase) % NCW + NCW) % NCW;
    if constexpr (C::F32) {
      consume_f32(sg, npg, first, gbase, ok);
    } else {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        qf[nt][ks][0] = qn[nt][ks][0];
        qf[nt][ks][1] = qn[nt][ks][1];
      }
    if (have_n) load_q(qn, sn);  // prefetch the next segment's q

    float m_run[NT][2], l_run[NT][2], o[NT][D / 16][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m_run[nt][0] = m_run[nt][1] = NEG_INF;
      l_run[nt][0] = l_run[nt][1] = 0.f;
#pragma unroll
      for (int mt = 0; mt < D / 16; ++mt) o[nt][mt][0] = o[nt][mt][1] = o[nt][mt][2] = o[nt][mt][3] = 0.f;
    }

    for (int i = first; i < npg && ok; i += NCW) {
      const int gi = gbase + i;
      const SO so(gi);
      const int s = so.s;
      const bool waited = mbar_wait(&full[s], so.round & 1);
#ifdef FE_TIMELINE
      if (gi == 0 && lane == 0) FE_TL(3);
#endif
      if (!__all_sync(0xffffffffu, waited)) {
        if (lane == 0) atomicOr(p.err, kErrWaitTimeout);
        ok = false;
        break;
      }
      const int t0 = (sg.p0 + i) * BS;
      const int vlo = max(sg.lo - t0, 0), vhi = min(sg.hi - t0, BS);
      const uint32_t ks = ring + s * STAGE, vs = ks + TILE;
      bool zeroed = false;
      if (stage_valid[s]) {
        if (vlo > 0 || vhi < BS) {
          // Rows outside the window may hold anything (NaN included); P is 0 there
          // but 0 * NaN is not, so clear those V rows before the PV product.
          uint8_t* vrow = smem + s * STAGE + TILE;
          if constexpr (KVL == kKvFlat) {
            for (int idx = lane; idx < BS * HALVES * 8; idx += 32) {
              const int row = (idx >> 3) % BS, h = idx / (8 * BS), ch = idx & 7;
              if (row < vlo || row >= vhi)
                *reinterpret_cast<uint4*>(vrow + h * BS * 128 + row * 128 + ch * 16) = make_uint4(0, 0, 0, 0);
            }
          } else {
            // V^T rows: one BS-token row per head dimension
            for (int dim = lane; dim < D; dim += 32) {
              uint16_t* vr = reinterpret_cast<uint16_t*>(vrow) + dim * BS;
#pragma unroll
              for (int tk = 0; tk < BS; ++tk)
                if (tk < vlo || tk >= vhi) vr[tk] = 0;
            }
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
                  KVL == kKvFlat
                      ? ks + (ch >> 3) * (BS * 128) + tok * 128 + ((((ch & 7) ^ (tok & 7))) << 4)
                      : ks + (ch * BS + tok) * 16;
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
          // O^T += V^T P^T : A = V^T, via ldmatrix.trans of the swizzled V tile (flat)
          // or plain ldmatrix of the V^T rows (vLLM layout)
          {
            const int mq = lane >> 3;
#pragma unroll
            for (int mt = 0; mt < D / 16; ++mt) {
              uint32_t a[4];
              if constexpr (KVL == kKvFlat) {
                const int tok = t * 16 + (lane & 7) + 8 * (mq >> 1);
                const int ch = 2 * mt + (mq & 1);
                const uint32_t addr =
                    vs + (ch >> 3) * (BS * 128) + tok * 128 + ((((ch & 7) ^ (tok & 7))) << 4);
                ldsm_x4_t(addr, a[0], a[1], a[2], a[3]);
              } else {
                const int dim = mt * 16 + (lane & 7) + 8 * (mq & 1);
                const int tok = t * 16 + 8 * (mq >> 1);
                ldsm_x4(vs + (dim * BS + tok) * 2, a[0], a[1], a[2], a[3]);
              }
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

    // ---- this warp's state of the segment into the merge buffers
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
    }  // bf16 / fp16 consumer
    gbase += npg;
    __syncwarp();
    named_bar(1, NCW * 32);

    // A segment that is the whole (sequence, head group) is finished here: as the
    // normalised output row, or (partials mode) as that row's merged partial.
    // Pieces of longer sequences go to this CTA's fixup slot.
    const bool whole = sg.nslots == 1;
    for (int idx = tid; idx < HPC * D; idx += NCW * 32) {
      const int hl = idx / D, dim = idx - hl * D;
      const int gh = sg.hc * HPC + hl;
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
      const size_t row = static_cast<size_t>(sg.seq) * p.num_heads + sg.kvh * G + gh;
      if (whole && direct_final) {
        reinterpret_cast<T*>(p.out)[row * D + dim] = E::cvt(L > 0.f ? O / L : 0.f);
      } else if (whole) {
        emit_partial(row, dim, O, L > 0.f ? M : NEG_INF, L);
      } else {
        const size_t fix = (static_cast<size_t>(blockIdx.x) * 2 + sg.slot) * HPC + hl;
        part_o[fix * D + dim] = O;
        if (dim == 0) {
          part_ml[fix * 2 + 0] = M;
          part_ml[fix * 2 + 1] = L;
        }
      }
    }
    if (!whole && tid == 0) {
      // A piece of a longer sequence: counted in after this CTA's last segment.
      Pending& pd = pend[sg.slot];
      pd.cfirst = sg.cfirst;
      pd.nslots = sg.nslots;
      pd.seq = sg.seq;
      pd.kvh = sg.kvh;
      pd.hc = sg.hc;
      pd.last = 0;
    }
    __syncwarp();
    named_bar(2, NCW * 32);
    sg = sn;
    have = have_n;
    if (have) have_n = it.next(sn);
  }

  // Count this CTA's pieces in (at most two: the chunk's first and last segment)
  // and merge every sequence whose last piece this was. The CTA barrier orders all
  // threads' partial writes before thread 0's fence and counter update (the
  // release); thread 0's fence after the update orders the merge's reads after the
  // other CTAs' releases (the acquire).
  if (flat) {
    named_bar(2, NCW * 32);
    if (tid == 0) {
      // both updates in flight together; acq_rel at GPU scope is the release of this
      // CTA's pieces and the acquire of the earlier arrivals' pieces
      const bool has0 = pend[0].nslots > 1, has1 = pend[1].nslots > 1;
      const int old0 = has0 ? atom_add_acq_rel_gpu(counters + pend[0].cfirst, 1) : 0;
      const int old1 = has1 ? atom_add_acq_rel_gpu(counters + pend[1].cfirst, 1) : 0;
#pragma unroll
      for (int k = 0; k < 2; ++k) {
        Pending& pd = pend[k];
        if (pd.nslots <= 1) continue;
        const int old = k == 0 ? old0 : old1;
        if (old >= pd.nslots) atomicOr(p.err, kErrWorkspace);
        pd.last = old == pd.nslots - 1;
        if (pd.last) st_relaxed_gpu(counters + pd.cfirst, 0);  // zero for the next launch
      }
    }
    named_bar(2, NCW * 32);
#ifdef FE_TIMELINE
    const unsigned long long tm0 = globaltimer_ns();
#endif
    constexpr int PER = D / 32;
    for (int k = 0; k < 2; ++k) {
      const Pending pd = pend[k];
      if (pd.nslots <= 1 || !pd.last) continue;
      for (int hl = warp; hl < HPC; hl += NCW) {
        const int gh = pd.hc * HPC + hl;
        if (gh >= G) break;
        float M, L, acc[PER];
        lse_combine_warp<PER, 8>(
            part_o, part_ml, pd.nslots, D,
            [&](int j) -> size_t {
              // piece j sits in CTA cfirst + j: the first piece in slot 1, the
              // continuations in slot 0
              return (static_cast<size_t>(pd.cfirst + j) * 2 + (j == 0 ? 1 : 0)) * HPC +
                     hl;
            },
            [&](size_t slot) { return slot * D; }, [&](size_t slot) { return slot * 2; }, M, L,
            acc);
        const size_t row = static_cast<size_t>(pd.seq) * p.num_heads + pd.kvh * G + gh;
        const float inv = L > 0.f ? 1.f / L : 0.f;
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          const int dim = lane + 32 * e;
          if (direct_final) {
            reinterpret_cast<T*>(p.out)[row * D + dim] = E::cvt(acc[e] * inv);
          } else {
            emit_partial(row, dim, acc[e], L > 0.f ? M : NEG_INF, L);
          }
        }
      }
    }
#ifdef FE_TIMELINE
    __syncwarp();
    if (tid == 0) g_timeline[blockIdx.x][7] = globaltimer_ns() - tm0;
#endif
  }

  if (tid == 0) FE_TL(4);
}

// ---------------------------------------------------------------------------
// Log-sum-exp merge of partials laid out [ranks, rows, parts_per_rank] (the
// all-gathered per-rank partials of KV-range sharding, or the splits of the dense
// fp32 flash decoding). One warp per output row.
template <int DMAX, int ROWS>
__global__ void __launch_bounds__(256) merge_kernel(const MergeParams mp) {
  constexpr int PER = DMAX / 32;
  const int D = mp.head_dim;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  griddep_wait();  // the producing grid's partials are complete and visible
  for (int rr = warp; rr < ROWS; rr += 8) {
    const int row = blockIdx.x * ROWS + rr;
    if (row >= mp.rows) break;
    const int nparts = mp.parts_per_rank;
    float M, L, acc[PER];
    // part j = (rank j / nparts, split j % nparts)
    const long long rs_o = mp.rank_stride_out ? mp.rank_stride_out
                                              : static_cast<long long>(mp.rows) * nparts * D;
    const long long rs_s = mp.rank_stride_stats ? mp.rank_stride_stats
                                                : static_cast<long long>(mp.rows) * nparts * 2;
    lse_combine_warp<PER, 8>(
        mp.part_out, mp.part_stats, mp.ranks * nparts, D, [&](int j) -> size_t { return j; },
        [&](size_t j) {
          const int rk = static_cast<int>(j) / nparts, pj = static_cast<int>(j) - rk * nparts;
          return rk * rs_o + (static_cast<long long>(row) * nparts + pj) * D;
        },
        [&](size_t j) {
          const int rk = static_cast<int>(j) / nparts, pj = static_cast<int>(j) - rk * nparts;
          return rk * rs_s + (static_cast<long long>(row) * nparts + pj) * 2;
        },
        M, L, acc);
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
}

// ---------------------------------------------------------------------------
// Merge of one KV-range exchange step: each rank's decode stored its (O, m, l) rows
// as step-tagged words into slot [rank] of this buffer. One warp per row loads every
// rank's words of the row at once, re-reads the ones that do not carry this step yet
// (bounded wait), and combines the world partials (src/flash_decoding.cu:151-223
// arithmetic). A wait that runs out sets kErrWaitTimeout and the row is written as
// zeros. The last CTA advances the step count.
template <int DMAX, int ROWS>
__global__ void __launch_bounds__(256) xmerge_kernel(const XMergeParams xp) {
  constexpr int PER = DMAX / 32;
  // Launched with programmatic dependent launch: the CTAs may be placed while this
  // GPU's decode is still finishing; griddepcontrol.wait holds them until it has
  // completed, so the re-reads below only ever wait for other GPUs.
  griddep_launch_dependents();
  griddep_wait();
  XHeader* h = reinterpret_cast<XHeader*>(xp.xbuf);
  const unsigned step = ld_volatile_u32(&h->step) + 1u;  // the step being merged
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int D = xp.head_dim, W = xp.world;
  const int par = static_cast<int>(step & 1u);
  const unsigned long long* words =
      reinterpret_cast<const unsigned long long*>(xp.xbuf + sizeof(XHeader));
  const unsigned long long t0 = globaltimer_ns();
  // Re-reads *w until its tag is `step`; false once the wait limit has passed.
  auto settle = [&](const unsigned long long* addr, unsigned long long& w) -> bool {
    while (static_cast<unsigned>(w >> 32) != step) {
      if (globaltimer_ns() - t0 > kWaitLimitNs) return false;
      w = ld_volatile_u64(addr);
    }
    return true;
  };
  for (int rr = warp; rr < ROWS; rr += 8) {
    const int row = blockIdx.x * ROWS + rr;
    if (row >= xp.rows) break;
    // stats of rank `lane`, O words of every rank for this lane's dims: one round trip
    unsigned long long wm = 0, wl = 0;
    const unsigned long long* am = nullptr;
    if (lane < W) {
      am = words + x_ml_word(par, W, lane, xp.max_rows, row, D);
      wm = ld_volatile_u64(am);
      wl = ld_volatile_u64(am + 1);
    }
    unsigned long long wo[kMaxRanks][PER];
#pragma unroll
    for (int j = 0; j < kMaxRanks; ++j) {
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        const int dim = lane + 32 * e;
        wo[j][e] = (j < W && dim < D)
                       ? ld_volatile_u64(words + x_o_word(par, W, j, xp.max_rows, row, D) + dim)
                       : (static_cast<unsigned long long>(step) << 32);
      }
    }
    bool ok = true;
    if (lane < W) ok = settle(am, wm) && settle(am + 1, wl);
#pragma unroll
    for (int j = 0; j < kMaxRanks; ++j) {
#pragma unroll
      for (int e = 0; e < PER; ++e) {
        const int dim = lane + 32 * e;
        if (j < W && dim < D && ok)
          ok = settle(words + x_o_word(par, W, j, xp.max_rows, row, D) + dim, wo[j][e]);
      }
    }
    ok = __all_sync(0xffffffffu, ok);
    if (!ok && lane == 0) atomicOr(xp.err, kErrWaitTimeout);
    const float m = __uint_as_float(static_cast<unsigned>(wm));
    const float l = lane < W ? __uint_as_float(static_cast<unsigned>(wl)) : 0.f;
    float M = l > 0.f ? m : NEG_INF;
    M = flash_engine::cuda::warp_reduce_max(M);
    const float wgt = l > 0.f ? ex2(m - M) : 0.f;
    float L = l * wgt;
    L = flash_engine::cuda::warp_reduce_sum(L);
    float acc[PER];
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxRanks; ++j) {
      const float wj = __shfl_sync(0xffffffffu, wgt, j);
#pragma unroll
      for (int e = 0; e < PER; ++e)
        acc[e] += (j < W ? __uint_as_float(static_cast<unsigned>(wo[j][e])) : 0.f) * wj;
    }
    const float inv = (ok && L > 0.f) ? 1.f / L : 0.f;
#pragma unroll
    for (int e = 0; e < PER; ++e) {
      const int dim = lane + 32 * e;
      if (dim >= D) continue;
      const size_t oi = static_cast<size_t>(row) * D + dim;
      if (xp.out_dtype == 0) {
        reinterpret_cast<float*>(xp.out)[oi] = acc[e] * inv;
      } else if (xp.out_dtype == 1) {
        reinterpret_cast<__nv_bfloat16*>(xp.out)[oi] = __float2bfloat16_rn(acc[e] * inv);
      } else {
        reinterpret_cast<half*>(xp.out)[oi] = __float2half_rn(acc[e] * inv);
      }
    }
  }
  // The last CTA of this merge advances the step (read by the next decode and merge).
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&h->merge_ctas, 1u) == gridDim.x - 1) {
      atomicExch(&h->merge_ctas, 0u);
      atomicExch(&h->step, step);
    }
  }
}

// ---------------------------------------------------------------------------
// host launch

template <typename T, int D, int BS, int NT, int KVL>
static cudaError_t launch_cfg(const Params& p, const void* kc, const void* vc, long long kv_rows,
                              int* grid_out, cudaStream_t stream) {
  constexpr int NCW = 4;
  // NCW consumer warps x DEPTH private stages each; ~64 KB of stages per CTA.
  constexpr int NSTAGE = NCW * ring_depth<T, D, BS, NCW>();
  using C = Cfg<T, D, BS, NT, NCW, NSTAGE>;
  auto kern = paged_decode_kernel<T, D, BS, NT, NCW, NSTAGE, KVL>;
  const int smem = C::smem_bytes(p.num_seqs);
  cudaError_t e = ensure_smem_optin(reinterpret_cast<const void*>(kern), smem);
  if (e != cudaSuccess) return e;
  CUtensorMap km = {}, vm = {};
  if (KVL == kKvFlat && !C::F32) {
    const bool bf16 = std::is_same<T, __nv_bfloat16>::value;
    e = encode_tma_2d_b16(&km, kc, bf16, D, kv_rows, D, 64, BS);
    if (e != cudaSuccess) return e;
    e = encode_tma_2d_b16(&vm, vc, bf16, D, kv_rows, D, 64, BS);
    if (e != cudaSuccess) return e;
  }
  int occ = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, C::NTHREADS, smem);
  if (e != cudaSuccess) return e;
  if (occ < 1) return cudaErrorInvalidConfiguration;
#ifdef FE_DECODE_CTAS_PER_SM
  occ = min(occ, FE_DECODE_CTAS_PER_SM);  // build-time tuning of the resident grid
#endif
  int grid = min(sm_count() * occ, kCounterSlots);
  if (p.max_grid > 0) grid = min(grid, p.max_grid);
  if (grid_out) *grid_out = grid;
  Params pp = p;
  pp.dbg_kv_rows = kv_rows;
  pp.k_cache = kc;
  pp.v_cache = vc;
  // programmatic dependent launch: see the top of paged_decode_kernel
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(C::NTHREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, km, vm, pp);
}

template <typename T>
cudaError_t launch_decode(const Params& p, int head_dim, int block_size, const void* kc,
                          const void* vc, long long kv_rows, int nt, int kv_layout, int* grid_out,
                          cudaStream_t stream) {
#define FE_CASE(D_, BS_, NT_, L_)                                                   \
  if (head_dim == D_ && block_size == BS_ && nt == NT_ && kv_layout == L_)          \
    return launch_cfg<T, D_, BS_, NT_, L_>(p, kc, vc, kv_rows, grid_out, stream);
  FE_CASE(128, 16, 1, kKvFlat)
  FE_CASE(128, 16, 2, kKvFlat)
  FE_CASE(64, 16, 1, kKvFlat)
  FE_CASE(64, 16, 2, kKvFlat)
  FE_CASE(128, 32, 1, kKvFlat)
  FE_CASE(128, 32, 2, kKvFlat)
  FE_CASE(64, 32, 1, kKvFlat)
  FE_CASE(64, 32, 2, kKvFlat)
  if constexpr (!std::is_same<T, float>::value) {
    FE_CASE(128, 16, 1, kKvVllm)
    FE_CASE(128, 16, 2, kKvVllm)
    FE_CASE(64, 16, 1, kKvVllm)
    FE_CASE(64, 16, 2, kKvVllm)
  }
#undef FE_CASE
  return cudaErrorInvalidValue;
}

template <typename T, int D, int BS, int NT>
static long long grid_max_cfg() {
  constexpr int NCW = 4;
  constexpr int NSTAGE = NCW * ring_depth<T, D, BS, NCW>();
  using C = Cfg<T, D, BS, NT, NCW, NSTAGE>;
  auto kern = paged_decode_kernel<T, D, BS, NT, NCW, NSTAGE, kKvFlat>;
  const int smem = C::smem_bytes(1);
  if (ensure_smem_optin(reinterpret_cast<const void*>(kern), smem) != cudaSuccess) return -1;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, C::NTHREADS, smem) != cudaSuccess)
    return -1;
  const long long g = static_cast<long long>(sm_count()) * (occ > 0 ? occ : 1);
  return g < kCounterSlots ? g : kCounterSlots;
}

template <typename T>
static long long grid_max_of(int head_dim, int block_size, int nt) {
  long long g = -1;
#define FE_CASE(D_, BS_, NT_)                                                           \
  if (head_dim == D_ && block_size == BS_ && nt == NT_) g = grid_max_cfg<T, D_, BS_, NT_>();
  FE_CASE(128, 16, 1) FE_CASE(128, 16, 2) FE_CASE(64, 16, 1) FE_CASE(64, 16, 2)
  FE_CASE(128, 32, 1) FE_CASE(128, 32, 2) FE_CASE(64, 32, 1) FE_CASE(64, 32, 2)
#undef FE_CASE
  return g;
}

FixupLayout fixup_layout(int dtype, int head_dim, int block_size, int nt) {
  // bf16 and fp16 kernels share their shapes and occupancy
  const long long g = dtype == kF32 ? grid_max_of<float>(head_dim, block_size, nt)
                                    : grid_max_of<__nv_bfloat16>(head_dim, block_size, nt);
  FixupLayout f{-1, 0, -1};
  if (g < 0) return f;
  f.grid_max = g;
  f.slot_rows = g * 2 * heads_per_cta(dtype, nt);
  f.floats = kCounterSlots + f.slot_rows * (head_dim + 2);
  return f;
}

cudaError_t launch_xmerge(const XMergeParams& xp, cudaStream_t stream) {
  if (xp.rows <= 0) return cudaSuccess;
  if (xp.world < 1 || xp.world > kMaxRanks || xp.head_dim < 1) return cudaErrorInvalidValue;
  constexpr int ROWS = 8;
  const dim3 grid((xp.rows + ROWS - 1) / ROWS);
  void (*kern)(XMergeParams) = nullptr;
  if (xp.head_dim <= 64) kern = xmerge_kernel<64, ROWS>;
  else if (xp.head_dim <= 128) kern = xmerge_kernel<128, ROWS>;
  else return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, xp);
}

// ---------------------------------------------------------------------------
// Cache append of the decode step's new token: K and V rows of sequence s (position
// context_lens[s] - 1) are written into row pos % BS of physical block
// block_tables[s, pos / BS], K rotated at that position first when tables are given
// (pairs (2i, 2i+1): x0 c - x1 s, x0 s + x1 c, src/fused_rope.cu:33-43). One CTA per
// sequence, one thread per (KV head, pair). Not launched with programmatic dependent
// launch, so a decode that follows on the stream starts after it completes.
template <typename T>
__device__ __forceinline__ float to_f(T x) { return static_cast<float>(x); }
template <typename T>
__device__ __forceinline__ T from_f(float x) { return static_cast<T>(x); }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <>
__device__ __forceinline__ half from_f<half>(float x) { return __float2half_rn(x); }

template <typename T>
__global__ void __launch_bounds__(256) kv_append_kernel(const AppendParams ap) {
  const int s = blockIdx.x;
  const int pos = __ldg(ap.context_lens + s) - 1;
  if (pos < 0) return;
  const int half_d = ap.head_dim / 2;
  const int blk = pos / ap.block_size, off = pos % ap.block_size;
  if (blk >= ap.max_blocks_per_seq) {
    if (threadIdx.x == 0) atomicOr(ap.err, kErrBadBlock);
    return;
  }
  const int phys = __ldg(ap.block_tables + static_cast<size_t>(s) * ap.max_blocks_per_seq + blk);
  if (phys < 0 || (ap.num_blocks > 0 && phys >= ap.num_blocks)) {
    if (threadIdx.x == 0) atomicOr(ap.err, kErrBadBlock);
    return;
  }
  const bool rope = ap.rope_cos != nullptr;
  if (rope && pos >= ap.rope_max_pos) {
    if (threadIdx.x == 0) atomicOr(ap.err, kErrBadBlock);
    return;
  }
  const T* kn = static_cast<const T*>(ap.k_new);
  const T* vn = static_cast<const T*>(ap.v_new);
  T* kc = static_cast<T*>(ap.k_cache);
  T* vc = static_cast<T*>(ap.v_cache);
  const int D = ap.head_dim, BS = ap.block_size;
  for (int idx = threadIdx.x; idx < ap.num_kv_heads * half_d; idx += blockDim.x) {
    const int h = idx / half_d, i = idx - h * half_d;
    const size_t src = (static_cast<size_t>(s) * ap.num_kv_heads + h) * D + 2 * i;
    float k0 = to_f(kn[src]), k1 = to_f(kn[src + 1]);
    if (rope) {
      const float c = __ldg(ap.rope_cos + static_cast<size_t>(pos) * half_d + i);
      const float sn = __ldg(ap.rope_sin + static_cast<size_t>(pos) * half_d + i);
      const float r0 = k0 * c - k1 * sn, r1 = k0 * sn + k1 * c;
      k0 = r0;
      k1 = r1;
    }
    const size_t page = static_cast<size_t>(phys) * ap.num_kv_heads + h;  // (block, KV head)
    for (int e = 0; e < 2; ++e) {
      const int dim = 2 * i + e;
      size_t kd, vd;
      if (ap.kv_layout == kKvFlat) {
        kd = vd = (page * BS + off) * D + dim;
      } else {  // vLLM: K [.., D/8, BS, 8], V [.., D, BS]
        kd = ((page * (D / 8) + dim / 8) * BS + off) * 8 + dim % 8;
        vd = (page * D + dim) * BS + off;
      }
      kc[kd] = from_f<T>(e == 0 ? k0 : k1);
      vc[vd] = vn[src + e];
    }
  }
}

template <typename T>
cudaError_t launch_kv_append(const AppendParams& ap, cudaStream_t stream) {
  if (ap.num_seqs <= 0) return cudaSuccess;
  kv_append_kernel<T><<<ap.num_seqs, 256, 0, stream>>>(ap);
  return cudaGetLastError();
}
template cudaError_t launch_kv_append<__nv_bfloat16>(const AppendParams&, cudaStream_t);
template cudaError_t launch_kv_append<half>(const AppendParams&, cudaStream_t);
template cudaError_t launch_kv_append<float>(const AppendParams&, cudaStream_t);

#ifdef FE_TIMELINE
extern "C" int fe_debug_timeline(unsigned long long* host, int ctas) {
  if (ctas > kCounterSlots) ctas = kCounterSlots;
  return static_cast<int>(
      cudaMemcpyFromSymbol(host, g_timeline, sizeof(unsigned long long) * 12 * ctas));
}
#endif

template cudaError_t launch_decode<__nv_bfloat16>(const Params&, int, int, const void*, const void*,
                                                  long long, int, int, int*, cudaStream_t);
template cudaError_t launch_decode<half>(const Params&, int, int, const void*, const void*,
                                         long long, int, int, int*, cudaStream_t);
template cudaError_t launch_decode<float>(const Params&, int, int, const void*, const void*,
                                          long long, int, int, int*, cudaStream_t);

cudaError_t launch_merge(const MergeParams& mp, int head_dim, cudaStream_t stream) {
  if (mp.rows <= 0) return cudaSuccess;
  constexpr int ROWS = 8;  // one row per warp
  MergeParams m2 = mp;
  m2.head_dim = head_dim;
  if (head_dim < 1) return cudaErrorInvalidValue;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((mp.rows + ROWS - 1) / ROWS);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  void (*kern)(MergeParams) = nullptr;
  if (head_dim <= 64) kern = merge_kernel<64, ROWS>;
  else if (head_dim <= 128) kern = merge_kernel<128, ROWS>;
  else if (head_dim <= 256) kern = merge_kernel<256, ROWS>;
  else return cudaErrorInvalidValue;
  return cudaLaunchKernelEx(&cfg, kern, m2);
}

}  // namespace paged
}  // namespace fe
