// Public entry points of libflash_engine_b200.so: the extern "C" ABI declared in
// include/flash_engine_c.h and the C++ launchers declared in include/*.cuh with
// the reference's namespaces and signatures. Argument validation happens here;
// the kernels live in paged_decode.cu, attention_fp32.cu and prefill_sm100.cu.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <dlfcn.h>
#include <limits.h>
#include <nccl.h>  // types only: the functions are resolved at run time
#include <math.h>
#include <stdint.h>

#include <string.h>

#include <algorithm>
#include <map>
#include <mutex>
#include <thread>
#include <tuple>
#include <type_traits>
#include <utility>

#include "../../include/flash_engine.h"
#include "fp32_kernels.h"
#include "internal.h"
#include "paged_decode.h"
#include "prefill.h"
#include "ptx.cuh"
#include "rope.h"

namespace {

inline float resolve_scale(float s, int d) { return s > 0.f ? s : 1.0f / sqrtf(static_cast<float>(d)); }
inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
constexpr int kMaxSeqsPerLaunch = 4096;
// Pages of streaming that a sequence start inside a CTA's chunk costs the flat-mode
// decode (segment change, partial writes, piece count-in), measured per CTA with
// %globaltimer on the config 3 / 5 shard shapes: about 2.5-3.5 us, 6-8 pages. Swept
// over 0/6/8/10 on those shapes: 8 is the best (config 3: 108.0 -> 104.8 us at N = 1,
// 22.3 -> 20.5 us on the N = 8 shard; config 5 N = 8 shard: 55.1 -> 47.5 us).
#ifndef FE_DECODE_SEG_COST
#define FE_DECODE_SEG_COST 8
#endif
constexpr int kSegCostPages = FE_DECODE_SEG_COST;
constexpr int kErr = static_cast<int>(cudaErrorInvalidValue);

bool dense_args_ok(int B, int H, int N, int M, int d) {
  return B >= 0 && H >= 0 && N >= 0 && M >= 1 && d >= 1;
}

struct PagedArgs {
  const void* q;
  const void* kc;
  const void* vc;
  void* out;
  const int* bt;
  const int* lens;
  int S, H, Hkv, d, bs, max_ctx, maxb, num_blocks;
  float scale;
  int kv_layout = fe::paged::kKvFlat;
  const float* rope_cos = nullptr;
  const float* rope_sin = nullptr;
  int rope_max_pos = 0;
};

template <typename T>
constexpr int dtype_of() {
  return std::is_same<T, float>::value ? fe::paged::kF32
         : std::is_same<T, half>::value ? fe::paged::kF16
                                        : fe::paged::kBf16;
}

// Shapes the persistent decode kernel takes (paged_decode.cu): head_dim 64 or 128,
// block size 16 or 32, 16-byte aligned caches; the fp32 decode reads the flat layout
// with 128-bit (d = 128) or 64-bit (d = 64) q loads.
template <typename T>
int paged_check(const PagedArgs& a) {
  if (a.S < 0 || a.H <= 0 || a.Hkv <= 0 || a.H % a.Hkv != 0 || a.d <= 0 || a.bs <= 0 ||
      a.maxb < 0)
    return kErr;
  if (!(a.d == 64 || a.d == 128) || !(a.bs == 16 || a.bs == 32)) return kErr;
  if (a.kv_layout != fe::paged::kKvFlat && a.kv_layout != fe::paged::kKvVllm) return kErr;
  if (a.kv_layout == fe::paged::kKvVllm && (a.bs != 16 || std::is_same<T, float>::value))
    return kErr;
  if (!aligned(a.kc, 16) || !aligned(a.vc, 16)) return kErr;
  if (std::is_same<T, float>::value) {
    if (!aligned(a.q, a.d == 128 ? 16 : 8) || !aligned(a.out, 4)) return kErr;
  } else if (!aligned(a.q, 4) || !aligned(a.out, 2)) {
    return kErr;
  }
  if (a.num_blocks > 0 &&
      static_cast<long long>(a.num_blocks) * a.Hkv * a.bs > static_cast<long long>(INT_MAX))
    return kErr;
  return 0;
}

// Arguments the generic fp32 kernels (attention_fp32.cu) take.
int paged_check_generic(const PagedArgs& a) {
  if (a.S < 0 || a.H <= 0 || a.Hkv <= 0 || a.H % a.Hkv != 0 || a.d <= 0 || a.bs <= 0 ||
      a.maxb < 0)
    return kErr;
  if (a.d > 256 || a.d % 4 != 0) return kErr;
  return 0;
}

// How the tensor-core decode cuts and finishes the work.
struct DecodePlan {
  int tok_begin = 0, tok_end = INT_MAX;
  bool flat = false;          // stream-K chunking with fixup partials (needs workspace)
  bool direct_final = true;   // normalised output rows (else merged partials)
  float* merged_out = nullptr;
  float* merged_stats = nullptr;
  // exchange mode (partials stored into every rank's exchange buffer)
  char* xbuf[fe::paged::kMaxRanks] = {};
  int xworld = 0, xrank = 0, xmax_rows = 0;
  // flat mode on a slot of the library's stream scratch instead of `ws`
  int ws_slot = -1;
};

inline int decode_nt(int dtype, int H, int Hkv) { return fe::paged::decode_nt(dtype, H / Hkv); }

long long workspace_floats_dtype(int dtype, int H, int Hkv, int d, int bs) {
  if (H <= 0 || Hkv <= 0 || H % Hkv) return -1;
  return fe::paged::fixup_layout(dtype, d, bs, decode_nt(dtype, H, Hkv)).floats;
}

// Workspace of the split-KV decode for this head configuration: the largest over the
// element types, so that one workspace serves bf16, fp16 and fp32 calls.
long long workspace_floats_for(int H, int Hkv, int d, int bs) {
  const long long a = workspace_floats_dtype(fe::paged::kBf16, H, Hkv, d, bs);
  const long long b = workspace_floats_dtype(fe::paged::kF32, H, Hkv, d, bs);
  return a < 0 || b < 0 ? -1 : std::max(a, b);
}

// Runs the tensor-core decode over all sequences, in launches of at most
// kMaxSeqsPerLaunch sequences. In flat mode `ws` holds the arrival counters and
// fixup slots (fixup_layout); the kernel merges split sequences itself.
template <typename T>
int paged_tc_run(const PagedArgs& a, const DecodePlan& pl, float* ws, cudaStream_t st) {
  constexpr int dt = dtype_of<T>();
  const int nt = decode_nt(dt, a.H, a.Hkv);
  const int hpc = fe::paged::heads_per_cta(dt, nt);
  const int head_chunks = (a.H / a.Hkv + hpc - 1) / hpc;
  const long long kv_rows = a.num_blocks > 0
                                ? static_cast<long long>(a.num_blocks) * a.Hkv * a.bs
                                : static_cast<long long>(INT_MAX);
  unsigned* err = fe::device_error_word();
  if (!err) return static_cast<int>(cudaErrorInitializationError);
  float* part_o = nullptr;
  float* part_ml = nullptr;
  int* counters = nullptr;
  int max_grid = 0;
  if (pl.flat && pl.ws_slot >= 0) {
    max_grid = fe::paged::slot_grid_cap(dt, a.d, nt);
  } else if (pl.flat) {
    const fe::paged::FixupLayout f = fe::paged::fixup_layout(dt, a.d, a.bs, nt);
    if (f.floats <= 0 || !ws) return kErr;
    counters = reinterpret_cast<int*>(ws);
    part_o = ws + fe::paged::kCounterSlots;
    part_ml = part_o + f.slot_rows * a.d;
  }
  for (int s0 = 0; s0 < a.S; s0 += kMaxSeqsPerLaunch) {
    const int n = a.S - s0 < kMaxSeqsPerLaunch ? a.S - s0 : kMaxSeqsPerLaunch;
    const size_t row0 = static_cast<size_t>(s0) * a.H;
    fe::paged::Params p{};
    p.q = static_cast<const T*>(a.q) + row0 * a.d;
    p.out = a.out ? static_cast<T*>(a.out) + row0 * a.d : nullptr;
    p.block_tables = a.bt + static_cast<size_t>(s0) * a.maxb;
    p.context_lens = a.lens + s0;
    p.part_o = part_o;
    p.part_ml = part_ml;
    p.counters = counters;
    p.ws_slot = pl.flat ? pl.ws_slot : -1;
    p.max_grid = max_grid;
    p.merged_o = pl.merged_out ? pl.merged_out + row0 * a.d : nullptr;
    p.merged_ml = pl.merged_stats ? pl.merged_stats + row0 * 2 : nullptr;
    p.num_seqs = n;
    p.num_heads = a.H;
    p.num_kv_heads = a.Hkv;
    p.max_blocks_per_seq = a.maxb;
    p.num_phys_blocks = a.num_blocks;
    p.head_chunks = head_chunks;
    p.tok_begin = pl.tok_begin;
    p.tok_end = pl.tok_end;
    p.pages_per_split = pl.flat ? 1 : INT_MAX / 2;
    p.seg_cost_pages = pl.flat ? kSegCostPages : 0;
    p.flat = pl.flat ? 1 : 0;
    p.direct_final = pl.direct_final ? 1 : 0;
    p.scale_log2 = resolve_scale(a.scale, a.d) * fe::kLog2e;
    p.rope_cos = a.rope_cos;
    p.rope_sin = a.rope_sin;
    p.rope_max_pos = a.rope_max_pos;
    p.err = err;
    for (int r = 0; r < fe::paged::kMaxRanks; ++r) p.xbuf[r] = pl.xbuf[r];
    p.xworld = pl.xworld;
    p.xrank = pl.xrank;
    p.xmax_rows = pl.xmax_rows;
    const cudaError_t e = fe::paged::launch_decode<T>(p, a.d, a.bs, a.kc, a.vc, kv_rows, nt,
                                                      a.kv_layout, nullptr, st);
    if (e != cudaSuccess) return static_cast<int>(e);
  }
  return 0;
}

template <typename T>
int paged_v1_tc(const PagedArgs& a, cudaStream_t st) {
  const int rc = paged_check<T>(a);
  if (rc) return rc;
  if (a.S == 0) return 0;
  // Unit mode, one segment per sequence whatever its length: every segment
  // writes its final rows, no scratch.
  DecodePlan pl;
  return paged_tc_run<T>(a, pl, nullptr, st);
}

template <typename T>
int paged_v2_tc(const PagedArgs& a, float* ws, size_t ws_floats, cudaStream_t st) {
  const int rc = paged_check<T>(a);
  if (rc) return rc;
  const long long need = workspace_floats_dtype(dtype_of<T>(), a.H, a.Hkv, a.d, a.bs);
  if (need <= 0 || !ws || static_cast<long long>(ws_floats) < need) return kErr;
  if (a.S == 0) return 0;
  DecodePlan pl;
  pl.flat = true;
  pl.direct_final = true;
  return paged_tc_run<T>(a, pl, ws, st);
}

// Split-KV scratch for the entry points whose reference signature passes none (the
// v1 paged launchers), which may not allocate: the kStreamSlots slots of the static
// array in paged_decode.cu. A slot is bound to a stream on the first v1 call on that
// stream and stays bound for the life of the process, so work captured into a CUDA
// graph keeps a valid slot. Calls on one stream are ordered and can share its slot.
// The per-thread default stream is one handle for every thread, so it is keyed with
// the calling thread as well. Returns -1 once every slot is bound (those streams run
// the single-pass kernel). Binding allocates nothing on the device and does not
// synchronise, so it is also allowed while the stream is being captured.
int stream_slot(cudaStream_t st) {
  static std::mutex mu;
  static std::map<std::tuple<int, uintptr_t, std::thread::id>, int> bound;
  static int used[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  const std::thread::id tid =
      st == cudaStreamPerThread ? std::this_thread::get_id() : std::thread::id();
  const auto key = std::make_tuple(dev, reinterpret_cast<uintptr_t>(st), tid);
  std::lock_guard<std::mutex> lk(mu);
  auto it = bound.find(key);
  if (it != bound.end()) return it->second;
  if (used[dev] >= fe::paged::kStreamSlots) return -1;
  const int slot = used[dev]++;
  bound.emplace(key, slot);
  return slot;
}

// The reference's v1 entry points: the split-KV kernel on the stream's scratch slot
// (the single-pass kernel when every slot is taken).
template <typename T>
int paged_v1_entry(const PagedArgs& a, cudaStream_t st) {
  const int rc = paged_check<T>(a);
  if (rc) return rc;
  if (a.S == 0) return 0;
  const int slot = stream_slot(st);
  if (slot < 0) return paged_v1_tc<T>(a, st);
  DecodePlan pl;
  pl.flat = true;
  pl.direct_final = true;
  pl.ws_slot = slot;
  return paged_tc_run<T>(a, pl, nullptr, st);
}

// NCCL, resolved at run time from the libnccl.so.2 the process already holds (e.g.
// the one PyTorch loaded), else the system one; the library does not link NCCL.
struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t,
                             cudaStream_t);
  bool ok;
};
const NcclApi& nccl_api() {
  static const NcclApi api = [] {
    NcclApi a{};
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h) {
      a.get_unique_id = reinterpret_cast<decltype(a.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
      a.comm_init_rank = reinterpret_cast<decltype(a.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
      a.comm_destroy = reinterpret_cast<decltype(a.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
      a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
    }
    a.ok = a.get_unique_id && a.comm_init_rank && a.comm_destroy && a.all_gather;
    return a;
  }();
  return api;
}
constexpr int kNcclErrBase = 1000;  // status = 1000 + ncclResult_t for NCCL failures
inline int nccl_status(ncclResult_t r) { return r == ncclSuccess ? 0 : kNcclErrBase + static_cast<int>(r); }

// Token window of `rank` under KV-range sharding: ceil(M / world) rounded up to whole
// blocks (the split rule of python/flash_engine/ops.py:112-121 across GPUs); the last
// rank ends at M; an empty window is [0, 0).
void kv_range_window(int M, int world, int rank, int bs, int* tb, int* te) {
  const int mm = M > 1 ? M : 1;
  int per = (mm + world - 1) / world;
  per = (per + bs - 1) / bs * bs;
  const long long b = std::min<long long>(static_cast<long long>(rank) * per, M);
  const long long e = rank == world - 1 ? M : std::min<long long>(static_cast<long long>(rank + 1) * per, M);
  *tb = static_cast<int>(b);
  *te = static_cast<int>(e);
  if (*te <= *tb) *tb = *te = 0;
}

}  // namespace

// =========================================================================
// extern "C"
extern "C" {

int fe_flash_attention_forward_fp32(const float* q, const float* k, const float* v, float* o,
                                    int B, int H, int N, int M, int d, int causal, float scale,
                                    void* stream) {
  if (!dense_args_ok(B, H, N, M, d) || d > 128) return kErr;
  if (B * H == 0 || N == 0) return 0;
  return static_cast<int>(fe::simt::launch_fa2_fp32(q, k, v, o, B, H, N, M, d,
                                                    resolve_scale(scale, d), causal,
                                                    as_stream(stream)));
}

int fe_naive_attention_forward_fp32(const float* q, const float* k, const float* v, float* o,
                                    int B, int H, int N, int M, int d, int causal, float scale,
                                    void* stream) {
  if (!dense_args_ok(B, H, N, M, d) || d > 256) return kErr;
  if (B * H == 0 || N == 0) return 0;
  return static_cast<int>(fe::simt::launch_naive_fp32(q, k, v, o, B, H, N, M, d,
                                                      resolve_scale(scale, d), causal,
                                                      as_stream(stream)));
}

int fe_flash_attention_forward_bf16(const void* q, const void* k, const void* v, void* o, int B,
                                    int H, int N, int M, int d, int causal, float scale,
                                    void* stream) {
  if (!dense_args_ok(B, H, N, M, d)) return kErr;
  if (B * H == 0 || N == 0) return 0;
  return static_cast<int>(fe::prefill::launch_prefill(q, k, v, o, B, H, N, M, d, causal,
                                                      resolve_scale(scale, d), true,
                                                      as_stream(stream)));
}

int fe_flash_attention_forward_fp16(const void* q, const void* k, const void* v, void* o, int B,
                                    int H, int N, int M, int d, int causal, float scale,
                                    void* stream) {
  if (!dense_args_ok(B, H, N, M, d)) return kErr;
  if (B * H == 0 || N == 0) return 0;
  return static_cast<int>(fe::prefill::launch_prefill(q, k, v, o, B, H, N, M, d, causal,
                                                      resolve_scale(scale, d), false,
                                                      as_stream(stream)));
}

int fe_rope_forward(const void* in, const float* cos_table, const float* sin_table, void* out,
                    int B, int H, int seq_len, int head_dim, int dtype, void* stream) {
  if (B < 0 || H < 0 || seq_len < 0 || head_dim < 2 || head_dim % 2 || dtype < 0 || dtype > 2 ||
      !cos_table || !sin_table)
    return kErr;
  if (B * H == 0 || seq_len == 0) return 0;
  return static_cast<int>(fe::rope::launch_rope(in, cos_table, sin_table, out, B, H, seq_len,
                                                head_dim, dtype, as_stream(stream)));
}

int fe_flash_attention_forward_ex(const void* q, const void* k, const void* v, void* o, int B,
                                  int H, int N, int M, int d, int causal, float scale, int dtype,
                                  const float* rope_cos, const float* rope_sin, int rope_max_pos,
                                  void* q_rotated, void* k_rotated, void* stream) {
  if (!dense_args_ok(B, H, N, M, d) || (dtype != 0 && dtype != 1)) return kErr;
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return kErr;
  if (rope_cos && (rope_max_pos < N || rope_max_pos < M || !q_rotated || !k_rotated))
    return kErr;
  if (B * H == 0 || N == 0) return 0;
  cudaStream_t st = as_stream(stream);
  const void* qq = q;
  const void* kk = k;
  if (rope_cos) {
    // Q and K rotated once each by one streaming RoPE launch into the caller's buffers
    // (each key tile is read by every query tile of its head, so rotating it inside the
    // attention kernel would repeat the work; k_rotated keeps the keys a KV cache stores)
    const cudaError_t e = fe::rope::launch_rope_qk(q, k, rope_cos, rope_sin, q_rotated, k_rotated,
                                                   B, H, N, M, d, dtype, st);
    if (e != cudaSuccess) return static_cast<int>(e);
    qq = q_rotated;
    kk = k_rotated;
  }
  return static_cast<int>(fe::prefill::launch_prefill(qq, kk, v, o, B, H, N, M, d, causal,
                                                      resolve_scale(scale, d), dtype == 0, st));
}

int fe_paged_attention_v1_fp32(const float* q, const float* kc, const float* vc, float* out,
                               const int* bt, const int* lens, int S, int H, int Hkv, int d,
                               int bs, int max_ctx, int maxb, int num_blocks, float scale,
                               void* stream) {
  PagedArgs a{q, kc, vc, out, bt, lens, S, H, Hkv, d, bs, max_ctx, maxb, num_blocks, scale};
  cudaStream_t st = as_stream(stream);
  // The persistent split-KV decode where its shapes allow (paged_decode.cu), else the
  // generic single-pass kernel (any block size, head_dim % 4 == 0 up to 256).
  if (paged_check<float>(a) == 0) return paged_v1_entry<float>(a, st);
  const int rc = paged_check_generic(a);
  if (rc) return rc;
  if (S == 0) return 0;
  return static_cast<int>(fe::simt::launch_paged_fp32(q, kc, vc, out, bt, lens, S, H, Hkv, d, bs,
                                                      maxb, num_blocks, resolve_scale(scale, d),
                                                      st));
}

int fe_paged_attention_v1_fp16(const void* q, const void* kc, const void* vc, void* out,
                               const int* bt, const int* lens, int S, int H, int Hkv, int d,
                               int bs, int max_ctx, int maxb, int num_blocks, float scale,
                               void* stream) {
  PagedArgs a{q, kc, vc, out, bt, lens, S, H, Hkv, d, bs, max_ctx, maxb, num_blocks, scale};
  a.kv_layout = fe::paged::kKvVllm;  // the layout include/paged_attention.cuh:29-30 declares
  return paged_v1_entry<half>(a, as_stream(stream));
}

int fe_paged_attention_ex(const void* q, const void* kc, const void* vc, void* out,
                          const int* bt, const int* lens, int S, int H, int Hkv, int d, int bs,
                          int maxb, int num_blocks, float scale, int dtype, int kv_layout,
                          const float* rope_cos, const float* rope_sin, int rope_max_pos,
                          float* workspace, size_t workspace_floats, void* stream) {
  PagedArgs a{q, kc, vc, out, bt, lens, S, H, Hkv, d, bs, 0, maxb, num_blocks, scale};
  a.kv_layout = kv_layout;
  if ((rope_cos == nullptr) != (rope_sin == nullptr)) return kErr;
  if (rope_cos && rope_max_pos < 1) return kErr;
  a.rope_cos = rope_cos;
  a.rope_sin = rope_sin;
  a.rope_max_pos = rope_max_pos;
  cudaStream_t st = as_stream(stream);
  if (!workspace && workspace_floats == FE_WORKSPACE_LIBRARY) {
    // split-KV on the stream's slot of the library scratch (as the v1 entries)
    if (dtype == 0) return paged_v1_entry<__nv_bfloat16>(a, st);
    if (dtype == 1) return paged_v1_entry<half>(a, st);
    if (dtype == 2) return paged_v1_entry<float>(a, st);
    return kErr;
  }
  if (dtype == 0) {
    return workspace ? paged_v2_tc<__nv_bfloat16>(a, workspace, workspace_floats, st)
                     : paged_v1_tc<__nv_bfloat16>(a, st);
  }
  if (dtype == 1) {
    return workspace ? paged_v2_tc<half>(a, workspace, workspace_floats, st)
                     : paged_v1_tc<half>(a, st);
  }
  if (dtype == 2) {
    return workspace ? paged_v2_tc<float>(a, workspace, workspace_floats, st)
                     : paged_v1_tc<float>(a, st);
  }
  return kErr;
}

int fe_paged_attention_v1_bf16(const void* q, const void* kc, const void* vc, void* out,
                               const int* bt, const int* lens, int S, int H, int Hkv, int d,
                               int bs, int max_ctx, int maxb, int num_blocks, float scale,
                               void* stream) {
  PagedArgs a{q, kc, vc, out, bt, lens, S, H, Hkv, d, bs, max_ctx, maxb, num_blocks, scale};
  return paged_v1_entry<__nv_bfloat16>(a, as_stream(stream));
}

int fe_paged_attention_v2_bf16(const void* q, const void* kc, const void* vc, void* out,
                               const int* bt, const int* lens, int S, int H, int Hkv, int d,
                               int bs, int max_ctx, int maxb, int num_blocks, float scale,
                               float* workspace, size_t workspace_floats, void* stream) {
  PagedArgs a{q, kc, vc, out, bt, lens, S, H, Hkv, d, bs, max_ctx, maxb, num_blocks, scale};
  return paged_v2_tc<__nv_bfloat16>(a, workspace, workspace_floats, as_stream(stream));
}

int fe_paged_kv_append(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                       const int* bt, const int* lens, int S, int Hkv, int d, int bs, int maxb,
                       int num_blocks, int dtype, int kv_layout, const float* rope_cos,
                       const float* rope_sin, int rope_max_pos, void* stream) {
  if (S < 0 || Hkv <= 0 || d <= 0 || d % 2 != 0 || bs <= 0 || maxb < 0) return kErr;
  if (kv_layout != fe::paged::kKvFlat && kv_layout != fe::paged::kKvVllm) return kErr;
  if (kv_layout == fe::paged::kKvVllm && (dtype == 2 || d % 8 != 0)) return kErr;
  if ((rope_cos == nullptr) != (rope_sin == nullptr) || (rope_cos && rope_max_pos < 1))
    return kErr;
  if (S == 0) return 0;
  unsigned* err = fe::device_error_word();
  if (!err) return static_cast<int>(cudaErrorInitializationError);
  fe::paged::AppendParams ap{k_new, v_new, k_cache, v_cache, bt, lens, S, Hkv, d, bs, maxb,
                             num_blocks, kv_layout, rope_cos, rope_sin, rope_max_pos, err};
  cudaStream_t st = as_stream(stream);
  if (dtype == 0) return static_cast<int>(fe::paged::launch_kv_append<__nv_bfloat16>(ap, st));
  if (dtype == 1) return static_cast<int>(fe::paged::launch_kv_append<half>(ap, st));
  if (dtype == 2) return static_cast<int>(fe::paged::launch_kv_append<float>(ap, st));
  return kErr;
}

size_t fe_paged_attention_v2_workspace_floats(int H, int Hkv, int d, int bs) {
  const long long n = workspace_floats_for(H, Hkv, d, bs);
  return n > 0 ? static_cast<size_t>(n) : 0;
}

// ---- no-alloc split-KV decode ------------------------------------------------
// Scratch for callers that cannot allocate: one array per device that loads the
// library, shared by every call (see flash_engine_c.h for the contract). It holds the
// largest split-KV workspace any device can ask for (grids are capped at kCounterSlots
// CTAs, at most 16 query heads a CTA, head_dim <= 128), so its size does not depend on
// the GPU.
static __device__ __align__(256) float g_noalloc_scratch[FE_NOALLOC_SCRATCH_FLOATS];
static_assert(fe::paged::kStreamSlots == FE_STREAM_SCRATCH_SLOTS,
              "the header states the library's scratch slot count");
static_assert(FE_NOALLOC_SCRATCH_FLOATS >=
                  fe::paged::kCounterSlots + 1LL * fe::paged::kCounterSlots * 2 * 16 * (128 + 2),
              "the no-alloc scratch must hold the workspace of the largest decode grid");

// Device address of g_noalloc_scratch on the current device, looked up once per
// device. In host code the array's name only stands in for the symbol, so it is
// never passed to a kernel directly.
static int noalloc_scratch_ptr(float** out) {
  static std::mutex mu;
  static float* ptrs[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return static_cast<int>(e);
  if (dev < 0 || dev >= 64) return static_cast<int>(cudaErrorInvalidDevice);
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    // The array is zero when the module loads, so the split-KV arrival counters at
    // its start begin at zero; every call leaves them so.
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return static_cast<int>(e);
    ptrs[dev] = static_cast<float*>(p);
  }
  *out = ptrs[dev];
  return 0;
}

int fe_paged_attention_v2_bf16_noalloc(const void* q, const void* kc, const void* vc, void* out,
                                       const int* bt, const int* lens, int S, int H, int Hkv,
                                       int d, int bs, int max_ctx, int maxb, int num_blocks,
                                       float scale, void* stream) {
  if (S < 0 || H <= 0 || Hkv <= 0 || d <= 0) return kErr;
  const long long need = workspace_floats_dtype(fe::paged::kBf16, H, Hkv, d, bs);
  if (need <= 0 || need > FE_NOALLOC_SCRATCH_FLOATS) return kErr;
  PagedArgs a{q, kc, vc, out, bt, lens, S, H, Hkv, d, bs, max_ctx, maxb, num_blocks, scale};
  const int rc = paged_check<__nv_bfloat16>(a);
  if (rc) return rc;
  if (S == 0) return 0;
  float* base = nullptr;
  const int e = noalloc_scratch_ptr(&base);
  if (e) return e;
  return paged_v2_tc<__nv_bfloat16>(a, base, FE_NOALLOC_SCRATCH_FLOATS, as_stream(stream));
}

int fe_flash_decoding_forward_fp32(const float* q, const float* k, const float* v, float* out,
                                   float* sout, float* sstats, int B, int H, int M, int d,
                                   int splits, float scale, void* stream) {
  if (B < 0 || H < 0 || M < 1 || d < 1 || d > 256 || d % 4 != 0 || splits < 1) return kErr;
  if (B * H == 0) return 0;
  cudaStream_t st = as_stream(stream);
  cudaError_t e = fe::simt::launch_decode_split_fp32(q, k, v, sout, sstats, B * H, M, d, splits,
                                                     resolve_scale(scale, d), st);
  if (e != cudaSuccess) return static_cast<int>(e);
  fe::paged::MergeParams mp{};
  mp.part_out = sout;
  mp.part_stats = sstats;
  mp.rows = B * H;
  mp.ranks = 1;
  mp.parts_per_rank = splits;
  mp.out = out;
  mp.out_dtype = 0;
  return static_cast<int>(fe::paged::launch_merge(mp, d, st));
}

int fe_paged_decode_partials_bf16(const void* q, const void* kc, const void* vc, const int* bt,
                                  const int* lens, int S, int H, int Hkv, int d, int bs, int maxb,
                                  int num_blocks, float scale, int tb, int te, float* workspace,
                                  size_t workspace_floats, float* mout, float* mstats,
                                  void* stream) {
  PagedArgs a{q, kc, vc, nullptr, bt, lens, S, H, Hkv, d, bs, 0, maxb, num_blocks, scale};
  int rc = paged_check<__nv_bfloat16>(a);
  if (rc) return rc;
  const bool lib = !workspace && workspace_floats == FE_WORKSPACE_LIBRARY;
  const long long need = workspace_floats_for(H, Hkv, d, bs);
  if (need <= 0 || (!lib && (!workspace || static_cast<long long>(workspace_floats) < need)))
    return kErr;
  if (tb < 0 || te < tb || !mout || !mstats || tb % bs != 0) return kErr;
  if (S == 0) return 0;
  cudaStream_t st = as_stream(stream);
  DecodePlan pl;
  pl.tok_begin = tb;
  pl.tok_end = te;
  pl.flat = true;
  pl.direct_final = false;
  pl.merged_out = mout;
  pl.merged_stats = mstats;
  if (lib) {  // the stream's slot of the library scratch, else one segment per row
    pl.ws_slot = stream_slot(st);
    pl.flat = pl.ws_slot >= 0;
  }
  return paged_tc_run<__nv_bfloat16>(a, pl, workspace, st);
}

int fe_paged_decode_kv_exchange_bf16(const void* q, const void* kc, const void* vc,
                                     const int* bt, const int* lens, int S, int H, int Hkv, int d,
                                     int bs, int maxb, int num_blocks, float scale, int tb, int te,
                                     float* workspace, size_t workspace_floats,
                                     void* const* xbufs, int world, int rank, int max_rows,
                                     void* out, int phases, void* stream) {
  PagedArgs a{q, kc, vc, nullptr, bt, lens, S, H, Hkv, d, bs, 0, maxb, num_blocks, scale};
  int rc = paged_check<__nv_bfloat16>(a);
  if (rc) return rc;
  if (world < 1 || world > fe::paged::kMaxRanks || rank < 0 || rank >= world || !xbufs)
    return kErr;
  if (phases < 1 || phases > 3 || S > kMaxSeqsPerLaunch) return kErr;
  if (static_cast<long long>(S) * H > max_rows || tb < 0 || te < tb || tb % bs != 0) return kErr;
  for (int r = 0; r < world; ++r)
    if (!xbufs[r] || !aligned(xbufs[r], 256)) return kErr;
  if (S == 0) return 0;
  cudaStream_t st = as_stream(stream);
  if (phases & 1) {
    const bool lib = !workspace && workspace_floats == FE_WORKSPACE_LIBRARY;
    const long long need = workspace_floats_for(H, Hkv, d, bs);
    if (need <= 0 || (!lib && (!workspace || static_cast<long long>(workspace_floats) < need)))
      return kErr;
    DecodePlan pl;
    pl.tok_begin = tb;
    pl.tok_end = te;
    pl.flat = true;
    pl.direct_final = false;
    if (lib) {  // the stream's slot of the library scratch, else one segment per row
      pl.ws_slot = stream_slot(st);
      pl.flat = pl.ws_slot >= 0;
    }
    for (int r = 0; r < world; ++r) pl.xbuf[r] = static_cast<char*>(xbufs[r]);
    pl.xworld = world;
    pl.xrank = rank;
    pl.xmax_rows = max_rows;
    rc = paged_tc_run<__nv_bfloat16>(a, pl, workspace, st);
    if (rc) return rc;
  }
  if (phases & 2) {
    if (!out || !aligned(out, 2)) return kErr;
    unsigned* err = fe::device_error_word();
    if (!err) return static_cast<int>(cudaErrorInitializationError);
    fe::paged::XMergeParams xp{};
    xp.xbuf = static_cast<char*>(xbufs[rank]);
    xp.world = world;
    xp.max_rows = max_rows;
    xp.rows = S * H;
    xp.head_dim = d;
    xp.out = out;
    xp.out_dtype = 1;
    xp.err = err;
    return static_cast<int>(fe::paged::launch_xmerge(xp, st));
  }
  return 0;
}

size_t fe_kv_exchange_bytes(int world, int max_rows, int head_dim) {
  if (world < 1 || world > fe::paged::kMaxRanks || max_rows < 1 || head_dim < 1) return 0;
  return static_cast<size_t>(fe::paged::x_buffer_bytes(world, max_rows, head_dim));
}

int fe_kv_exchange_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes < sizeof(fe::paged::XHeader)) return kErr;
  *ptr = nullptr;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return static_cast<int>(e);
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    cudaFree(p);
    return static_cast<int>(e);
  }
  *ptr = p;
  return 0;
}

int fe_kv_exchange_free(void* ptr) { return static_cast<int>(cudaFree(ptr)); }

int fe_kv_exchange_ipc_handle(void* ptr, void* handle_out) {
  if (!ptr || !handle_out) return kErr;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return static_cast<int>(e);
  memcpy(handle_out, &h, sizeof(h));
  return 0;
}

int fe_kv_exchange_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return kErr;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return static_cast<int>(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int fe_kv_exchange_ipc_close(void* ptr) { return static_cast<int>(cudaIpcCloseMemHandle(ptr)); }

int fe_nccl_unique_id(void* id_out) {
  const NcclApi& n = nccl_api();
  if (!n.ok) return static_cast<int>(cudaErrorNotSupported);
  if (!id_out) return kErr;
  ncclUniqueId id;
  const int rc = nccl_status(n.get_unique_id(&id));
  if (rc == 0) memcpy(id_out, &id, sizeof(id));
  return rc;
}

int fe_nccl_comm_init(void** comm_out, int world, const void* id, int rank) {
  const NcclApi& n = nccl_api();
  if (!n.ok) return static_cast<int>(cudaErrorNotSupported);
  if (!comm_out || !id || world < 1 || rank < 0 || rank >= world) return kErr;
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof(uid));
  ncclComm_t c = nullptr;
  const int rc = nccl_status(n.comm_init_rank(&c, world, uid, rank));
  *comm_out = rc == 0 ? c : nullptr;
  return rc;
}

int fe_nccl_comm_destroy(void* comm) {
  const NcclApi& n = nccl_api();
  if (!n.ok) return static_cast<int>(cudaErrorNotSupported);
  return comm ? nccl_status(n.comm_destroy(static_cast<ncclComm_t>(comm))) : 0;
}

size_t fe_kv_range_nccl_scratch_floats(int world, int num_seqs, int num_heads, int head_dim) {
  if (world < 1 || num_seqs < 0 || num_heads < 1 || head_dim < 1) return 0;
  return static_cast<size_t>(world + 1) * num_seqs * num_heads * (head_dim + 2);
}

int fe_paged_decode_kv_range_nccl_bf16(const void* q, const void* kc, const void* vc,
                                       const int* bt, const int* lens, int S, int H, int Hkv,
                                       int d, int bs, int maxb, int num_blocks, float scale,
                                       int max_context_len, float* workspace,
                                       size_t workspace_floats, void* comm, int rank, int world,
                                       float* scratch, size_t scratch_floats, void* out,
                                       void* stream) {
  PagedArgs a{q, kc, vc, nullptr, bt, lens, S, H, Hkv, d, bs, 0, maxb, num_blocks, scale};
  int rc = paged_check<__nv_bfloat16>(a);
  if (rc) return rc;
  if (!comm || world < 1 || rank < 0 || rank >= world || max_context_len < 0 || !out ||
      !aligned(out, 2))
    return kErr;
  const long long need = workspace_floats_for(H, Hkv, d, bs);
  if (need <= 0 || !workspace || static_cast<long long>(workspace_floats) < need) return kErr;
  const size_t sneed = fe_kv_range_nccl_scratch_floats(world, S, H, d);
  if (!scratch || scratch_floats < sneed || S > kMaxSeqsPerLaunch) return kErr;
  const NcclApi& n = nccl_api();
  if (!n.ok) return static_cast<int>(cudaErrorNotSupported);
  if (S == 0) return 0;
  cudaStream_t st = as_stream(stream);
  const long long rows = static_cast<long long>(S) * H;
  const long long blk = rows * (d + 2);  // one rank's partials: O rows, then (m, l) pairs
  float* send = scratch;
  float* recv = scratch + blk;
  // 1. this rank's window: one merged (O, m, l) partial per (sequence, query head)
  DecodePlan pl;
  kv_range_window(max_context_len, world, rank, bs, &pl.tok_begin, &pl.tok_end);
  pl.flat = true;
  pl.direct_final = false;
  pl.merged_out = send;
  pl.merged_stats = send + rows * d;
  rc = paged_tc_run<__nv_bfloat16>(a, pl, workspace, st);
  if (rc) return rc;
  // 2. all-gather the partials of every rank
  rc = nccl_status(n.all_gather(send, recv, static_cast<size_t>(blk), ncclFloat,
                                static_cast<ncclComm_t>(comm), st));
  if (rc) return rc;
  // 3. log-sum-exp merge of the world partials of each row
  fe::paged::MergeParams mp{};
  mp.part_out = recv;
  mp.part_stats = recv + rows * d;
  mp.rows = static_cast<int>(rows);
  mp.ranks = world;
  mp.parts_per_rank = 1;
  mp.rank_stride_out = blk;
  mp.rank_stride_stats = blk;
  mp.out = out;
  mp.out_dtype = 1;
  return static_cast<int>(fe::paged::launch_merge(mp, d, st));
}

int fe_merge_partials(const float* part_out, const float* part_stats, int rows, int ranks,
                      int parts_per_rank, int d, void* out, float* out_stats, int out_dtype,
                      void* stream) {
  if (rows < 0 || ranks < 1 || parts_per_rank < 1 || d < 1 || d > 256 || out_dtype < 0 ||
      out_dtype > 3 || (out_dtype == 2 && !out_stats))
    return kErr;
  fe::paged::MergeParams mp{};
  mp.part_out = part_out;
  mp.part_stats = part_stats;
  mp.rows = rows;
  mp.ranks = ranks;
  mp.parts_per_rank = parts_per_rank;
  mp.out = out;
  mp.out_stats = out_stats;
  mp.out_dtype = out_dtype;
  return static_cast<int>(fe::paged::launch_merge(mp, d, as_stream(stream)));
}

}  // extern "C"

// =========================================================================
// C++ API with the reference's namespaces and signatures.
namespace flash_engine {

void print_device_info(int device_id) { fe_print_device_info(device_id); }

namespace attention {

cudaError_t launch_flash_attention_forward_fp32(const float* q, const float* k, const float* v,
                                                float* o, const AttentionConfig& c,
                                                cudaStream_t s) {
  return static_cast<cudaError_t>(fe_flash_attention_forward_fp32(
      q, k, v, o, c.batch_size, c.num_heads, c.seq_len_q, c.seq_len_kv, c.head_dim, c.is_causal,
      c.softmax_scale, s));
}
cudaError_t launch_flash_attention_forward_fp16(const half* q, const half* k, const half* v,
                                                half* o, const AttentionConfig& c,
                                                cudaStream_t s) {
  return static_cast<cudaError_t>(fe_flash_attention_forward_fp16(
      q, k, v, o, c.batch_size, c.num_heads, c.seq_len_q, c.seq_len_kv, c.head_dim, c.is_causal,
      c.softmax_scale, s));
}
cudaError_t launch_flash_attention_forward_bf16(const __nv_bfloat16* q, const __nv_bfloat16* k,
                                                const __nv_bfloat16* v, __nv_bfloat16* o,
                                                const AttentionConfig& c, cudaStream_t s) {
  return static_cast<cudaError_t>(fe_flash_attention_forward_bf16(
      q, k, v, o, c.batch_size, c.num_heads, c.seq_len_q, c.seq_len_kv, c.head_dim, c.is_causal,
      c.softmax_scale, s));
}
cudaError_t launch_naive_attention_forward_fp32(const float* q, const float* k, const float* v,
                                                float* o, const AttentionConfig& c,
                                                cudaStream_t s) {
  return static_cast<cudaError_t>(fe_naive_attention_forward_fp32(
      q, k, v, o, c.batch_size, c.num_heads, c.seq_len_q, c.seq_len_kv, c.head_dim, c.is_causal,
      c.softmax_scale, s));
}

}  // namespace attention

namespace paged_attention {

cudaError_t launch_paged_attention_v1_fp16(const half* q, const half* kc, const half* vc,
                                           half* out, const int* bt, const int* lens,
                                           const PagedAttentionConfig& c, cudaStream_t s) {
  return static_cast<cudaError_t>(fe_paged_attention_v1_fp16(
      q, kc, vc, out, bt, lens, c.num_seqs, c.num_heads, c.num_kv_heads, c.head_dim, c.block_size,
      c.max_context_len, c.max_num_blocks_per_seq, 0, c.scale, s));
}
cudaError_t launch_paged_attention_v1_fp32(const float* q, const float* kc, const float* vc,
                                           float* out, const int* bt, const int* lens,
                                           const PagedAttentionConfig& c, cudaStream_t s) {
  return static_cast<cudaError_t>(fe_paged_attention_v1_fp32(
      q, kc, vc, out, bt, lens, c.num_seqs, c.num_heads, c.num_kv_heads, c.head_dim, c.block_size,
      c.max_context_len, c.max_num_blocks_per_seq, 0, c.scale, s));
}
cudaError_t launch_paged_attention_v1_bf16(const __nv_bfloat16* q, const __nv_bfloat16* kc,
                                           const __nv_bfloat16* vc, __nv_bfloat16* out,
                                           const int* bt, const int* lens,
                                           const PagedAttentionConfig& c, cudaStream_t s) {
  return static_cast<cudaError_t>(fe_paged_attention_v1_bf16(
      q, kc, vc, out, bt, lens, c.num_seqs, c.num_heads, c.num_kv_heads, c.head_dim, c.block_size,
      c.max_context_len, c.max_num_blocks_per_seq, 0, c.scale, s));
}
cudaError_t launch_paged_attention_v2_bf16(const __nv_bfloat16* q, const __nv_bfloat16* kc,
                                           const __nv_bfloat16* vc, __nv_bfloat16* out,
                                           const int* bt, const int* lens,
                                           const PagedAttentionConfig& c, float* workspace,
                                           size_t workspace_floats, cudaStream_t s) {
  return static_cast<cudaError_t>(fe_paged_attention_v2_bf16(
      q, kc, vc, out, bt, lens, c.num_seqs, c.num_heads, c.num_kv_heads, c.head_dim, c.block_size,
      c.max_context_len, c.max_num_blocks_per_seq, 0, c.scale, workspace, workspace_floats, s));
}

cudaError_t launch_paged_decode_kv_range_bf16(
    const __nv_bfloat16* q, const __nv_bfloat16* kc, const __nv_bfloat16* vc,
    __nv_bfloat16* out, const int* bt, const int* lens, const PagedAttentionConfig& c,
    ncclComm_t comm, int rank, int world, float* workspace, size_t workspace_floats,
    float* scratch, size_t scratch_floats, cudaStream_t s) {
  return static_cast<cudaError_t>(fe_paged_decode_kv_range_nccl_bf16(
      q, kc, vc, bt, lens, c.num_seqs, c.num_heads, c.num_kv_heads, c.head_dim, c.block_size,
      c.max_num_blocks_per_seq, 0, c.scale, c.max_context_len, workspace, workspace_floats, comm,
      rank, world, scratch, scratch_floats, out, s));
}

}  // namespace paged_attention

namespace rope {

cudaError_t launch_fused_rope_fp32(const float* d_in, const float* d_cos, const float* d_sin,
                                   float* d_out, const RoPEConfig& c, cudaStream_t s) {
  return static_cast<cudaError_t>(fe_rope_forward(d_in, d_cos, d_sin, d_out, c.batch_size,
                                                  c.num_heads, c.seq_len, c.head_dim, 2, s));
}
cudaError_t launch_fused_rope_bf16(const __nv_bfloat16* d_in, const float* d_cos,
                                   const float* d_sin, __nv_bfloat16* d_out, const RoPEConfig& c,
                                   cudaStream_t s) {
  return static_cast<cudaError_t>(fe_rope_forward(d_in, d_cos, d_sin, d_out, c.batch_size,
                                                  c.num_heads, c.seq_len, c.head_dim, 0, s));
}
cudaError_t launch_fused_rope_fp16(const half* d_in, const float* d_cos, const float* d_sin,
                                   half* d_out, const RoPEConfig& c, cudaStream_t s) {
  return static_cast<cudaError_t>(fe_rope_forward(d_in, d_cos, d_sin, d_out, c.batch_size,
                                                  c.num_heads, c.seq_len, c.head_dim, 1, s));
}

}  // namespace rope

namespace decoding {

cudaError_t launch_flash_decoding_forward_fp32(const float* q, const float* k, const float* v,
                                               float* out, float* sout, float* sstats,
                                               const FlashDecodingConfig& c, cudaStream_t s) {
  return static_cast<cudaError_t>(fe_flash_decoding_forward_fp32(
      q, k, v, out, sout, sstats, c.batch_size, c.num_heads, c.seq_len_kv, c.head_dim,
      c.num_splits, c.scale, s));
}

}  // namespace decoding
}  // namespace flash_engine
