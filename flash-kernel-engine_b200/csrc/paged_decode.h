// Internal interface of the tensor-core paged decode kernels (paged_decode.cu).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace fe {
namespace paged {

// KV-cache layouts of the tensor-core decode.
enum KvLayout : int {
  kKvFlat = 0,  // K and V [num_blocks, Hkv, BS, D] (the reference's fp32 layout)
  kKvVllm = 1,  // vLLM: K [num_blocks, Hkv, D/8, BS, 8], V [num_blocks, Hkv, D, BS]
};

// KV-range exchange buffer (one per rank, the same layout on every rank; the peers'
// copies are mapped into this process). Header, then two generations (step parity)
// of partial rows in 8-byte words (value bits | step << 32): a reader knows a word is
// from the step it wants by its upper half, so no fence or flag is needed between the
// peer stores and the reads. O [2][world][max_rows][D], (m log2, l) [2][world][max_rows][2].
constexpr int kMaxRanks = 8;
struct XHeader {
  unsigned step;              // steps this rank has merged (its merge kernels)
  unsigned merge_ctas;        // merge CTAs of the running step that have finished
  unsigned pad[62];           // 256 bytes in all
};
static_assert(sizeof(XHeader) == 256, "exchange header is 256 bytes");
inline __host__ __device__ long long x_o_word(int parity, int world, int rank, int max_rows,
                                               long long row, int d) {
  return ((static_cast<long long>(parity) * world + rank) * max_rows + row) * d;
}
inline __host__ __device__ long long x_ml_word(int parity, int world, int rank, int max_rows,
                                                long long row, int d) {
  return 2LL * world * max_rows * d +
         ((static_cast<long long>(parity) * world + rank) * max_rows + row) * 2;
}
// Bytes of one exchange buffer.
inline long long x_buffer_bytes(int world, int max_rows, int d) {
  return static_cast<long long>(sizeof(XHeader)) + 8LL * 2 * world * max_rows * (d + 2);
}

struct Params {
  const void* q;           // [S, H, D] (T; float for the fp32 decode)
  const void* k_cache;     // used by the bulk-copy (vLLM layout) path
  const void* v_cache;
  void* out;               // [S, H, D] (T), written for single-split sequences
  const int* block_tables; // [S, max_blocks_per_seq]
  const int* context_lens; // [S]
  float* part_o;           // fixup slots [grid][2][HPC][D] fp32 partial O (unnormalised)
  float* part_ml;          // fixup slots [grid][2][HPC][2] (m in log2 units, l)
  int* counters;           // flat mode: [grid] piece-arrival counters; zero before the
                           // launch, and left zero by it
  int ws_slot;             // >= 0: counters and fixup slots live in slot ws_slot of the
                           // library's static stream scratch (part_o etc. unused)
  int max_grid;            // > 0: at most this many CTAs (the fixup slots must fit)
  float* merged_o;         // partials mode: [S, H, D] merged partial of whole rows
  float* merged_ml;        // partials mode: [S, H, 2]
  int num_seqs, num_heads, num_kv_heads, max_blocks_per_seq;
  int num_phys_blocks;     // 0 = unknown (no range check)
  int head_chunks;         // ceil(G / (8 * NT))
  int tok_begin, tok_end;  // token window [tok_begin, tok_end) of every sequence
  int pages_per_split;     // unit mode: pages per segment
  int seg_cost_pages;      // flat mode: pages a CTA's share shrinks by for each sequence
                           // that starts in its chunk (see FlatPartition)
  int flat;                // 1: flat (stream-K) chunking, 0: unit mode
  int direct_final;        // 1: whole rows are written normalised to `out`;
                           // 0: as merged partials to merged_o / merged_ml
  float scale_log2;        // softmax scale * log2(e)
  // Optional rotary embedding of the query token (position context_len - 1): pair
  // (2i, 2i+1) is rotated by cos/sin[pos][i] of [rope_max_pos, D/2] fp32 tables.
  const float* rope_cos;
  const float* rope_sin;
  int rope_max_pos;
  unsigned* err;           // device error word
  long long dbg_kv_rows;   // rows of the K/V tensor maps (bounds checks in debug builds)
  // KV-range exchange (partials mode with xworld > 0): every finished partial row is
  // stored, tagged with the step, into all xworld ranks' exchange buffers (peer stores
  // over NVLink) at this rank's slot instead of merged_o / merged_ml. xbuf[xrank] is
  // this rank's own buffer.
  char* xbuf[kMaxRanks];
  int xworld, xrank, xmax_rows;
};

// Merge of one KV-range exchange step on this rank: reads every rank's partials of
// each row, re-reading (bounded) each word until it carries this step, combines them
// and writes the output row; the last merge CTA advances the step count.
struct XMergeParams {
  char* xbuf;              // this rank's exchange buffer
  int world, max_rows, rows, head_dim;
  void* out;               // [rows, D] final output
  int out_dtype;           // 0 f32, 1 bf16, 3 fp16
  unsigned* err;
};
cudaError_t launch_xmerge(const XMergeParams& xp, cudaStream_t stream);

struct MergeParams {
  const float* part_out;   // [ranks, rows, parts_per_rank, D]
  const float* part_stats; // [ranks, rows, parts_per_rank, 2] (m in log2 units, l)
  int rows;
  int ranks;
  int parts_per_rank;
  void* out;
  float* out_stats;
  int out_dtype;           // 0 f32 final, 1 bf16 final, 2 merged partial, 3 fp16 final
  int head_dim;            // set by launch_merge
  // floats between consecutive ranks' blocks of part_out / part_stats; 0 = packed
  // ([ranks, rows, parts_per_rank, ...] contiguous)
  long long rank_stride_out, rank_stride_stats;
};

// Splits of the page range [0, pages) into `splits` pieces of pages_per_split.
inline int pages_per_split_for(int max_pages, int splits) {
  if (splits < 1) splits = 1;
  return (max_pages + splits - 1) / splits;
}

// Launches the decode kernel; *grid_out receives its CTA count. T is __nv_bfloat16,
// half or float (fp32 cache: flat layout only).
template <typename T>
cudaError_t launch_decode(const Params& p, int head_dim, int block_size, const void* k_cache,
                          const void* v_cache, long long kv_rows, int nt, int kv_layout,
                          int* grid_out, cudaStream_t stream);

cudaError_t launch_merge(const MergeParams& mp, int head_dim, cudaStream_t stream);

// Cache append of the new token of every sequence (kv_append_kernel).
struct AppendParams {
  const void* k_new;        // [S, Hkv, D] (T)
  const void* v_new;        // [S, Hkv, D]
  void* k_cache;            // flat [blocks, Hkv, BS, D] or vLLM K [blocks, Hkv, D/8, BS, 8]
  void* v_cache;            // flat, or vLLM V [blocks, Hkv, D, BS]
  const int* block_tables;  // [S, max_blocks_per_seq]
  const int* context_lens;  // [S]; the new token sits at position context_lens[s] - 1
  int num_seqs, num_kv_heads, head_dim, block_size, max_blocks_per_seq, num_blocks;
  int kv_layout;
  const float* rope_cos;    // optional [rope_max_pos, D/2]: K rotated at its position
  const float* rope_sin;
  int rope_max_pos;
  unsigned* err;
};
template <typename T>
cudaError_t launch_kv_append(const AppendParams& ap, cudaStream_t stream);

// Flat-mode scratch: kCounterSlots int arrival counters at the start (the same
// place for every shape, so a workspace shared by several shapes keeps them at
// zero), then `slot_rows` fixup rows of O (D floats each) and of stats (2 each).
constexpr int kCounterSlots = 1024;  // also the largest flat-mode grid
struct FixupLayout {
  long long grid_max;   // largest CTA count of the decode grid on this device
  long long slot_rows;  // grid_max * 2 * HPC
  long long floats;     // kCounterSlots + slot_rows * (D + 2)
};
// Element type of the decode (q, cache and output).
enum DecodeType : int { kBf16 = 0, kF16 = 1, kF32 = 2 };
// Query heads one CTA segment covers: 8 * nt for the tensor-core (bf16/fp16) decode,
// 4 * nt for the fp32 decode.
inline int heads_per_cta(int dtype, int nt) { return dtype == kF32 ? 4 * nt : 8 * nt; }
// nt of a head group of G query heads.
inline int decode_nt(int dtype, int G) { return G <= heads_per_cta(dtype, 1) ? 1 : 2; }
// Layout for this shape, or floats = -1 if the shape is unsupported.
FixupLayout fixup_layout(int dtype, int head_dim, int block_size, int nt);

// Split-KV scratch owned by the library for the entry points whose reference
// signature passes none (the v1 paged launchers): kStreamSlots slots of
// kStreamSlotFloats floats in a static __device__ array of paged_decode.cu (zero
// when the module loads; the kernel names it directly, so no host-side address is
// needed). A launch with Params::ws_slot = k keeps its counters at the start of slot
// k and its fixup slots after them, and must be capped (Params::max_grid) so that
// kCounterSlots + grid * 2 * HPC * (D + 2) <= kStreamSlotFloats.
constexpr int kStreamSlots = 4;
constexpr long long kStreamSlotFloats = 1LL << 20;
inline int slot_grid_cap(int dtype, int head_dim, int nt) {
  const long long per_cta = 2LL * heads_per_cta(dtype, nt) * (head_dim + 2);
  return static_cast<int>((kStreamSlotFloats - kCounterSlots) / per_cta);
}

}  // namespace paged
}  // namespace fe
