/*
 * flash_engine_c.h -- C ABI of the B200 (sm_100a) inference-attention library
 * (libflash_engine_b200.so).
 *
 * Plain pointers, ints and floats only; no C++ or torch types. Every entry point
 * is stream-ordered on `stream` (a cudaStream_t passed as void*, NULL = legacy
 * default stream), never allocates, never frees and never synchronises. The
 * caller owns every device buffer, exactly as with the reference's launchers.
 *
 * Return value: a cudaError_t as int. 0 = cudaSuccess; 1 = cudaErrorInvalidValue
 * for arguments the kernels do not support (the reference silently mis-dispatches
 * those: src/flash_attention.cu:339-342, src/flash_decoding.cu:244-262); any other
 * value is the launch status from cudaGetLastError(), as the reference returns
 * (src/flash_attention.cu:344).
 *
 * Layouts (row-major, contiguous):
 *   dense attention  Q,O [B, H, N, d]; K,V [B, H, M, d]
 *   paged decode     q,out [S, H, d]; k_cache,v_cache [num_blocks, Hkv, block_size, d];
 *                    block_tables [S, max_blocks_per_seq] int32; context_lens [S] int32
 *   dense split-KV   scratch_out [B, H, num_splits, d] f32; scratch_stats
 *   scratch          [B, H, num_splits, 2] f32 = (m, l), m in log2 units of the
 *                    scaled score, l = sum 2^(s*scale*log2e - m)
 *
 * bf16 / fp16 buffers are passed as `const void*` (__nv_bfloat16 / half in C++).
 */
#ifndef FLASH_ENGINE_C_H_
#define FLASH_ENGINE_C_H_

#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Version string, "1.2.0-b200". Replaces flash_engine::get_version()
 * (include/flash_engine.h:24-26). */
const char* fe_get_version(void);

/* Prints device properties. Replaces flash_engine::print_device_info
 * (include/flash_engine.h:29, src/flash_engine_api.cu:7-27). */
int fe_print_device_info(int device_id);

/* Reads and clears the library's device error word on the current device
 * (bit 0: a bounded wait timed out; bit 1: a block-table entry was out of range;
 * bit 2: tensor-memory allocation failed; bit 3: a split-KV workspace's arrival
 * counters were not zero when a call started). Synchronises the device. The reference
 * has no device-side checking; this is new. */
int fe_get_device_errors(unsigned int* errors_out);

/* ---------------------------------------------------------------- prefill
 * FA2 online-softmax forward O = softmax(Q K^T * scale [+ causal mask]) V.
 * Causal masking is top-left aligned (query row i sees keys j <= i), as
 * src/flash_attention.cu:224 and python/flash_engine/ops.py:43-45.
 * softmax_scale <= 0 selects 1/sqrt(d) (AttentionConfig, include/flash_attention.cuh:19-21).
 */

/* fp32. Replaces launch_flash_attention_forward_fp32 (include/flash_attention.cuh:60-67,
 * src/flash_attention.cu:304-345). Any head_dim in 1..128 (the reference dispatches 32,
 * 64 and 128 and sends others to its naive kernel, which also stops at 128). head_dim
 * 32, 64 and 128 with 16-byte aligned tensors run a 3xTF32 tcgen05 tensor-core kernel;
 * other shapes a CUDA-core kernel. Both hold the 1e-3 relative fp32 tolerance. */
int fe_flash_attention_forward_fp32(const float* q, const float* k, const float* v, float* o,
                                    int batch, int heads, int seq_q, int seq_kv, int head_dim,
                                    int is_causal, float softmax_scale, void* stream);

/* fp16 in/out, fp32 accumulate. Replaces launch_flash_attention_forward_fp16
 * (include/flash_attention.cuh:69-76, src/flash_attention.cu:486-524). head_dim 32, 64
 * or 128 (32 runs the 64 kernel with zero-filled columns), as the reference dispatches
 * (src/flash_attention.cu:514-521). */
int fe_flash_attention_forward_fp16(const void* q, const void* k, const void* v, void* o,
                                    int batch, int heads, int seq_q, int seq_kv, int head_dim,
                                    int is_causal, float softmax_scale, void* stream);

/* bf16 in/out, fp32 accumulate (tcgen05 / TMEM / TMA kernel). New sibling of the fp16
 * entry with identical parameters. head_dim 32, 64 or 128. */
int fe_flash_attention_forward_bf16(const void* q, const void* k, const void* v, void* o,
                                    int batch, int heads, int seq_q, int seq_kv, int head_dim,
                                    int is_causal, float softmax_scale, void* stream);

/* Rotary position embedding of a dense [batch, heads, seq_len, head_dim] tensor (dtype
 * 0 bf16, 1 fp16, 2 fp32): row r of batch*heads*seq_len is rotated at position
 * r % seq_len with fp32 tables [>= seq_len, head_dim/2]; out may be in. Replaces
 * launch_fused_rope_fp32 (include/fused_rope.cuh:21-28, src/fused_rope.cu:13-69); the
 * bf16 / fp16 types are new. */
int fe_rope_forward(const void* in, const float* cos_table, const float* sin_table, void* out,
                    int batch, int heads, int seq_len, int head_dim, int dtype, void* stream);

/* bf16 (dtype 0) or fp16 (dtype 1) FA2 forward of fe_flash_attention_forward_bf16 /
 * _fp16 with an optional rotary embedding of Q and K: rope_cos / rope_sin (NULL = off)
 * are fp32 tables [rope_max_pos, head_dim/2] (16-byte aligned, rope_max_pos >= seq_q and
 * >= seq_kv); query row i and key row j of every (batch, head) are rotated at positions
 * i and j (pairs (2i, 2i+1), src/fused_rope.cu:33-43) by the streaming RoPE pass
 * (fe_rope_forward) into the caller's q_rotated / k_rotated buffers (like q / k; they may
 * be q / k themselves), which the attention kernel then reads; k_rotated keeps the
 * rotated keys a KV cache stores. New: the reference runs its RoPE and attention
 * kernels as separate calls. */
int fe_flash_attention_forward_ex(const void* q, const void* k, const void* v, void* o,
                                  int batch, int heads, int seq_q, int seq_kv, int head_dim,
                                  int is_causal, float softmax_scale, int dtype,
                                  const float* rope_cos, const float* rope_sin, int rope_max_pos,
                                  void* q_rotated, void* k_rotated, void* stream);

/* Row-per-thread fp32 attention. Replaces launch_naive_attention_forward_fp32
 * (include/flash_attention.cuh:79-86, src/flash_attention.cu:86-104). */
int fe_naive_attention_forward_fp32(const float* q, const float* k, const float* v, float* o,
                                    int batch, int heads, int seq_q, int seq_kv, int head_dim,
                                    int is_causal, float softmax_scale, void* stream);

/* ---------------------------------------------------------------- paged decode
 * out[s, h] = softmax(q[s, h] . K[s, h/(H/Hkv)]^T * scale) V[...] over context_lens[s]
 * tokens; token t of sequence s is row t % block_size of physical block
 * block_tables[s, t / block_size] (src/paged_attention.cu:54-84). A sequence
 * with context_len <= 0 gets a zero output row (python/flash_engine/ops.py:74-78).
 * num_blocks > 0 enables a device-side range check of every block-table entry
 * (bad entries are skipped and flagged in the device error word); 0 = unknown.
 * scale <= 0 selects 1/sqrt(head_dim).
 * The bf16/fp16 decode kernels are launched with programmatic dependent launch and
 * read context_lens and the first block-table entries before they wait for the
 * previous kernel in the stream. No kernel of this library writes those two arrays,
 * and a kernel that does not trigger programmatic launch itself (or a copy) always
 * completes first. So the one case to avoid is a kernel of the caller's that writes
 * them and signals programmatic completion early, placed directly before a decode.
 */

/* fp32 cache. Replaces launch_paged_attention_v1_fp32 (include/paged_attention.cuh:39-48,
 * src/paged_attention.cu:181-215). Any block_size >= 1, head_dim % 4 == 0, <= 256.
 * head_dim 64 or 128 with block_size 16 or 32 and 16-byte aligned q / caches runs the
 * persistent split-KV decode of fe_paged_attention_v2_bf16 with fp32 arithmetic on the
 * stream's library scratch slot (see fe_paged_attention_v1_bf16); other shapes run a
 * single-pass CUDA-core kernel with one CTA per (sequence, KV head). */
int fe_paged_attention_v1_fp32(const float* q, const float* k_cache, const float* v_cache,
                               float* out, const int* block_tables, const int* context_lens,
                               int num_seqs, int num_heads, int num_kv_heads, int head_dim,
                               int block_size, int max_context_len, int max_blocks_per_seq,
                               int num_blocks, float scale, void* stream);

/* fp16 cache in the layout the reference's header declares for this entry
 * (include/paged_attention.cuh:27-36, vLLM's x-packed layout, x = 8 halves):
 * K [num_blocks, Hkv, head_dim/8, block_size, 8], V [num_blocks, Hkv, head_dim,
 * block_size]. Replaces the launch_paged_attention_v1_fp16 stub
 * (src/paged_attention.cu:218-230, which launches nothing). block_size 16,
 * head_dim 64 or 128. Runs the split-KV kernel on scratch the library owns (see
 * fe_paged_attention_v1_bf16). */
int fe_paged_attention_v1_fp16(const void* q, const void* k_cache, const void* v_cache,
                               void* out, const int* block_tables, const int* context_lens,
                               int num_seqs, int num_heads, int num_kv_heads, int head_dim,
                               int block_size, int max_context_len, int max_blocks_per_seq,
                               int num_blocks, float scale, void* stream);

/* General paged decode: dtype 0 = bf16, 1 = fp16 (tensor cores), 2 = fp32 (CUDA
 * cores; flat layout, 16-byte aligned q); kv_layout 0 = flat
 * [num_blocks, Hkv, block_size, d] (K and V), 1 = vLLM x-packed (K [num_blocks, Hkv,
 * d/8, block_size, 8], V [num_blocks, Hkv, d, block_size]; block_size 16). With a
 * workspace (fe_paged_attention_v2_workspace_floats floats) it runs the split-KV
 * path, without one (NULL) the single-pass path. workspace = NULL with
 * workspace_floats = FE_WORKSPACE_LIBRARY runs the split-KV path on the stream's slot
 * of the library's scratch, as the v1 entries do (see fe_paged_attention_v1_bf16).
 * rope_cos / rope_sin (NULL = off): fp32 tables [rope_max_pos, d/2]; the query of
 * sequence s is rotated at position context_lens[s] - 1 in the kernel prologue,
 * pairs (2i, 2i+1) as in the reference's src/fused_rope.cu:33-43 (the cached keys are
 * expected to be rotated already, as a cache-writing step stores them). New. */
int fe_paged_attention_ex(const void* q, const void* k_cache, const void* v_cache, void* out,
                          const int* block_tables, const int* context_lens, int num_seqs,
                          int num_heads, int num_kv_heads, int head_dim, int block_size,
                          int max_blocks_per_seq, int num_blocks, float scale, int dtype,
                          int kv_layout, const float* rope_cos, const float* rope_sin,
                          int rope_max_pos, float* workspace, size_t workspace_floats,
                          void* stream);

/* bf16 cache, v1 calling convention (the caller passes no scratch). New bf16 sibling
 * of launch_paged_attention_v1_fp32. block_size 16 or 32, head_dim 64 or 128.
 * Runs the split-KV kernel of fe_paged_attention_v2_bf16 on scratch the library owns
 * and never allocates: FE_STREAM_SCRATCH_SLOTS slots of a static device array (4 MiB
 * each) that every GPU loading the library holds until the process exits. The first
 * v1 call on a stream binds a free slot to that (device, stream) for the life of the
 * process (the per-thread default stream is bound per calling thread); this needs no
 * allocation and no synchronisation, so it also works while the stream is being
 * captured into a CUDA graph. Calls on one stream are ordered and share its slot;
 * a graph that captured a v1 call uses its stream's slot when replayed, so replays
 * must not overlap other work on that stream. A stream whose handle is destroyed and
 * reused by a new stream inherits the slot: destroy a stream only once its v1 work has
 * finished. When every slot is bound, other streams run the single-pass kernel (one
 * unit of work per (sequence, KV head), no scratch), which is also what
 * fe_paged_attention_ex runs without a workspace. */
int fe_paged_attention_v1_bf16(const void* q, const void* k_cache, const void* v_cache,
                               void* out, const int* block_tables, const int* context_lens,
                               int num_seqs, int num_heads, int num_kv_heads, int head_dim,
                               int block_size, int max_context_len, int max_blocks_per_seq,
                               int num_blocks, float scale, void* stream);

/* bf16 cache, split-KV with a caller-owned workspace (the v2 form of vLLM's paged
 * attention; the reference has only v1). The (KV head, sequence, page) space is cut
 * into equal chunks, one per persistent CTA, whatever the context-length mix; a
 * sequence crossing chunk boundaries leaves fp32 partials in the workspace, and the
 * CTA that finishes its last piece combines them (log-sum-exp merge) in the same
 * kernel. workspace must hold fe_paged_attention_v2_workspace_floats(num_heads,
 * num_kv_heads, head_dim, block_size) floats (about 2.5 MB at d = 128; independent of
 * the batch and of the context lengths). Its first 1024 floats (4 KiB) are arrival
 * counters: zero-fill the workspace once before its first use (cudaMemset); every
 * call leaves the counters at zero, so the workspace can be reused for any shape.
 * Calls that share a workspace must not overlap on the GPU. max_context_len is not
 * used. */
int fe_paged_attention_v2_bf16(const void* q, const void* k_cache, const void* v_cache,
                               void* out, const int* block_tables, const int* context_lens,
                               int num_seqs, int num_heads, int num_kv_heads, int head_dim,
                               int block_size, int max_context_len, int max_blocks_per_seq,
                               int num_blocks, float scale, float* workspace,
                               size_t workspace_floats, void* stream);

/* Cache append of the decode step's new token, with the rotary embedding of the key
 * fused in: for every sequence s with context_lens[s] > 0, the K row k_new[s, h] (rotated
 * at position context_lens[s] - 1 when rope_cos / rope_sin are given: fp32 tables
 * [rope_max_pos, d/2], pairs (2i, 2i+1) as src/fused_rope.cu:33-43) and the V row
 * v_new[s, h] ([S, Hkv, d] each) are written into row (ctx - 1) % block_size of physical
 * block block_tables[s, (ctx - 1) / block_size] for every KV head h. dtype 0 bf16, 1
 * fp16, 2 fp32; kv_layout 0 flat, 1 vLLM (16-bit types). Launched without programmatic
 * completion, so a decode that follows on the stream reads the appended rows; with the
 * decode's rope tables the query is rotated at the same position, so Q and K both carry
 * the embedding. Out-of-range block-table entries set bit 1 of the device error word.
 * New: the reference has no cache writer (its fused RoPE, src/fused_rope.cu:13-69,
 * rotates a dense Q or K tensor). */
int fe_paged_kv_append(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                       const int* block_tables, const int* context_lens, int num_seqs,
                       int num_kv_heads, int head_dim, int block_size, int max_blocks_per_seq,
                       int num_blocks, int dtype, int kv_layout, const float* rope_cos,
                       const float* rope_sin, int rope_max_pos, void* stream);

/* Scratch slots of the v1 entry points (see fe_paged_attention_v1_bf16). */
#define FE_STREAM_SCRATCH_SLOTS 4
/* workspace_floats value that asks fe_paged_attention_ex (with workspace = NULL) for the
 * library's per-stream scratch slot. */
#define FE_WORKSPACE_LIBRARY ((size_t)-1)

/* Workspace floats the split-KV decode (fe_paged_attention_v2_bf16,
 * fe_paged_attention_ex with any dtype, fe_paged_decode_partials_bf16) needs on the
 * current device for this head configuration; 0 if the shape is not supported. */
size_t fe_paged_attention_v2_workspace_floats(int num_heads, int num_kv_heads, int head_dim,
                                              int block_size);

/* Maximum scratch of fe_paged_attention_v2_bf16_noalloc, in floats (17 MiB): the
 * workspace of the largest decode grid any GPU can launch (1024 CTAs of 16 query
 * heads at head_dim 128), so the limit does not depend on the device. */
#define FE_NOALLOC_SCRATCH_FLOATS (4352 * 1024)

/* The split-KV bf16 decode of fe_paged_attention_v2_bf16 for callers that cannot
 * allocate device memory: plugin hosts that own every device buffer and hand a
 * library only its inputs and outputs, and serving loops that may not call
 * cudaMalloc because it synchronises the whole device. The split partials live in
 * a fixed 16 MiB array inside this library (FE_NOALLOC_SCRATCH_FLOATS), which
 * every GPU that loads the library holds until the process exits; nothing is
 * allocated or freed by this call. It has no counterpart in the reference.
 *   - Returns cudaErrorInvalidValue (1), before touching the GPU, when the
 *     configuration needs more than FE_NOALLOC_SCRATCH_FLOATS floats
 *     (fe_paged_attention_v2_workspace_floats).
 *   - The first call on a device looks up the array's device address on the
 *     current device; make that first call before any stream capture.
 *   - All calls share the one array: calls that can overlap on the GPU (other
 *     streams, other threads) race on it and must be serialised by the caller.
 *     The array is zero when the library is loaded and every call leaves its
 *     arrival counters at zero; after two calls did overlap, the counters may stay
 *     wrong for the rest of the process, and later calls can then return wrong
 *     rows (some of them flagged as bit 3 of the device error word).
 * Other arguments and limits are those of fe_paged_attention_v2_bf16. */
int fe_paged_attention_v2_bf16_noalloc(const void* q, const void* k_cache, const void* v_cache,
                                       void* out, const int* block_tables,
                                       const int* context_lens, int num_seqs, int num_heads,
                                       int num_kv_heads, int head_dim, int block_size,
                                       int max_context_len, int max_blocks_per_seq,
                                       int num_blocks, float scale, void* stream);

/* ---------------------------------------------------------------- split-KV decoding
 * Dense [B, H, M, d] fp32 flash decoding with caller-owned scratch. Replaces
 * launch_flash_decoding_forward_fp32 (include/flash_decoding.cuh:22-31,
 * src/flash_decoding.cu:225-263). Split s covers [s*ceil(M/S), min(M, (s+1)*ceil(M/S)))
 * (src/flash_decoding.cu:29-32; python/flash_engine/ops.py:112-121). Any head_dim
 * % 4 == 0 up to 256 (the reference launches nothing for d not in {64,128}). */
int fe_flash_decoding_forward_fp32(const float* q, const float* k, const float* v, float* out,
                                   float* scratch_out, float* scratch_stats, int batch, int heads,
                                   int seq_kv, int head_dim, int num_splits, float scale,
                                   void* stream);

/* Paged, GQA partial attention over the logical token window [token_begin,
 * token_end) of every sequence (clipped to its context length), bf16 cache: ONE
 * merged partial per (sequence, query head) in merged_out [S, H, d] f32
 * (unnormalised O) and merged_stats [S, H, 2] (m in log2 units of the scaled score,
 * l = sum 2^(s*scale*log2e - m)); a sequence whose window is empty gets (0, -inf, 0).
 * The work is spread like fe_paged_attention_v2_bf16 and needs the same workspace
 * (or workspace = NULL with workspace_floats = FE_WORKSPACE_LIBRARY: the stream's slot of
 * the library scratch, as for fe_paged_attention_ex; also in fe_paged_decode_kv_exchange_bf16).
 * token_begin must be a multiple of block_size. Used for KV-range sharding across
 * GPUs: each GPU runs its own window, the merged partials are all-gathered and
 * fe_merge_partials combines them. New (the reference has no paged split-KV). */
int fe_paged_decode_partials_bf16(const void* q, const void* k_cache, const void* v_cache,
                                  const int* block_tables, const int* context_lens, int num_seqs,
                                  int num_heads, int num_kv_heads, int head_dim, int block_size,
                                  int max_blocks_per_seq, int num_blocks, float scale,
                                  int token_begin, int token_end, float* workspace,
                                  size_t workspace_floats, float* merged_out,
                                  float* merged_stats, void* stream);

/* Log-sum-exp combine of partials -- the stage-2 reduction of
 * src/flash_decoding.cu:151-223 / python/flash_engine/ops.py:133-143:
 * g = max m_p; L = sum l_p 2^(m_p-g); O = sum O_p 2^(m_p-g) / L.
 * The partials of output row `row` from rank r, split p live at index
 * ((r * rows + row) * parts_per_rank + p) of part_out (times head_dim) and of
 * part_stats (times 2): ranks = 1 is the plain [rows, P, ...] scratch of one
 * launch; ranks > 1 is the [ranks, rows, P, ...] buffer an all-gather produces.
 * Output:
 *   out_dtype 0: fp32 final  [rows, d] in out
 *   out_dtype 1: bf16 final  [rows, d] in out
 *   out_dtype 2: merged partial, out = O (fp32, unnormalised) [rows, d] and
 *                out_stats = (g, L) [rows, 2].
 * Rows whose partials are all empty (l = 0) produce zeros (and (-inf, 0)). */
int fe_merge_partials(const float* part_out, const float* part_stats, int rows, int ranks,
                      int parts_per_rank, int head_dim, void* out, float* out_stats,
                      int out_dtype, void* stream);

/* ---------------------------------------------------------------- KV-range exchange
 * KV-range-sharded decode with the all-gather done by the decode kernel itself over
 * peer memory (NVLink), replacing fe_paged_decode_partials_bf16 + an NCCL all-gather
 * + fe_merge_partials. New: the reference is single-GPU.
 *
 * Every rank owns one exchange buffer of fe_kv_exchange_bytes(world, max_rows,
 * head_dim) bytes (fe_kv_exchange_alloc: cudaMalloc + zero fill, synchronous) and maps
 * the other ranks' buffers (fe_kv_exchange_ipc_handle on the owner, the 64-byte handle
 * sent to the others, fe_kv_exchange_ipc_open there). xbufs[r] is rank r's buffer as
 * seen by this process (xbufs[rank] is its own).
 *
 * fe_paged_decode_kv_exchange_bf16 over the token window [token_begin, token_end):
 *   phases & 1: the decode kernel computes one (O, m, l) partial per (sequence, query
 *     head) row, as fe_paged_decode_partials_bf16 does, and stores it into slot
 *     [rank] of every rank's buffer as 8-byte words tagged with the step number.
 *   phases & 2: a merge kernel reads every rank's words of each row, re-reading
 *     (bounded, 2 s) those not yet tagged with this step, combines the world partials
 *     (log-sum-exp, as fe_merge_partials) into out [S, H, d] bf16, and advances the
 *     step count. head_dim 64 or 128.
 * phases = 3 on one GPU per rank. Ranks emulated on one GPU must run phase 1 of
 * every rank before phase 2 of any. All ranks must call it the same number of times;
 * two generations of slots let a rank run one step ahead of a slower one. Requires
 * num_seqs <= 4096 and num_seqs * num_heads <= max_rows; workspace as for
 * fe_paged_attention_v2_bf16. A wait that runs out sets bit 0 of the device error
 * word and writes zeros. */
size_t fe_kv_exchange_bytes(int world, int max_rows, int head_dim);
int fe_kv_exchange_alloc(size_t bytes, void** ptr);
int fe_kv_exchange_free(void* ptr);
int fe_kv_exchange_ipc_handle(void* ptr, void* handle_out /* 64 bytes */);
int fe_kv_exchange_ipc_open(const void* handle /* 64 bytes */, void** ptr);
int fe_kv_exchange_ipc_close(void* ptr);
int fe_paged_decode_kv_exchange_bf16(const void* q, const void* k_cache, const void* v_cache,
                                     const int* block_tables, const int* context_lens,
                                     int num_seqs, int num_heads, int num_kv_heads,
                                     int head_dim, int block_size, int max_blocks_per_seq,
                                     int num_blocks, float scale, int token_begin, int token_end,
                                     float* workspace, size_t workspace_floats,
                                     void* const* xbufs, int world, int rank, int max_rows,
                                     void* out, int phases, void* stream);

/* ---------------------------------------------------------------- KV-range over NCCL
 * The same KV-range-sharded step with the exchange done by NCCL, for hosts that hold an
 * NCCL communicator (one rank per GPU). New: the reference is single-GPU.
 * NCCL is not linked: its functions are taken at run time from the libnccl.so.2
 * already loaded in the process, else the system's. Without NCCL these return
 * cudaErrorNotSupported (801); an NCCL failure returns 1000 + its ncclResult_t.
 *   fe_nccl_unique_id: ncclGetUniqueId into 128 bytes (rank 0 sends them to the others).
 *   fe_nccl_comm_init / fe_nccl_comm_destroy: ncclCommInitRank / ncclCommDestroy on
 *     the current device; the communicator is an ncclComm_t.
 *   fe_paged_decode_kv_range_nccl_bf16: rank `rank` of `world` decodes the token window
 *     of its KV range (ceil(max_context_len / world) rounded up to whole blocks, the
 *     last rank to the end; the cache and block table hold that window's blocks), one
 *     ncclAllGather of the (O, m, l) partials, then the log-sum-exp merge into out
 *     [S, H, d] bf16 on every rank. scratch: fe_kv_range_nccl_scratch_floats floats;
 *     workspace as for fe_paged_attention_v2_bf16. Stream-ordered on `stream`, which
 *     must be the communicator's device's. */
int fe_nccl_unique_id(void* id_out /* 128 bytes */);
int fe_nccl_comm_init(void** comm_out, int world, const void* id /* 128 bytes */, int rank);
int fe_nccl_comm_destroy(void* comm);
size_t fe_kv_range_nccl_scratch_floats(int world, int num_seqs, int num_heads, int head_dim);
int fe_paged_decode_kv_range_nccl_bf16(const void* q, const void* k_cache, const void* v_cache,
                                       const int* block_tables, const int* context_lens,
                                       int num_seqs, int num_heads, int num_kv_heads,
                                       int head_dim, int block_size, int max_blocks_per_seq,
                                       int num_blocks, float scale, int max_context_len,
                                       float* workspace, size_t workspace_floats, void* comm,
                                       int rank, int world, float* scratch,
                                       size_t scratch_floats, void* out, void* stream);

/* ---------------------------------------------------------------- CUDA graphs
 * Capture-once / replay-per-step of a decode step (kernels, merges and -- when the
 * recorded function issues them -- NCCL collectives). Wraps the CUDAGraphRunner of
 * include/cuda_graph_runner.h, the C++ class of the reference's
 * include/cuda_graph_runner.h:10-35 / src/cuda_graph_runner.cu:14-55.
 * `record(stream, user)` enqueues the step on `stream` during capture. */
typedef void (*fe_record_fn)(void* stream, void* user);
int fe_graph_capture(fe_record_fn record, void* user, void* stream, void** graph_out);
int fe_graph_launch(void* graph, void* stream);
void fe_graph_destroy(void* graph);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* FLASH_ENGINE_C_H_ */
