/*
 * clover_b200.h — C ABI of the B200-native paged decode-attention library
 * (libclover_b200.so).
 *
 * It is the drop-in boundary for CloverInfer's attention hot path: the
 * per-layer decode of `AttentionNode` (src/core/nodes.py:154) through
 * `CpuAttentionBackend.decode_layer` (src/core/attention_backend.py:82-123)
 * and the paged GPU op behind `KVCacheManager` (src/core/memory_manager.py:19-239,
 * src/kernels/csrc/manager.cpp:19-42).
 *
 * Conventions
 *   - Plain device pointers and sizes; no framework types.  All memory is
 *     caller-owned (the caller allocates caches, tables, outputs and the
 *     split-K workspace).  The one entry point that allocates device memory
 *     is clover_b200_ipc_alloc, the set-up of a fused-gather receive buffer
 *     (cudaMalloc, so that peers can map it with CUDA IPC); no decode, append
 *     or allocator call allocates.
 *   - Every entry point returns CLOVER_B200_OK (0) or a negative
 *     CLOVER_B200_ERR_* code and never throws; clover_b200_last_error()
 *     returns a thread-local description of the last failure.
 *   - Work is enqueued on `stream` (a cudaStream_t passed as void*; NULL =
 *     the legacy default stream) and is asynchronous.
 *   - Kernels report bad indices (slot or block id out of range, table
 *     overflow, allocator exhaustion) by OR-ing CLOVER_B200_DEV_* bits into
 *     the caller's int32 `dev_status` word; the offending element is skipped.
 *     No kernel traps.
 *   - Layouts follow KVCacheManager: one cache per layer for K and one for V,
 *     `[num_blocks, block_size, num_kv_heads, head_dim]` contiguous
 *     (memory_manager.py:35-46); token `t` of a sequence lives in slot
 *     `table[t / block_size] * block_size + t % block_size`; padded tables
 *     hold -1 (memory_manager.py:167).
 */
#ifndef CLOVER_B200_H
#define CLOVER_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define CLOVER_B200_API __attribute__((visibility("default")))
#else
#define CLOVER_B200_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (host return values) ---------------------------------- */
#define CLOVER_B200_OK               0
#define CLOVER_B200_ERR_INVALID_ARG -1  /* null pointer, bad size or stride   */
#define CLOVER_B200_ERR_UNSUPPORTED -2  /* dtype / head_dim / block_size combo */
#define CLOVER_B200_ERR_CUDA        -3  /* a CUDA runtime/driver call failed   */
#define CLOVER_B200_ERR_WORKSPACE   -4  /* split-K workspace too small         */

/* ---- device status bits (OR-ed into *dev_status by kernels) -------------- */
#define CLOVER_B200_DEV_BAD_SLOT      0x1  /* slot >= num_blocks*block_size        */
#define CLOVER_B200_DEV_BAD_BLOCK     0x2  /* table entry outside [0, num_blocks)  */
#define CLOVER_B200_DEV_TABLE_FULL    0x4  /* sequence needs more than table_stride blocks */
#define CLOVER_B200_DEV_OOM           0x8  /* free stack exhausted (batch left unchanged) */
#define CLOVER_B200_DEV_TIMEOUT      0x10  /* a bounded wait gave up                */
#define CLOVER_B200_DEV_CTX_RANGE    0x20  /* a context exceeds max_ctx_len        */

/* ---- dtypes --------------------------------------------------------------- */
#define CLOVER_B200_F32  0
#define CLOVER_B200_F16  1
#define CLOVER_B200_BF16 2
/* KV cache only: 1-byte e4m3 values (no scale; values are stored as given),
 * read by the decode as exact fp16.  Queries and outputs stay F32 or F16;
 * the decode takes it on the tensor-core path (head_dim 128 or 256, block
 * 16 or 32).  No counterpart in the reference, which keeps fp16/fp32 caches. */
#define CLOVER_B200_FP8_E4M3 3

/* Library version (major*10000 + minor*100 + patch). */
CLOVER_B200_API int clover_b200_version(void);

/* Thread-local description of the last error returned on this thread. */
CLOVER_B200_API const char* clover_b200_last_error(void);

/*
 * Limit, in nanoseconds, of the kernels' bounded waits: a TMA copy that has
 * not landed, and the fused gather's wait for the other ranks' words.  When a
 * wait runs out the kernel sets CLOVER_B200_DEV_TIMEOUT in *dev_status and
 * returns (missing gathered values read as 0; later CTAs exit at once until
 * the caller clears the word).  Process-wide; applies to launches made after
 * the call (a captured graph keeps the limit it was captured with).  ns <= 0
 * restores the default of 1 s; values are clamped to [1 ms, 60 s].  Returns
 * the previous limit.  No counterpart in the reference, whose kernels never
 * wait; it bounds how long a rank waits for a peer that failed, the device
 * side of AttentionNode's surfaced errors (src/core/nodes.py:167-170).
 */
CLOVER_B200_API int64_t clover_b200_set_wait_limit_ns(int64_t ns);

/*
 * Host helper: copy n host buffers back to back into dst (a pinned staging
 * buffer), so a batch of per-request tensors becomes one H2D copy.
 * Replaces: the per-item tensor hand-off of AttentionNode.decode_layer_batch
 * (src/core/nodes.py:154) into the batched call; no device work.
 */
CLOVER_B200_API int clover_b200_host_gather(const void* const* srcs, const int64_t* nbytes,
                                            int32_t n, void* dst);

/*
 * Block allocator — the free-block stack and block tables of
 * KVCacheManager, resident in device memory.
 *
 * free_stack[num_blocks] int32 and *free_top (int32, device) form the LIFO
 * stack of memory_manager.py:49 (`list(range(num_blocks))`, top = length):
 * a pop takes free_stack[top-1].  block_tables is [rows, table_stride] int32
 * (-1 padded) and table_len[rows] the number of blocks each row owns.
 */

/*
 * Grow rows so that row rows[i] can hold target_tokens[i] tokens, popping the
 * missing blocks in item order and, within an item, in table order — the
 * same blocks the upstream manager hands out for the equivalent sequence of
 * `allocate(id, seq_len)` (target = seq_len + 1, memory_manager.py:55-72) and
 * `append_slot(id)` calls (target = len + 1, :95-121).  If the whole batch
 * does not fit, nothing changes and CLOVER_B200_DEV_OOM is raised.
 * Replaces: KVCacheManager.allocate / append_slot block growth (memory_manager.py:55-72, :95-121).
 */
CLOVER_B200_API int clover_b200_block_reserve(int32_t* free_stack, int32_t* free_top, int32_t num_blocks,
                              int32_t* block_tables, int32_t table_stride, int32_t* table_len,
                              const int32_t* rows, const int32_t* target_tokens, int32_t n_items,
                              int32_t block_size, int32_t* dev_status, void* stream);

/*
 * Return every block of rows[0..n_items) to the stack, row by row in table
 * order (the upstream `free`, memory_manager.py:134-143), reset the rows to
 * -1 and their length to 0.  Rows that own no block are a no-op.
 * Replaces: KVCacheManager.free (memory_manager.py:134-143).
 */
CLOVER_B200_API int clover_b200_block_free(int32_t* free_stack, int32_t* free_top, int32_t num_blocks,
                           int32_t* block_tables, int32_t table_stride, int32_t* table_len,
                           const int32_t* rows, int32_t n_items, int32_t* dev_status, void* stream);

/*
 * Slot mapping for new tokens: item i writes tokens at positions
 * positions[i] .. positions[i] + (token_offsets[i+1]-token_offsets[i]) - 1
 * of table row rows[i]; slot_mapping[token_offsets[i] + j] receives the flat
 * slot of position positions[i]+j.  The `(block, offset)` pair that
 * append_slot returns is (slot / block_size, slot % block_size).
 * Replaces: KVCacheManager.append_slot's slot arithmetic (memory_manager.py:113-121).
 */
CLOVER_B200_API int clover_b200_compute_slots(const int32_t* block_tables, int32_t table_stride,
                              const int32_t* rows, const int32_t* positions,
                              const int32_t* token_offsets, int32_t n_items, int32_t block_size,
                              int64_t num_blocks, int64_t* slot_mapping, int32_t* dev_status,
                              void* stream);

/*
 * KV append (reshape-and-cache): copy k_new/v_new token j ([num_kv_heads,
 * head_dim], token stride `new_token_stride` elements) into slot
 * slot_mapping[j] of k_cache/v_cache.  Negative slots are skipped (padding);
 * slots >= num_blocks*block_size raise CLOVER_B200_DEV_BAD_SLOT.  A bit copy.
 * Replaces: KVCacheManager.write_new_kv / load_initial_kv slice stores
 * (memory_manager.py:74-93, :123-132) and the torch.cat append of
 * CpuAttentionBackend.decode_layer (attention_backend.py:105-110).
 */
CLOVER_B200_API int clover_b200_kv_append(void* k_cache, void* v_cache, const void* k_new, const void* v_new,
                          int64_t new_token_stride, const int64_t* slot_mapping, int64_t n_tokens,
                          int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                          int64_t num_blocks, int32_t dtype, int32_t* dev_status, void* stream);

/*
 * KV append for n_layers layers in one launch: layer l's new tokens start at
 * k_new / v_new + l * new_layer_stride elements (token stride
 * new_token_stride, as in clover_b200_kv_append) and go to the caches at
 * k_cache / v_cache + l * cache_layer_stride elements, every layer through
 * the same slot_mapping (all layers of a sequence hold the same tokens).
 * Used to ingest a request's prefill KV of every layer from one staging
 * buffer.  Layer regions must not overlap (the strides are checked).
 * Replaces: the per-layer initial_kv load of CpuAttentionBackend.init_request
 * (attention_backend.py:68-80) fed by the prefill KV export
 * (model_adapter.py:173-182), and KVCacheManager.load_initial_kv
 * (memory_manager.py:74-93) repeated per layer.
 */
CLOVER_B200_API int clover_b200_kv_append_layers(void* k_cache, void* v_cache, int64_t cache_layer_stride,
                          const void* k_new, const void* v_new, int64_t new_layer_stride,
                          int64_t new_token_stride, const int64_t* slot_mapping, int64_t n_tokens,
                          int32_t n_layers, int32_t num_kv_heads, int32_t head_dim,
                          int32_t block_size, int64_t num_blocks, int32_t dtype,
                          int32_t* dev_status, void* stream);

/*
 * partition_tokens = CLOVER_B200_PARTITION_BALANCED asks for the balanced
 * split on the tensor-core path (bf16/fp16 cache, head_dim 64/128/256, block
 * 16/32, at most 1024 sequences): the KV blocks of all sequences are divided
 * evenly over every resident warp instead of into fixed-length partitions, so
 * ragged batches launch no empty work.  Elsewhere, and for the sharded step
 * (clover_b200_decode_step_gather and its workspace query), it means the
 * library's choice (as 0).
 */
#define CLOVER_B200_PARTITION_BALANCED (-1)

/*
 * Bytes of split-K workspace clover_b200_paged_decode needs for a call with
 * the same sizes, dtypes and partition_tokens (0 = the library's choice);
 * 0 when every context fits one partition, -1 on invalid sizes.
 */
CLOVER_B200_API int64_t clover_b200_decode_workspace_bytes(int32_t n_seqs, int32_t n_query_rows,
                                           int32_t max_queries_per_seq, int32_t max_ctx_len,
                                           int32_t num_q_heads, int32_t num_kv_heads,
                                           int32_t head_dim, int32_t block_size, int32_t kv_dtype,
                                           int32_t q_dtype, int32_t partition_tokens);

/*
 * The split-K partition length (tokens) clover_b200_paged_decode uses for a
 * call with these sizes (the library's choice when partition_tokens = 0; 0
 * for the balanced split), or a negative error code.
 */
CLOVER_B200_API int clover_b200_decode_partition_tokens(int32_t n_seqs, int32_t n_query_rows,
                                           int32_t max_queries_per_seq, int32_t max_ctx_len,
                                           int32_t num_q_heads, int32_t num_kv_heads,
                                           int32_t head_dim, int32_t block_size, int32_t kv_dtype,
                                           int32_t q_dtype, int32_t partition_tokens);

/*
 * Paged decode attention with GQA and split-K (flash-decoding).
 *
 * Batch of n_seqs sequences; sequence b owns query rows
 * query_start_loc[b] .. query_start_loc[b+1]-1 (one row per new token; a
 * plain decode step has query_start_loc = 0,1,..,n_seqs) and block-table row
 * seq_rows ? seq_rows[b] : b.  Query row r attends causally to tokens
 * [0, ctx_lens[r]) of its sequence.
 *
 *   q   [n_rows, num_q_heads, head_dim]  row stride q_row_stride elements,
 *                                          dtype q_dtype (F32 or kv_dtype)
 *   out [n_rows, num_q_heads, head_dim]  row stride out_row_stride, dtype q_dtype
 *   out[r,h,:] = softmax(score_scale * q[r,h,:] . K^T) . V  over the KV head
 *                h / (num_q_heads / num_kv_heads), accumulated in fp32.
 *
 * score_scale is applied by the kernel (q may be pre-scaled, as OPT does
 * upstream: model_adapter.py:373, :386).  partition_tokens = 0 lets the
 * library pick the split; an explicit value must be a multiple of
 * block_size and at most 64 * block_size on the tensor-core path; workspace must hold
 * clover_b200_decode_workspace_bytes(...) bytes (device) — it may be NULL
 * when every context fits in one partition.  Within a call, zero-length
 * contexts produce zeros.
 * Replaces: CpuAttentionBackend.decode_layer scoring (attention_backend.py:113-118),
 * KVCacheManager.attention (memory_manager.py:175-190) and
 * paged_attention (src/kernels/csrc/manager.cpp:19-38, attention.cu:16-149).
 */
CLOVER_B200_API int clover_b200_paged_decode(void* out, int64_t out_row_stride,
                             const void* q, int64_t q_row_stride, int32_t q_dtype,
                             const void* k_cache, const void* v_cache, int32_t kv_dtype,
                             int64_t num_blocks, int32_t block_size,
                             const int32_t* block_tables, int32_t table_stride,
                             const int32_t* seq_rows, const int32_t* query_start_loc,
                             const int32_t* ctx_lens, int32_t n_seqs, int32_t n_query_rows,
                             int32_t max_queries_per_seq, int32_t max_ctx_len,
                             int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                             float score_scale, int32_t partition_tokens,
                             void* workspace, int64_t workspace_bytes,
                             int32_t* dev_status, void* stream);

/*
 * One attention step: KV append fused with paged decode.  Query row r brings
 * one new token, k_new/v_new[r] ([num_kv_heads, head_dim], token stride
 * new_token_stride elements, kv_dtype); it is written to position
 * ctx_lens[r] - 1 of its sequence (the block table must already cover that
 * position) and then every row attends exactly as clover_b200_paged_decode.
 * When a sequence's columns (rows x GQA group) fit one CTA (the usual decode
 * step) the append happens inside the decode kernel — the CTA owning the
 * token's partition writes it before its TMA loads — otherwise a separate
 * append kernel runs first.  Same workspace as clover_b200_paged_decode.
 * Replaces: the append-then-attend of CpuAttentionBackend.decode_layer
 * (attention_backend.py:105-118) and AttnPartition's write_new_kv + attention
 * (src/core/graph_compiler.py:115-122).
 */
CLOVER_B200_API int clover_b200_decode_step(void* out, int64_t out_row_stride,
                             const void* q, int64_t q_row_stride, int32_t q_dtype,
                             void* k_cache, void* v_cache, int32_t kv_dtype,
                             int64_t num_blocks, int32_t block_size,
                             const void* k_new, const void* v_new, int64_t new_token_stride,
                             const int32_t* block_tables, int32_t table_stride,
                             const int32_t* seq_rows, const int32_t* query_start_loc,
                             const int32_t* ctx_lens, int32_t n_seqs, int32_t n_query_rows,
                             int32_t max_queries_per_seq, int32_t max_ctx_len,
                             int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                             float score_scale, int32_t partition_tokens,
                             void* workspace, int64_t workspace_bytes,
                             int32_t* dev_status, void* stream);

/*
 * Fused output all-gather for KV-head sharding (one process per GPU of a node).
 *
 * Rank r of n_ranks owns the contiguous query heads [r * num_q_heads,
 * (r + 1) * num_q_heads) of total = n_ranks * num_q_heads (equal shards).
 * decode_step_gather runs the fused append + decode of clover_b200_decode_step
 * and then a split-K reduce that sends every output value, tagged with the
 * call's epoch in one 8-byte word, straight into EVERY rank's receive buffer
 * over NVLink (plain peer stores, no multicast), waits (bounded) for the
 * words of its rows from every rank and writes out[rows, total, head_dim]
 * (row stride out_row_stride, q dtype): the all-gathered output, on every
 * rank, without a fence, a global barrier or a second kernel.
 *
 *   peer_recv[n_ranks]  device array of each rank's receive buffer (mapped here
 *                       with clover_b200_ipc_open; this rank's own at [rank]):
 *                       2 * recv_half_words uint64 words, zeroed at allocation.
 *   sync                this rank's clover_b200_gather_sync_bytes() of
 *                       zeroed device memory (call count, CTA count).
 *
 * Every rank must make the same sequence of calls with the same sizes.  A
 * rank that does not arrive within 1 s makes the others finish with
 * CLOVER_B200_DEV_TIMEOUT set (missing values read as 0).  Workspace:
 * clover_b200_decode_gather_workspace_bytes(...).  k_new/v_new may be NULL
 * (attend only).  Replaces: the per-layer hand-off of attention contexts to the
 * dense node (src/core/scheduler.py:1058-1059) for heads split across GPUs by
 * the head-grouping policy (src/core/attention_backend.py:429-438).
 */
#define CLOVER_B200_IPC_HANDLE_BYTES 64

/* cudaMalloc'd, zeroed device buffer plus its IPC handle (64 bytes). */
CLOVER_B200_API int clover_b200_ipc_alloc(int64_t bytes, void** dev_ptr, void* handle);
/* Map a peer process's buffer from its handle (enables peer access). */
CLOVER_B200_API int clover_b200_ipc_open(const void* handle, void** dev_ptr);
/* Unmap a buffer opened with clover_b200_ipc_open. */
CLOVER_B200_API int clover_b200_ipc_close(void* dev_ptr);
/* Free a buffer from clover_b200_ipc_alloc (after every peer closed it). */
CLOVER_B200_API int clover_b200_ipc_free(void* dev_ptr);
CLOVER_B200_API int64_t clover_b200_gather_sync_bytes(void);
CLOVER_B200_API int64_t clover_b200_decode_gather_workspace_bytes(int32_t n_seqs,
                                           int32_t n_query_rows, int32_t max_queries_per_seq,
                                           int32_t max_ctx_len, int32_t num_q_heads,
                                           int32_t num_kv_heads, int32_t head_dim,
                                           int32_t block_size, int32_t kv_dtype, int32_t q_dtype,
                                           int32_t partition_tokens);
CLOVER_B200_API int clover_b200_decode_step_gather(void* out, int64_t out_row_stride,
                             const void* q, int64_t q_row_stride, int32_t q_dtype,
                             void* k_cache, void* v_cache, int32_t kv_dtype,
                             int64_t num_blocks, int32_t block_size,
                             const void* k_new, const void* v_new, int64_t new_token_stride,
                             const int32_t* block_tables, int32_t table_stride,
                             const int32_t* seq_rows, const int32_t* query_start_loc,
                             const int32_t* ctx_lens, int32_t n_seqs, int32_t n_query_rows,
                             int32_t max_queries_per_seq, int32_t max_ctx_len,
                             int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                             float score_scale, int32_t partition_tokens,
                             void* const* peer_recv, int32_t* sync, int32_t n_ranks, int32_t rank,
                             int64_t recv_half_words, void* workspace, int64_t workspace_bytes,
                             int32_t* dev_status, void* stream);

/*
 * clover_b200_decode_step_gather writing the all-gathered output in out_dtype
 * (F32, F16 or BF16, independent of q_dtype) into a caller-given consumer
 * buffer: row r of out (row stride out_row_stride elements) receives the
 * [total_q_heads * head_dim] context of query row r, e.g. the dense node's
 * o_proj input [rows, hidden] in the model's dtype.  Every other argument and
 * result as clover_b200_decode_step_gather.
 * Replaces: the hand-off of the gathered contexts to the dense node, which
 * reshapes them into its o_proj input (src/core/scheduler.py:1058-1059,
 * src/core/model_adapter.py:572).
 */
CLOVER_B200_API int clover_b200_decode_step_gather_into(void* out, int64_t out_row_stride,
                             int32_t out_dtype, const void* q, int64_t q_row_stride, int32_t q_dtype,
                             void* k_cache, void* v_cache, int32_t kv_dtype,
                             int64_t num_blocks, int32_t block_size,
                             const void* k_new, const void* v_new, int64_t new_token_stride,
                             const int32_t* block_tables, int32_t table_stride,
                             const int32_t* seq_rows, const int32_t* query_start_loc,
                             const int32_t* ctx_lens, int32_t n_seqs, int32_t n_query_rows,
                             int32_t max_queries_per_seq, int32_t max_ctx_len,
                             int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                             float score_scale, int32_t partition_tokens,
                             void* const* peer_recv, int32_t* sync, int32_t n_ranks, int32_t rank,
                             int64_t recv_half_words, void* workspace, int64_t workspace_bytes,
                             int32_t* dev_status, void* stream);

/*
 * Allocation-free paged decode.  No counterpart in the upstream project: it
 * exists for callers that cannot call cudaMalloc (a serving engine that owns
 * all of HBM through its own pool, or a foreign-function host without a CUDA
 * allocator).  Same arguments and results as clover_b200_paged_decode minus
 * the workspace: split-K scratch comes from a static device array of
 * CLOVER_B200_NOALLOC_SCRATCH_BYTES held by every GPU that loads the library.
 * Calls needing more scratch than that return CLOVER_B200_ERR_WORKSPACE.  The
 * first call on a device looks the array up (make it before any stream
 * capture).  All calls share the array: calls that overlap on the GPU race.
 */
#define CLOVER_B200_NOALLOC_SCRATCH_BYTES (16ll << 20)

CLOVER_B200_API int clover_b200_paged_decode_noalloc(void* out, int64_t out_row_stride,
                             const void* q, int64_t q_row_stride, int32_t q_dtype,
                             const void* k_cache, const void* v_cache, int32_t kv_dtype,
                             int64_t num_blocks, int32_t block_size,
                             const int32_t* block_tables, int32_t table_stride,
                             const int32_t* seq_rows, const int32_t* query_start_loc,
                             const int32_t* ctx_lens, int32_t n_seqs, int32_t n_query_rows,
                             int32_t max_queries_per_seq, int32_t max_ctx_len,
                             int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
                             float score_scale, int32_t partition_tokens,
                             int32_t* dev_status, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* CLOVER_B200_H */
