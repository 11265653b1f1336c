// Allocation-free variant of clover_b200_paged_decode.
//
// Some callers cannot call cudaMalloc: a serving engine that has reserved
// (almost) all of HBM for its own pool — the KV cache — and hands out nothing
// else, or a host reached through a foreign-function binding that has no CUDA
// allocator at all.  They still need split-K decode, whose partial results
// live in scratch memory.  This entry point takes that scratch from a
// file-scope device array of fixed size instead of a caller-provided
// workspace, so the caller passes only inputs and outputs.
//
// Behaviour:
//   * the array holds CLOVER_B200_NOALLOC_SCRATCH_BYTES bytes on every GPU that
//     loads the library, for the life of the process;
//   * calls whose split-K workspace would exceed that size are rejected with
//     CLOVER_B200_ERR_WORKSPACE and a message naming both sizes; nothing runs;
//   * the first call on a device looks up the array's device address
//     (cudaGetSymbolAddress, with that device current) and caches it; make
//     that first call before any stream capture;
//   * every call shares the one array and it keeps the last call's contents.
//     Nothing in it needs to start at zero: each call writes every partial it
//     later reads.  Calls that overlap on the GPU (two streams, or two host
//     threads on one device) race on the array and must be serialised;
//   * no cudaMalloc, cudaFree or other allocating routine is called.
#include <mutex>

#include "common.cuh"

namespace clover {

static __device__ __align__(256) uint8_t g_noalloc_scratch[CLOVER_B200_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
static void* g_scratch_ptr[kMaxDevices] = {};
static std::mutex g_scratch_mu;

// Device address of this device's copy of the scratch array (set-up on first use).
static int scratch_for_current_device(void** out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(CLOVER_B200_ERR_UNSUPPORTED, "paged_decode_noalloc: device ordinal %d", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* p = nullptr;
    rc = check_cuda(cudaGetSymbolAddress(&p, g_noalloc_scratch), "cudaGetSymbolAddress(scratch)");
    if (rc) return rc;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return CLOVER_B200_OK;
}

}  // namespace clover

using namespace clover;

extern "C" int clover_b200_paged_decode_noalloc(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, int32_t q_dtype,
    const void* k_cache, const void* v_cache, int32_t kv_dtype, int64_t num_blocks,
    int32_t block_size, const int32_t* block_tables, int32_t table_stride,
    const int32_t* seq_rows, const int32_t* query_start_loc, const int32_t* ctx_lens,
    int32_t n_seqs, int32_t n_query_rows, int32_t max_queries_per_seq, int32_t max_ctx_len,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, float score_scale,
    int32_t partition_tokens, int32_t* dev_status, void* stream) {
  // The plan query returns the same code (and message) clover_b200_paged_decode
  // would for these sizes (invalid sizes, or an unsupported dtype / shape).
  const int plan_rc = clover_b200_decode_partition_tokens(
      n_seqs, n_query_rows, max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads, head_dim,
      block_size, kv_dtype, q_dtype, partition_tokens);
  if (plan_rc < 0) return plan_rc;
  const int64_t need = clover_b200_decode_workspace_bytes(
      n_seqs, n_query_rows, max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads, head_dim,
      block_size, kv_dtype, q_dtype, partition_tokens);
  if (need < 0) return CLOVER_B200_ERR_INVALID_ARG;  // unreachable once the plan query passed
  if (need > (int64_t)CLOVER_B200_NOALLOC_SCRATCH_BYTES)
    return set_error(CLOVER_B200_ERR_WORKSPACE,
                     "paged_decode_noalloc: split-K scratch of %lld bytes exceeds the static "
                     "maximum of %lld bytes (fewer query rows, shorter contexts or larger "
                     "partition_tokens fit; or use clover_b200_paged_decode with a workspace)",
                     (long long)need, (long long)CLOVER_B200_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (need > 0) {
    const int rc = scratch_for_current_device(&scratch);
    if (rc) return rc;
  }
  return clover_b200_paged_decode(out, out_row_stride, q, q_row_stride, q_dtype, k_cache, v_cache,
                                  kv_dtype, num_blocks, block_size, block_tables, table_stride,
                                  seq_rows, query_start_loc, ctx_lens, n_seqs, n_query_rows,
                                  max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads,
                                  head_dim, score_scale, partition_tokens, scratch,
                                  (int64_t)CLOVER_B200_NOALLOC_SCRATCH_BYTES, dev_status, stream);
}
