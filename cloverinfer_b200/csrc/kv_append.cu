// KV append (reshape-and-cache): scatter new tokens' K/V rows into their
// paged slots.  Replaces the per-token slice stores of KVCacheManager
// (src/core/memory_manager.py:74-93, :123-132) and the torch.cat append of
// CpuAttentionBackend.decode_layer (src/core/attention_backend.py:105-110).
//
// One token's K (or V) for all local heads is a contiguous
// [num_kv_heads * head_dim] row in both the source and its cache slot, so the
// copy is a row copy in 16-byte vectors: HBM-bound, bit-exact.
#include "common.cuh"

namespace clover {

// vec-aligned path: one thread per 16-byte vector of a row; grid-stride.
// blockIdx.y is the layer: layer l reads its tokens at l * src_layer_vec and
// writes its cache at l * cache_layer_vec (16-byte units).
__global__ void kv_append_vec_kernel(uint4* __restrict__ kc, uint4* __restrict__ vc,
                                     const uint4* __restrict__ kn, const uint4* __restrict__ vn,
                                     int64_t src_stride_vec, const int64_t* __restrict__ slots,
                                     int64_t n_tokens, int32_t row_vecs, int64_t n_slots,
                                     int32_t* __restrict__ status, int64_t cache_layer_vec,
                                     int64_t src_layer_vec) {
  kc += blockIdx.y * cache_layer_vec;
  vc += blockIdx.y * cache_layer_vec;
  kn += blockIdx.y * src_layer_vec;
  vn += blockIdx.y * src_layer_vec;
  const int64_t total = n_tokens * row_vecs;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = idx / row_vecs;
    const int32_t v = (int32_t)(idx - t * row_vecs);
    const int64_t slot = __ldg(slots + t);
    if (slot < 0) continue;  // padding token
    if (slot >= n_slots) {
      if (v == 0) raise_status(status, CLOVER_B200_DEV_BAD_SLOT);
      continue;
    }
    const int64_t src = t * src_stride_vec + v;
    const int64_t dst = slot * row_vecs + v;
    kc[dst] = __ldg(kn + src);
    vc[dst] = __ldg(vn + src);
  }
}

// element path for rows that are not 16-byte multiples / aligned.
template <typename E>
__global__ void kv_append_elem_kernel(E* __restrict__ kc, E* __restrict__ vc,
                                      const E* __restrict__ kn, const E* __restrict__ vn,
                                      int64_t src_stride, const int64_t* __restrict__ slots,
                                      int64_t n_tokens, int32_t row_elems, int64_t n_slots,
                                      int32_t* __restrict__ status, int64_t cache_layer,
                                      int64_t src_layer) {
  kc += blockIdx.y * cache_layer;
  vc += blockIdx.y * cache_layer;
  kn += blockIdx.y * src_layer;
  vn += blockIdx.y * src_layer;
  const int64_t total = n_tokens * row_elems;
  for (int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = idx / row_elems;
    const int32_t e = (int32_t)(idx - t * row_elems);
    const int64_t slot = slots[t];
    if (slot < 0) continue;
    if (slot >= n_slots) {
      if (e == 0) raise_status(status, CLOVER_B200_DEV_BAD_SLOT);
      continue;
    }
    kc[slot * row_elems + e] = kn[t * src_stride + e];
    vc[slot * row_elems + e] = vn[t * src_stride + e];
  }
}

static inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace clover

using namespace clover;

// Shared body of kv_append (one layer) and kv_append_layers.
static int append_impl(void* k_cache, void* v_cache, int64_t cache_layer_stride,
                       const void* k_new, const void* v_new, int64_t new_layer_stride,
                       int64_t new_token_stride, const int64_t* slot_mapping, int64_t n_tokens,
                       int32_t n_layers, int32_t num_kv_heads, int32_t head_dim,
                       int32_t block_size, int64_t num_blocks, int32_t dtype,
                       int32_t* dev_status, void* stream) {
  if (n_tokens < 0 || n_layers < 0 || n_layers > 65535 || num_kv_heads <= 0 || head_dim <= 0 ||
      block_size <= 0 || num_blocks < 0)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "kv_append: bad sizes");
  if (n_tokens == 0 || n_layers == 0) return CLOVER_B200_OK;
  if (!k_cache || !v_cache || !k_new || !v_new || !slot_mapping)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "kv_append: null pointer");
  int esz;
  switch (dtype) {
    case CLOVER_B200_F32: esz = 4; break;
    case CLOVER_B200_F16:
    case CLOVER_B200_BF16: esz = 2; break;
    case CLOVER_B200_FP8_E4M3: esz = 1; break;
    default: return set_error(CLOVER_B200_ERR_UNSUPPORTED, "kv_append: dtype %d", dtype);
  }
  const int32_t row_elems = num_kv_heads * head_dim;
  if (new_token_stride < row_elems)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "kv_append: token stride < heads*head_dim");
  const int64_t n_slots = num_blocks * (int64_t)block_size;
  if (n_layers > 1 && (cache_layer_stride < n_slots * row_elems ||
                       new_layer_stride < (n_tokens - 1) * new_token_stride + row_elems))
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "kv_append_layers: layer strides overlap");
  cudaStream_t s = (cudaStream_t)stream;
  const int threads = 256;
  const bool vec = ((int64_t)row_elems * esz) % 16 == 0 && (new_token_stride * esz) % 16 == 0 &&
                   (cache_layer_stride * esz) % 16 == 0 && (new_layer_stride * esz) % 16 == 0 &&
                   aligned16(k_cache) && aligned16(v_cache) && aligned16(k_new) &&
                   aligned16(v_new);
  // ~16 CTAs per SM over all layers
  const int64_t per_layer_cap = (148 * 16 + n_layers - 1) / n_layers;
  if (vec) {
    const int32_t row_vecs = row_elems * esz / 16;
    const int64_t total = n_tokens * row_vecs;
    const int64_t want = (total + threads - 1) / threads;
    const dim3 grid((unsigned)(want < per_layer_cap ? want : per_layer_cap), (unsigned)n_layers);
    kv_append_vec_kernel<<<grid, threads, 0, s>>>(
        (uint4*)k_cache, (uint4*)v_cache, (const uint4*)k_new, (const uint4*)v_new,
        new_token_stride * esz / 16, slot_mapping, n_tokens, row_vecs, n_slots, dev_status,
        cache_layer_stride * esz / 16, new_layer_stride * esz / 16);
  } else {
    const int64_t total = n_tokens * row_elems;
    const int64_t want = (total + threads - 1) / threads;
    const dim3 grid((unsigned)(want < per_layer_cap ? want : per_layer_cap), (unsigned)n_layers);
    if (esz == 4) {
      kv_append_elem_kernel<uint32_t><<<grid, threads, 0, s>>>(
          (uint32_t*)k_cache, (uint32_t*)v_cache, (const uint32_t*)k_new, (const uint32_t*)v_new,
          new_token_stride, slot_mapping, n_tokens, row_elems, n_slots, dev_status,
          cache_layer_stride, new_layer_stride);
    } else if (esz == 2) {
      kv_append_elem_kernel<uint16_t><<<grid, threads, 0, s>>>(
          (uint16_t*)k_cache, (uint16_t*)v_cache, (const uint16_t*)k_new, (const uint16_t*)v_new,
          new_token_stride, slot_mapping, n_tokens, row_elems, n_slots, dev_status,
          cache_layer_stride, new_layer_stride);
    } else {
      kv_append_elem_kernel<uint8_t><<<grid, threads, 0, s>>>(
          (uint8_t*)k_cache, (uint8_t*)v_cache, (const uint8_t*)k_new, (const uint8_t*)v_new,
          new_token_stride, slot_mapping, n_tokens, row_elems, n_slots, dev_status,
          cache_layer_stride, new_layer_stride);
    }
  }
  return check_cuda(cudaGetLastError(), "kv_append launch");
}

extern "C" int clover_b200_kv_append(void* k_cache, void* v_cache, const void* k_new,
                                     const void* v_new, int64_t new_token_stride,
                                     const int64_t* slot_mapping, int64_t n_tokens,
                                     int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
                                     int64_t num_blocks, int32_t dtype, int32_t* dev_status,
                                     void* stream) {
  return append_impl(k_cache, v_cache, 0, k_new, v_new, 0, new_token_stride, slot_mapping,
                     n_tokens, 1, num_kv_heads, head_dim, block_size, num_blocks, dtype,
                     dev_status, stream);
}

extern "C" int clover_b200_kv_append_layers(void* k_cache, void* v_cache,
                                            int64_t cache_layer_stride, const void* k_new,
                                            const void* v_new, int64_t new_layer_stride,
                                            int64_t new_token_stride,
                                            const int64_t* slot_mapping, int64_t n_tokens,
                                            int32_t n_layers, int32_t num_kv_heads,
                                            int32_t head_dim, int32_t block_size,
                                            int64_t num_blocks, int32_t dtype,
                                            int32_t* dev_status, void* stream) {
  return append_impl(k_cache, v_cache, cache_layer_stride, k_new, v_new, new_layer_stride,
                     new_token_stride, slot_mapping, n_tokens, n_layers, num_kv_heads, head_dim,
                     block_size, num_blocks, dtype, dev_status, stream);
}
