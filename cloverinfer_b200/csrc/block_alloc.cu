// Device-resident KV block allocator: LIFO free stack + per-row block tables.
//
// Semantics follow KVCacheManager (src/core/memory_manager.py):
//   free stack  = list(range(num_blocks)), pop() from the end      (:49, :69, :110)
//   allocate    = ceil((seq_len + 1) / bs) blocks                  (:59)
//   append_slot = one pop when len == len(table) * bs              (:104-111)
//   free        = push the row's blocks back in table order        (:139-140)
// A batch is applied in item order, so the blocks each row receives are the
// ones the upstream manager would hand out for the same call sequence.  The
// whole batch is checked first: if it does not fit, nothing changes.
#include <cub/block/block_reduce.cuh>
#include <cub/block/block_scan.cuh>

#include "common.cuh"

namespace clover {

constexpr int kAllocThreads = 512;

__device__ __forceinline__ int32_t blocks_for(int32_t tokens, int32_t bs) {
  return tokens <= 0 ? 0 : (tokens + bs - 1) / bs;
}

// Index of the item whose [off[i], off[i] + n[i]) range holds k (off ascending).
__device__ __forceinline__ int find_item(const int32_t* off, int n, int32_t k) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (off[mid] <= k) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__global__ void __launch_bounds__(kAllocThreads)
block_reserve_kernel(int32_t* __restrict__ free_stack, int32_t* __restrict__ free_top,
                     int32_t num_blocks, int32_t* __restrict__ tables, int32_t stride,
                     int32_t* __restrict__ table_len, const int32_t* __restrict__ rows,
                     const int32_t* __restrict__ target, int32_t n, int32_t bs,
                     int32_t* __restrict__ status) {
  using Scan = cub::BlockScan<int32_t, kAllocThreads>;
  using Reduce = cub::BlockReduce<int32_t, kAllocThreads>;
  __shared__ union {
    typename Scan::TempStorage scan;
    typename Reduce::TempStorage reduce;
  } tmp;
  __shared__ int32_t s_off[kAllocThreads], s_row[kAllocThreads], s_have[kAllocThreads];
  __shared__ int32_t s_total, s_bad, s_chunk;
  const int tid = threadIdx.x;
  if (tid == 0) {
    s_total = 0;
    s_bad = 0;
  }
  __syncthreads();

  // Pass 1: total demand and validity (the batch is all-or-nothing).
  for (int base = 0; base < n; base += kAllocThreads) {
    const int i = base + tid;
    int32_t need = 0, bad = 0;
    if (i < n) {
      const int32_t want = blocks_for(target[i], bs);
      const int32_t have = table_len[rows[i]];
      if (want > stride) bad = CLOVER_B200_DEV_TABLE_FULL;
      need = want > have ? want - have : 0;
    }
    const int32_t tot = Reduce(tmp.reduce).Sum(need);
    __syncthreads();
    const int32_t anybad = Reduce(tmp.reduce).Reduce(bad, cub::Max());
    if (tid == 0) {
      s_total += tot;
      s_bad |= anybad;
    }
    __syncthreads();
  }
  const int32_t top = *free_top;
  if (s_bad || s_total > top || top > num_blocks) {
    if (tid == 0) raise_status(status, s_bad ? s_bad : CLOVER_B200_DEV_OOM);
    return;
  }

  // Pass 2: pops in item order — item i takes stack[top-1-(off_i+j)], j < need_i.
  // The pops of a chunk are spread over all threads (binary search of the scan).
  int32_t running = 0;
  for (int base = 0; base < n; base += kAllocThreads) {
    const int i = base + tid;
    const int cnt = min(kAllocThreads, n - base);
    int32_t need = 0, have = 0, row = 0;
    if (i < n) {
      row = rows[i];
      const int32_t want = blocks_for(target[i], bs);
      have = table_len[row];
      need = want > have ? want - have : 0;
    }
    int32_t off, chunk_total;
    Scan(tmp.scan).ExclusiveSum(need, off, chunk_total);
    s_off[tid] = off;
    s_row[tid] = row;
    s_have[tid] = have;
    if (tid == 0) s_chunk = chunk_total;
    __syncthreads();
    for (int32_t k = tid; k < s_chunk; k += kAllocThreads) {
      const int it = find_item(s_off, cnt, k);
      const int32_t j = k - s_off[it];
      tables[(int64_t)s_row[it] * stride + s_have[it] + j] = free_stack[top - 1 - (running + k)];
    }
    if (i < n && need > 0) table_len[row] = have + need;
    running += s_chunk;
    __syncthreads();
  }
  if (tid == 0) *free_top = top - s_total;
}

__global__ void __launch_bounds__(kAllocThreads)
block_free_kernel(int32_t* __restrict__ free_stack, int32_t* __restrict__ free_top,
                  int32_t num_blocks, int32_t* __restrict__ tables, int32_t stride,
                  int32_t* __restrict__ table_len, const int32_t* __restrict__ rows, int32_t n,
                  int32_t* __restrict__ status) {
  using Scan = cub::BlockScan<int32_t, kAllocThreads>;
  using Reduce = cub::BlockReduce<int32_t, kAllocThreads>;
  __shared__ union {
    typename Scan::TempStorage scan;
    typename Reduce::TempStorage reduce;
  } tmp;
  __shared__ int32_t s_off[kAllocThreads], s_row[kAllocThreads];
  __shared__ int32_t s_total, s_chunk;
  const int tid = threadIdx.x;
  if (tid == 0) s_total = 0;
  __syncthreads();
  for (int base = 0; base < n; base += kAllocThreads) {
    const int i = base + tid;
    const int32_t len = i < n ? table_len[rows[i]] : 0;
    const int32_t tot = Reduce(tmp.reduce).Sum(len);
    if (tid == 0) s_total += tot;
    __syncthreads();
  }
  const int32_t top = *free_top;
  if (top + s_total > num_blocks) {  // would overflow the stack: double free
    if (tid == 0) raise_status(status, CLOVER_B200_DEV_BAD_BLOCK);
    return;
  }
  // Pushes in item order, each row's blocks in table order.
  int32_t running = 0;
  for (int base = 0; base < n; base += kAllocThreads) {
    const int i = base + tid;
    const int cnt = min(kAllocThreads, n - base);
    int32_t len = 0, row = 0;
    if (i < n) {
      row = rows[i];
      len = table_len[row];
    }
    int32_t off, chunk_total;
    Scan(tmp.scan).ExclusiveSum(len, off, chunk_total);
    s_off[tid] = off;
    s_row[tid] = row;
    if (tid == 0) s_chunk = chunk_total;
    __syncthreads();
    for (int32_t k = tid; k < s_chunk; k += kAllocThreads) {
      const int it = find_item(s_off, cnt, k);
      int32_t* e = tables + (int64_t)s_row[it] * stride + (k - s_off[it]);
      free_stack[top + running + k] = *e;
      *e = -1;
    }
    __syncthreads();
    if (i < n) table_len[row] = 0;
    running += s_chunk;
    __syncthreads();
  }
  if (tid == 0) *free_top = top + s_total;
}

// gridDim.y CTAs per item (x = item); their threads cover the item's new tokens.
__global__ void __launch_bounds__(128)
compute_slots_kernel(const int32_t* __restrict__ tables, int32_t stride,
                     const int32_t* __restrict__ rows, const int32_t* __restrict__ positions,
                     const int32_t* __restrict__ offsets, int32_t bs, int64_t num_blocks,
                     int64_t* __restrict__ slots, int32_t* __restrict__ status) {
  const int i = blockIdx.x;
  const int32_t* tab = tables + (int64_t)rows[i] * stride;
  const int32_t pos0 = positions[i];
  const int32_t t0 = offsets[i], t1 = offsets[i + 1];
  const int32_t step = blockDim.x * gridDim.y;
  for (int32_t t = t0 + blockIdx.y * blockDim.x + threadIdx.x; t < t1; t += step) {
    const int32_t pos = pos0 + (t - t0);
    const int32_t bi = pos / bs;
    int64_t slot = -1;
    if (pos >= 0 && bi < stride) {
      const int32_t blk = tab[bi];
      if (blk >= 0 && blk < num_blocks) {
        slot = (int64_t)blk * bs + pos % bs;
      } else {
        raise_status(status, CLOVER_B200_DEV_BAD_BLOCK);
      }
    } else {
      raise_status(status, CLOVER_B200_DEV_TABLE_FULL);
    }
    slots[t] = slot;
  }
}

}  // namespace clover

using namespace clover;

extern "C" int clover_b200_block_reserve(int32_t* free_stack, int32_t* free_top,
                                         int32_t num_blocks, int32_t* block_tables,
                                         int32_t table_stride, int32_t* table_len,
                                         const int32_t* rows, const int32_t* target_tokens,
                                         int32_t n_items, int32_t block_size, int32_t* dev_status,
                                         void* stream) {
  if (n_items < 0 || block_size <= 0 || table_stride <= 0 || num_blocks < 0)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "block_reserve: bad sizes");
  if (n_items == 0) return CLOVER_B200_OK;
  if (!free_stack || !free_top || !block_tables || !table_len || !rows || !target_tokens)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "block_reserve: null pointer");
  block_reserve_kernel<<<1, kAllocThreads, 0, (cudaStream_t)stream>>>(
      free_stack, free_top, num_blocks, block_tables, table_stride, table_len, rows,
      target_tokens, n_items, block_size, dev_status);
  return check_cuda(cudaGetLastError(), "block_reserve launch");
}

extern "C" int clover_b200_block_free(int32_t* free_stack, int32_t* free_top, int32_t num_blocks,
                                      int32_t* block_tables, int32_t table_stride,
                                      int32_t* table_len, const int32_t* rows, int32_t n_items,
                                      int32_t* dev_status, void* stream) {
  if (n_items < 0 || table_stride <= 0 || num_blocks < 0)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "block_free: bad sizes");
  if (n_items == 0) return CLOVER_B200_OK;
  if (!free_stack || !free_top || !block_tables || !table_len || !rows)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "block_free: null pointer");
  block_free_kernel<<<1, kAllocThreads, 0, (cudaStream_t)stream>>>(
      free_stack, free_top, num_blocks, block_tables, table_stride, table_len, rows, n_items,
      dev_status);
  return check_cuda(cudaGetLastError(), "block_free launch");
}

extern "C" int clover_b200_compute_slots(const int32_t* block_tables, int32_t table_stride,
                                         const int32_t* rows, const int32_t* positions,
                                         const int32_t* token_offsets, int32_t n_items,
                                         int32_t block_size, int64_t num_blocks,
                                         int64_t* slot_mapping, int32_t* dev_status,
                                         void* stream) {
  if (n_items < 0 || block_size <= 0 || table_stride <= 0)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "compute_slots: bad sizes");
  if (n_items == 0) return CLOVER_B200_OK;
  if (!block_tables || !rows || !positions || !token_offsets || !slot_mapping)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "compute_slots: null pointer");
  // a few CTAs per item so prefill-sized items (tens of thousands of tokens)
  // are not a single CTA's serial loop
  const int per_item = n_items >= 1024 ? 1 : 16;
  compute_slots_kernel<<<dim3(n_items, per_item), 128, 0, (cudaStream_t)stream>>>(
      block_tables, table_stride, rows, positions, token_offsets, block_size, num_blocks,
      slot_mapping, dev_status);
  return check_cuda(cudaGetLastError(), "compute_slots launch");
}
