// Paged decode attention for B200 (sm_100a): GQA, causal multi-token rows,
// split-K flash-decoding and the split-K reduce.
//
// Computes, for every query row r and query head h (KV head h / group):
//     out[r,h,:] = softmax(score_scale * q[r,h,:] . K[0:ctx_r]^T) . V[0:ctx_r]
// over a paged cache `[num_blocks, block_size, num_kv_heads, head_dim]` —
// the math of CpuAttentionBackend.decode_layer (src/core/attention_backend.py:113-118)
// and of KVCacheManager.attention / paged_attention
// (src/core/memory_manager.py:175-239, src/kernels/csrc/attention.cu:16-115),
// with the scale passed in instead of fixed at 1/sqrt(D).
//
// Work decomposition: one CTA per (partition p, KV head, column chunk, sequence).
// A "column" is one (query row of the sequence, query head of the KV head's group)
// pair; a chunk holds up to 8 columns, so all query heads that share a KV head —
// and all new tokens of a multi-token step — read each KV block from HBM once.
//
// Tensor-core path (bf16/fp16 cache, head_dim 64/128/256, block 16/32):
//   * each warp owns a private ring of STAGES slots; lane 0 fetches a whole
//     KV block (K and V tiles, `block_size x head_dim`) of its KV head with
//     3-D TMA tiled loads (128-byte swizzle) completing on an mbarrier;
//   * S^T-free orientation: S[tokens x cols] = K . Q^T with mma.sync m16n8k16
//     (tokens = M, columns = N = 8), fp32 accumulate; fp32 queries are split
//     hi + lo into two 16-bit operands so scores keep ~fp32 accuracy;
//   * online softmax in the base-2 domain on the accumulator fragment;
//   * O^T[dims x cols] += V^T . P^T: V^T fragments come from ldmatrix.trans,
//     P^T from movmatrix.trans of the score fragment, P split hi + lo;
//   * warps merge their (m, l, O) in shared memory; a single-partition row is
//     written directly, otherwise (O/l, m + log2 l) goes to the workspace and
//     splitk_reduce_kernel combines partitions.
// SIMT path (fp32 cache or other shapes): same decomposition and workspace
// format with CUDA-core dot products.
#include <math.h>
#include <cmath>
#include <mutex>
#include <stdlib.h>
#include <utility>

#include <cudaTypedefs.h>

#include "decode_common.cuh"

namespace clover {


// Common CTA prologue: the token range this CTA owns.  Returns false if the
// CTA has no work.
struct CtaWork {
  int b, p, kvh, chunk, row0, nq, tok_begin, tok_end;
  const int32_t* tab;
};

// Columns whose context is empty attend to nothing: their output is zero.
__device__ __forceinline__ void zero_empty_columns(const DecodeArgs& a, const CtaWork& w, int D) {
  if (a.force_split) return;  // the gather reduce writes empty rows
  for (int idx = threadIdx.x; idx < a.cols_per_cta * D; idx += blockDim.x) {
    const int col = idx / D;
    const ColInfo ci = col_info(a, w.row0, w.nq, w.kvh, w.chunk * a.cols_per_cta + col);
    if (ci.valid && ci.limit <= 0)
      store_out(a, (int64_t)ci.qrow * a.out_stride + (int64_t)ci.qhead * D + (idx - col * D), 0.f);
  }
}

__device__ __forceinline__ bool cta_work(const DecodeArgs& a, CtaWork& w, int D) {
  // After a bounded wait gave up anywhere, later CTAs stop at once.
  if (a.status != nullptr && (*(volatile int32_t*)a.status & CLOVER_B200_DEV_TIMEOUT)) return false;
  w.b = blockIdx.z;
  w.p = blockIdx.x;
  w.kvh = blockIdx.y / a.col_chunks;
  w.chunk = blockIdx.y - w.kvh * a.col_chunks;
  w.row0 = __ldg(a.qsl + w.b);
  w.nq = __ldg(a.qsl + w.b + 1) - w.row0;
  const int c0 = w.chunk * a.cols_per_cta;
  if (w.nq <= 0 || c0 >= w.nq * a.group) return false;
  // The longest causal limit among this chunk's rows bounds the token range.
  const int j_lo = c0 / a.group;
  const int j_hi = min(w.nq - 1, (c0 + a.cols_per_cta - 1) / a.group);
  int ctx_end = 0;
  for (int j = j_lo; j <= j_hi; ++j) ctx_end = max(ctx_end, __ldg(a.ctx + w.row0 + j));
  if (ctx_end > a.max_parts * a.part_tokens) {
    if (threadIdx.x == 0 && w.p == 0 && w.kvh == 0) raise_status(a.status, CLOVER_B200_DEV_CTX_RANGE);
    ctx_end = a.max_parts * a.part_tokens;
  }
  w.tok_begin = w.p * a.part_tokens;
  if (w.tok_begin >= ctx_end) {
    if (w.p == 0) zero_empty_columns(a, w, D);
    return false;
  }
  w.tok_end = min(w.tok_begin + a.part_tokens, ctx_end);
  const int trow = a.seq_rows ? __ldg(a.seq_rows + w.b) : w.b;
  w.tab = a.tables + (int64_t)trow * a.table_stride;
  return true;
}

// Fused KV append: the CTA whose token range holds a row's new token writes
// it (this CTA's KV head) into its paged slot.  Every CTA of a sequence has
// the same column chunk when this is used, so each token has one writer and
// nothing else reads that block before this CTA does.  Returns true if
// anything was written (uniform across the CTA).
__device__ __forceinline__ bool append_new_tokens(const DecodeArgs& a, const CtaWork& w, int D) {
  const int vecs = D * a.kv_esz / 16;  // 16-byte vectors of one head row
  bool wrote = false;
  for (int j = 0; j < w.nq; ++j) {
    const int pos = __ldg(a.ctx + w.row0 + j) - 1;
    if (pos < w.tok_begin || pos >= w.tok_end) continue;
    wrote = true;
    const int bi = pos / a.block_size;
    const int blk = bi < a.table_stride ? __ldg(w.tab + bi) : -1;
    if (blk < 0 || blk >= a.num_blocks) {
      if (threadIdx.x == 0) raise_status(a.status, CLOVER_B200_DEV_BAD_BLOCK);
      continue;
    }
    const int64_t slot = (int64_t)blk * a.block_size + (pos - bi * a.block_size);
    const int64_t src = (((int64_t)(w.row0 + j)) * a.new_stride + (int64_t)w.kvh * D) * a.kv_esz / 16;
    const int64_t dst = ((slot * a.num_kv_heads + w.kvh) * D) * a.kv_esz / 16;
    const uint4* ks = static_cast<const uint4*>(a.k_new) + src;
    const uint4* vs = static_cast<const uint4*>(a.v_new) + src;
    uint4* kd = static_cast<uint4*>(const_cast<void*>(a.k_cache)) + dst;
    uint4* vd = static_cast<uint4*>(const_cast<void*>(a.v_cache)) + dst;
    for (int v = threadIdx.x; v < 2 * vecs; v += blockDim.x) {
      if (v < vecs) kd[v] = __ldg(ks + v);
      else vd[v - vecs] = __ldg(vs + (v - vecs));
    }
  }
  return wrote;
}

// Stand-alone append of every row's new token at ctx - 1 (one CTA per
// sequence, all local KV heads) for launches that cannot fuse it.
__global__ void __launch_bounds__(128)
append_at_ctx_kernel(const DecodeArgs a, int D) {
  const int b = blockIdx.x;
  const int row0 = __ldg(a.qsl + b), nq = __ldg(a.qsl + b + 1) - row0;
  const int trow = a.seq_rows ? __ldg(a.seq_rows + b) : b;
  const int32_t* tab = a.tables + (int64_t)trow * a.table_stride;
  const int esz = a.kv_esz;
  const int64_t row_elems = (int64_t)a.num_kv_heads * D;
  for (int j = 0; j < nq; ++j) {
    const int pos = __ldg(a.ctx + row0 + j) - 1;
    if (pos < 0) continue;
    const int bi = pos / a.block_size;
    const int blk = bi < a.table_stride ? __ldg(tab + bi) : -1;
    if (blk < 0 || blk >= a.num_blocks) {
      if (threadIdx.x == 0) raise_status(a.status, CLOVER_B200_DEV_BAD_BLOCK);
      continue;
    }
    const int64_t slot = (int64_t)blk * a.block_size + (pos - bi * a.block_size);
    const char* ks = static_cast<const char*>(a.k_new) + (int64_t)(row0 + j) * a.new_stride * esz;
    const char* vs = static_cast<const char*>(a.v_new) + (int64_t)(row0 + j) * a.new_stride * esz;
    char* kd = static_cast<char*>(const_cast<void*>(a.k_cache)) + slot * row_elems * esz;
    char* vd = static_cast<char*>(const_cast<void*>(a.v_cache)) + slot * row_elems * esz;
    for (int64_t e = threadIdx.x; e < row_elems * esz; e += blockDim.x) {
      kd[e] = ks[e];
      vd[e] = vs[e];
    }
  }
}

// Merge per-warp (m, l, O) partial states held in shared memory and store
// either the final output (single-partition rows) or the split-K partial.
// red_acc: [nw][cols][D+4], red_m/red_l: [nw][cols].
__device__ __forceinline__ void merge_store_rt(const DecodeArgs& a, const CtaWork& w,
                                               const float* red_acc, const float* red_m,
                                               const float* red_l, int cols, int D, int nw) {
  for (int idx = threadIdx.x; idx < cols * D; idx += blockDim.x) {
    const int col = idx / D;
    const int dim = idx - col * D;
    const ColInfo ci = col_info(a, w.row0, w.nq, w.kvh, w.chunk * a.cols_per_cta + col);
    if (!ci.valid) continue;
    if (ci.limit <= w.tok_begin) {
      if (w.p == 0 && !a.force_split)
        store_out(a, (int64_t)ci.qrow * a.out_stride + (int64_t)ci.qhead * D + dim, 0.f);
      continue;
    }
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < nw; ++k) M = fmaxf(M, red_m[k * cols + col]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int k = 0; k < nw; ++k) {
        const float e = fast_exp2(red_m[k * cols + col] - M);
        L += red_l[k * cols + col] * e;
        O += red_acc[(k * cols + col) * (D + 4) + dim] * e;
      }
    }
    const float o = L > 0.f ? O / L : 0.f;
    const int nparts = (ci.limit + a.part_tokens - 1) / a.part_tokens;
    if (nparts == 1 && !a.force_split) {
      store_out(a, (int64_t)ci.qrow * a.out_stride + (int64_t)ci.qhead * D + dim, o);
    } else {
      const int64_t base = ((int64_t)ci.qrow * a.num_q_heads + ci.qhead) * a.max_parts + w.p;
      a.part_out[base * D + dim] = o;
      if (dim == 0) a.part_lse[base] = L > 0.f ? M + fast_log2(L) : -INFINITY;
    }
  }
}


template <typename T, bool QF32, int D, int BS, int NT, bool F8, int CW>
__global__ void __launch_bounds__(kMmaThreads * CW, mma_min_ctas<D, NT, F8, CW>())
paged_decode_mma_kernel(const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmV, const DecodeArgs a) {
  using G = MmaGeom<D, BS, NT, F8, CW>;
  static_assert(CW == 1 || !F8, "column warps share 16-bit stages only");
  constexpr int NW = kMmaWarps;  // token warps (one ring each)
  constexpr int CCOLS = G::kCtaCols;
  constexpr int STAGES = G::kStages;
  constexpr int BPS = G::kBps;
  constexpr int TOK = G::kTok;
  constexpr int KK = D / 16;  // k-steps (QK) / m-tiles (PV) over head_dim
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[NW * STAGES];
  __shared__ int s_abort;

  const int lane = threadIdx.x & 31;
  // Warp (warp, cw): token warp `warp` owns a ring and issues its copies when
  // cw == 0; its CW column warps all read the ring's stages, each for its
  // own kCols columns, and agree on every stage (bar_red_or) before the slot
  // is refilled.
  const int warp = (threadIdx.x >> 5) % NW;
  const int cw = (threadIdx.x >> 5) / NW;
  // The prologue takes three dependent memory round trips before the first
  // KV copy lands: (1) the sequence's rows and table row, (2) the rows'
  // contexts and the block ids of the whole partition (ids past the context
  // are loaded but never used), (3) the first copies, with the queries
  // loaded alongside (an empty partition exits before loading them).
  //
  // (1) and (2) read only the step's metadata — rows, contexts, block
  // tables — which no kernel that triggers this launch early writes (the
  // split-K reduces write outputs and status words): they run before
  // griddepcontrol.wait, under the previous kernel's tail.  Everything the
  // preceding work may produce — queries, new K/V, cache contents,
  // workspace — is read, and every write is made, after it.
  CtaWork w;
  w.b = blockIdx.z;
  w.p = blockIdx.x;
  w.kvh = blockIdx.y / a.col_chunks;
  w.chunk = blockIdx.y - w.kvh * a.col_chunks;
  w.row0 = a.rows_identity ? w.b : __ldg(a.qsl + w.b);
  w.nq = a.rows_identity ? 1 : __ldg(a.qsl + w.b + 1) - w.row0;
  const int trow = a.seq_rows ? __ldg(a.seq_rows + w.b) : w.b;
  // after a bounded wait gave up anywhere, later CTAs stop at once
  const int stat = a.status != nullptr ? *(volatile int32_t*)a.status : 0;
  w.tab = a.tables + (int64_t)trow * a.table_stride;
  w.tok_begin = w.p * a.part_tokens;
  const int c0 = w.chunk * CCOLS;
  // (Every CTA waits before it ends, early exits too: a grid that finished
  // before its predecessor would let the next kernel's wait pass early.)
  if ((stat & CLOVER_B200_DEV_TIMEOUT) || w.nq <= 0 || c0 >= w.nq * a.group) {
    pdl_wait();
    pdl_trigger();
    return;
  }
  // lane j of warp w holds the BPS ids of the warp's j-th stage group
  // (groups w, w+NW, ... of the partition)
  const int blk0 = w.tok_begin / BS;
  const int n_grp_full = (a.part_tokens / BS + BPS - 1) / BPS;
  int my_blk[BPS];
#pragma unroll
  for (int i = 0; i < BPS; ++i) {
    const int gi = (warp + lane * NW) * BPS + i;  // block index within the partition
    const int bi = blk0 + gi;
    my_blk[i] = (cw == 0 && warp + lane * NW < n_grp_full && gi * BS < a.part_tokens &&
                 bi < a.table_stride)
                    ? __ldg(w.tab + bi)
                    : -1;
  }
  // the longest causal limit among this chunk's rows bounds the token range
  const int j_lo = c0 / a.group;
  const int j_hi = min(w.nq - 1, (c0 + CCOLS - 1) / a.group);
  int ctx_end = 0;
  for (int j = j_lo; j <= j_hi; ++j) ctx_end = max(ctx_end, __ldg(a.ctx + w.row0 + j));
  if (ctx_end > a.max_parts * a.part_tokens) {
    if (threadIdx.x == 0 && w.p == 0 && w.kvh == 0) raise_status(a.status, CLOVER_B200_DEV_CTX_RANGE);
    ctx_end = a.max_parts * a.part_tokens;
  }
  if (w.tok_begin >= ctx_end) {
    pdl_wait();
    if (w.p == 0) zero_empty_columns(a, w, D);
    pdl_trigger();
    return;
  }
  w.tok_end = min(w.tok_begin + a.part_tokens, ctx_end);
  const int n_blk = (w.tok_end - w.tok_begin + BS - 1) / BS;
  const int n_grp = (n_blk + BPS - 1) / BPS;
  const int n_mine = warp < n_grp ? (n_grp - warp + NW - 1) / NW : 0;
#pragma unroll
  for (int i = 0; i < BPS; ++i) {
    const int gi = (warp + lane * NW) * BPS + i;
    if (cw == 0 && lane < n_mine && gi < n_blk) {
      if (my_blk[i] < 0 || my_blk[i] >= a.num_blocks) {
        raise_status(a.status, CLOVER_B200_DEV_BAD_BLOCK);
        my_blk[i] = 0;  // keep the pipeline well-formed; the output is flagged invalid
      }
    } else {
      my_blk[i] = -1;
    }
  }
  pdl_wait();  // queries, new K/V, cache contents and workspace are final from here
  if (a.k_new != nullptr && append_new_tokens(a, w, D)) fence_proxy_async_global();
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));

  if (threadIdx.x == 0) {
    for (int i = 0; i < NW * STAGES; ++i) mbar_init(smem_addr(&bars[i]), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
    s_abort = 0;
  }
  __syncthreads();

  const uint32_t ring = smem_addr(smem) + warp * G::kWarpBytes;
  const uint32_t bar0 = smem_addr(&bars[warp * STAGES]);
  // fp8 cache: the fp16 staging stage (K then V) after this warp's ring
  const uint32_t conv = ring + STAGES * G::kStage;

  // Fetch this warp's k-th stage group (all lanes call: the ids are shuffled).
  auto issue = [&](int k) {
    int ids[BPS];
#pragma unroll
    for (int i = 0; i < BPS; ++i) ids[i] = __shfl_sync(0xffffffffu, my_blk[i], k);
    if (lane == 0) {
      const int s = k % STAGES;
      const uint32_t bar = bar0 + s * 8;
      const uint32_t kd = ring + s * G::kStage;
      const uint32_t vd = kd + G::kTile;
      int nb = 0;
#pragma unroll
      for (int i = 0; i < BPS; ++i) nb += ids[i] >= 0;
      mbar_arrive_expect_tx(bar, nb * 2 * BS * D * G::kEsz);
#pragma unroll
      for (int i = 0; i < BPS; ++i) {
        if (ids[i] < 0) continue;
#pragma unroll
        for (int c = 0; c < G::kChunks; ++c) {
          const uint32_t off = c * TOK * 128 + i * BS * 128;
          tma_load_3d(kd + off, &tmK, c * G::kChunkVals, w.kvh, ids[i] * BS, bar);
          tma_load_3d(vd + off, &tmV, c * G::kChunkVals, w.kvh, ids[i] * BS, bar);
        }
      }
    }
  };

  // First stages in flight, then the query fragments (MMA B operand) and the
  // causal limits of this thread's accumulator columns.
  const int npre = cw == 0 ? (n_mine < STAGES ? n_mine : STAGES) : 0;
  for (int k = 0; k < npre; ++k) issue(k);
  int issued = npre;
  int consumed = 0;
  const int wc0 = c0 + cw * G::kCols;  // this warp's first column
  const bool any_col = wc0 < w.nq * a.group;
  MmaCols<D, NT> c;
  load_cols<T, QF32, D, NT>(a, w.row0, w.nq, w.kvh, wc0, c, lane);
  c.reset();

  bool timed_out = false;

  for (int k = 0; k < n_mine; ++k) {
    const int s = k % STAGES;
    const bool landed = mbar_wait_bounded(bar0 + s * 8, (k / STAGES) & 1, a.wait_ns);
    if (CW == 1 && !landed) {
      timed_out = true;
      break;
    }
    uint32_t ks = ring + s * G::kStage;
    uint32_t vs = ks + G::kTile;
    if (F8) {
      // expand the landed fp8 stage into the fp16 staging stage, then the
      // ring slot is free for the next copy
      uint8_t* base = smem - smem_addr(smem);
      expand_fp8_tile<D, TOK>(base + ks, base + conv, lane);
      expand_fp8_tile<D, TOK>(base + vs, base + conv + TOK * D * 2, lane);
      __syncwarp();
      if (k + STAGES < n_mine) {
        issue(k + STAGES);
        ++issued;
      }
      ks = conv;
      vs = conv + TOK * D * 2;
    }
    const int tok0 = w.tok_begin + (warp + k * NW) * TOK;
    if (landed && any_col)
      mma_stage<T, QF32, D, TOK, NT>(ks, vs, smem + (vs - smem_addr(smem)), tok0,
                                     w.tok_end - tok0, a.scale_log2, c, lane);
    if (CW > 1) {
      // every column warp is done with the slot (or one gave up: all do)
      static_assert(NW == 2, "one named barrier per token warp");
      const bool fail = warp == 0 ? bar_red_or<1, 32 * CW>(!landed) : bar_red_or<2, 32 * CW>(!landed);
      if (fail) {
        timed_out = true;
        break;
      }
    } else {
      __syncwarp();
    }
    consumed = k + 1;
    if (!F8 && cw == 0 && k + STAGES < n_mine) {
      issue(k + STAGES);
      ++issued;
    }
  }

  if (timed_out) {
    // Drain this warp's copies still in flight (bounded) before giving up
    // (column warps other than the issuer have none).
    for (int k = consumed; k < issued; ++k)
      mbar_wait_bounded(bar0 + (k % STAGES) * 8, (k / STAGES) & 1, kWaitLimitNs);
    if (lane == 0) {
      raise_status(a.status, CLOVER_B200_DEV_TIMEOUT);
      atomicExch(&s_abort, 1);
    }
  }
#pragma unroll
  for (int nt = 0; nt < NT; ++nt)
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      c.l[nt][0] += __shfl_xor_sync(0xffffffffu, c.l[nt][0], off);
      c.l[nt][1] += __shfl_xor_sync(0xffffffffu, c.l[nt][1], off);
    }
  __syncthreads();  // every warp is done with its ring: reuse it for the merge
  if (s_abort) {
    pdl_trigger();
    return;
  }

  constexpr int COLS = CCOLS;
  float* red_acc = reinterpret_cast<float*>(smem);
  float* red_m = red_acc + NW * COLS * (D + 4);
  float* red_l = red_m + NW * COLS;
  {
    float* base = red_acc + (warp * COLS) * (D + 4);
    const int ca = cw * G::kCols + (lane & 3) * 2;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const int cc = nt * kMmaCols + ca;
#pragma unroll
      for (int dm = 0; dm < KK; ++dm) {
        const int d = dm * 16 + (lane >> 2);
        base[cc * (D + 4) + d] = c.acc[nt][dm][0];
        base[(cc + 1) * (D + 4) + d] = c.acc[nt][dm][1];
        base[cc * (D + 4) + d + 8] = c.acc[nt][dm][2];
        base[(cc + 1) * (D + 4) + d + 8] = c.acc[nt][dm][3];
      }
      if (lane < 4) {
        red_m[warp * COLS + cc] = c.m[nt][0];
        red_m[warp * COLS + cc + 1] = c.m[nt][1];
        red_l[warp * COLS + cc] = c.l[nt][0];
        red_l[warp * COLS + cc + 1] = c.l[nt][1];
      }
    }
  }
  __syncthreads();
  merge_store_rt(a, w, red_acc, red_m, red_l, COLS, D, NW);
  pdl_trigger();  // the split-K reduce may launch once every CTA got here
}

// ------------------------------------------------------------------ SIMT path
// Any head_dim <= 32 * EPL: lane l holds dims [l*EPL, l*EPL + EPL) of a token row.
template <typename KT, int EPL, int NC>
__global__ void __launch_bounds__(kThreads)
paged_decode_simt_kernel(const DecodeArgs a, int D) {
  constexpr int DMAX = 32 * EPL;
  __shared__ float red_acc[kNumWarps * NC * (DMAX + 4)];
  __shared__ float red_m[kNumWarps * NC], red_l[kNumWarps * NC];
  pdl_wait();
  CtaWork w;
  if (!cta_work(a, w, D)) {
    pdl_trigger();
    return;
  }
  if (a.k_new != nullptr && append_new_tokens(a, w, D)) __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int d0 = lane * EPL;

  float qv[NC][EPL];
  int lim[NC];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    const ColInfo ci = col_info(a, w.row0, w.nq, w.kvh, w.chunk * NC + c);
    lim[c] = ci.valid ? ci.limit : 0;
    const int64_t qb = (int64_t)ci.qrow * a.q_stride + (int64_t)ci.qhead * D + d0;
#pragma unroll
    for (int e = 0; e < EPL; ++e)
      qv[c][e] = (ci.valid && d0 + e < D) ? load_q(a, qb + e) * a.scale_log2 : 0.f;
  }
  float m[NC], l[NC], acc[NC][EPL];
#pragma unroll
  for (int c = 0; c < NC; ++c) {
    m[c] = -INFINITY;
    l[c] = 0.f;
#pragma unroll
    for (int e = 0; e < EPL; ++e) acc[c][e] = 0.f;
  }
  const KT* kc = static_cast<const KT*>(a.k_cache);
  const KT* vc = static_cast<const KT*>(a.v_cache);
  const int BS = a.block_size;
  for (int t = w.tok_begin + warp; t < w.tok_end; t += kNumWarps) {
    const int bi = t / BS;
    int blk = bi < a.table_stride ? __ldg(w.tab + bi) : -1;
    if (blk < 0 || blk >= a.num_blocks) {
      if (lane == 0) raise_status(a.status, CLOVER_B200_DEV_BAD_BLOCK);
      blk = 0;
    }
    const int64_t row = (((int64_t)blk * BS + (t - bi * BS)) * a.num_kv_heads + w.kvh) * D + d0;
    float kx[EPL], vx[EPL];
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const bool in = d0 + e < D;
      kx[e] = in ? load_f<KT>(kc + row + e) : 0.f;
      vx[e] = in ? load_f<KT>(vc + row + e) : 0.f;
    }
#pragma unroll
    for (int c = 0; c < NC; ++c) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) s = fmaf(qv[c][e], kx[e], s);
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      s = t < lim[c] ? s : -INFINITY;
      const float nm = fmaxf(m[c], s);
      const float u = nm == -INFINITY ? 0.f : nm;
      const float al = fast_exp2(m[c] - u);
      const float pe = fast_exp2(s - u);
      m[c] = nm;
      l[c] = l[c] * al + pe;
#pragma unroll
      for (int e = 0; e < EPL; ++e) acc[c][e] = fmaf(pe, vx[e], acc[c][e] * al);
    }
  }
#pragma unroll
  for (int c = 0; c < NC; ++c) {
#pragma unroll
    for (int e = 0; e < EPL; ++e)
      if (d0 + e < D) red_acc[(warp * NC + c) * (D + 4) + d0 + e] = acc[c][e];
    if (lane == 0) {
      red_m[warp * NC + c] = m[c];
      red_l[warp * NC + c] = l[c];
    }
  }
  __syncthreads();
  merge_store_rt(a, w, red_acc, red_m, red_l, NC, D, kNumWarps);
  pdl_trigger();
}

// ------------------------------------------------------------------ split-K reduce
// Grid (query row, head, 32-dim chunk), 4 warps.  The partitions'
// log-sum-exp weights are computed once per CTA into shared memory; warp w
// sums partitions w, w+4, ... for the chunk's 32 dims (lane = dim, coalesced
// 128-byte loads, 8 partitions in flight per warp); the four warp sums are
// combined in shared memory.
constexpr int kReduceWarps = 4;
constexpr int kReduceMaxParts = 1024;
constexpr int kReduceDims = 32;

// Combine the partitions of one (query row, head) for one dim per lane.
// Warp w takes partitions w, w+4, ..., all of whose log-sum-exp values and
// partial outputs it loads at once (one memory round trip per 64
// partitions), folding them into a running (max, sum, value); the four warps
// are merged in shared memory.  Every thread of the CTA must call it; the
// result is valid in warp 0.
constexpr int kGatherPartsPerWarp = 32;   // reduce_gather_kernel (a small grid)

// Partials of (query row r, head h): from the partition length for the
// partition kernels, as recorded by the decode for the stream kernel; 0 for an
// empty row.
__device__ __forceinline__ int partial_count(const DecodeArgs& a, int r, int h, int lim) {
  if (lim <= 0) return 0;
  const int np = a.part_count != nullptr ? __ldcg(a.part_count + (int64_t)r * a.num_q_heads + h)
                                         : (lim + a.part_tokens - 1) / a.part_tokens;
  return np < a.max_parts ? np : a.max_parts;
}

template <int PPW>
__device__ __forceinline__ float reduce_unit(const DecodeArgs& a, int r, int h, int dim, int D,
                                             int npp, float* s_m, float* s_l,
                                             float (*s_o)[kReduceDims]) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t base = ((int64_t)r * a.num_q_heads + h) * a.max_parts;
  float m = -INFINITY, l = 0.f, o = 0.f;
  for (int p0 = 0; p0 < npp; p0 += kReduceWarps * PPW) {
    float lv[PPW], ov[PPW];
#pragma unroll
    for (int i = 0; i < PPW; ++i) {
      const int p = p0 + warp + i * kReduceWarps;
      const bool ok = p < npp;
      lv[i] = ok ? __ldcg(a.part_lse + base + p) : -INFINITY;
      ov[i] = (ok && dim < D) ? __ldcg(a.part_out + (base + p) * D + dim) : 0.f;
    }
    float mm = m;
#pragma unroll
    for (int i = 0; i < PPW; ++i) mm = fmaxf(mm, lv[i]);
    const float u = mm == -INFINITY ? 0.f : mm;
    const float sc = fast_exp2(m - u);
    l *= sc;
    o *= sc;
#pragma unroll
    for (int i = 0; i < PPW; ++i) {
      const float e = fast_exp2(lv[i] - u);
      l += e;
      o = fmaf(e, ov[i], o);
    }
    m = mm;
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
  s_o[warp][lane] = o;
  __syncthreads();
  float v = 0.f;
  if (warp == 0) {
    float M = -INFINITY;
#pragma unroll
    for (int k = 0; k < kReduceWarps; ++k) M = fmaxf(M, s_m[k]);
    if (M != -INFINITY) {
      float L = 0.f, O = 0.f;
#pragma unroll
      for (int k = 0; k < kReduceWarps; ++k) {
        const float e = fast_exp2(s_m[k] - M);
        L += s_l[k] * e;
        O = fmaf(s_o[k][lane], e, O);
      }
      v = L > 0.f ? O / L : 0.f;
    }
  }
  __syncthreads();  // shared scratch is reused by the caller's next unit
  return v;
}

constexpr int kRedThreads = kReduceWarps * 32;

// One unit: (row r, head h, dims [d0, d0 + 32 EPL) of D); warp w adds
// partitions w, w + 4, ..., BATCH of them in flight.
template <int EPL, int BATCH>
__device__ __forceinline__ void reduce_rows_unit(const DecodeArgs& a, int r, int h, int d0,
                                                 int npp, int D, float* s_red,
                                                 float (*s_o)[32 * EPL]) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t base = ((int64_t)r * a.num_q_heads + h) * a.max_parts;
  // (1) max and sum of the weights 2^(lse_p - M) over the partitions
  float mx = -INFINITY;
  for (int p = tid; p < npp; p += kRedThreads) mx = fmaxf(mx, __ldcg(a.part_lse + base + p));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  if (lane == 0) s_red[warp] = mx;
  __syncthreads();
  const float M = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
  const float u = M == -INFINITY ? 0.f : M;
  float sum = 0.f;
  for (int p = tid; p < npp; p += kRedThreads) sum += fast_exp2(__ldcg(a.part_lse + base + p) - u);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
  if (lane == 0) s_red[4 + warp] = sum;
  // (2) weighted sum of the partial outputs
  float acc[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) acc[j] = 0.f;
  for (int p0 = warp; p0 < npp; p0 += kReduceWarps * BATCH) {
    float wv[BATCH], v[BATCH][EPL];
#pragma unroll
    for (int i = 0; i < BATCH; ++i) {
      const int p = p0 + i * kReduceWarps;
      const bool ok = p < npp;
      wv[i] = ok ? __ldcg(a.part_lse + base + p) : -INFINITY;
#pragma unroll
      for (int j = 0; j < EPL; ++j) {
        const int d = d0 + lane + 32 * j;
        v[i][j] = (ok && d < D) ? __ldcg(a.part_out + (base + p) * D + d) : 0.f;
      }
    }
#pragma unroll
    for (int i = 0; i < BATCH; ++i) {
      const float wi = fast_exp2(wv[i] - u);
#pragma unroll
      for (int j = 0; j < EPL; ++j) acc[j] = fmaf(wi, v[i][j], acc[j]);
    }
  }
#pragma unroll
  for (int j = 0; j < EPL; ++j) s_o[warp][lane + 32 * j] = acc[j];
  __syncthreads();
  const float L = s_red[4] + s_red[5] + s_red[6] + s_red[7];
  for (int i = tid; i < 32 * EPL; i += kRedThreads) {
    const int d = d0 + i;
    if (d >= D) continue;
    const float o = s_o[0][i] + s_o[1][i] + s_o[2][i] + s_o[3][i];
    store_out(a, (int64_t)r * a.out_stride + (int64_t)h * D + d, L > 0.f ? o / L : 0.f);
  }
  __syncthreads();  // shared scratch is reused by the next unit
}

// Split-K reduce for paged_decode / decode_step.  A unit is one (query row,
// head, 32 EPL dims); a CTA of 4 warps first screens up to 128 of its units
// at once (one round trip for their contexts or part counts) and then
// reduces only those with several partials: the CTA's threads take the
// log-sum-exp values (max, then the sum of the weights), then warp w adds
// partitions w, w + 4, ... (BATCH loads in flight per lane), and the four
// warp sums are added in shared memory.  Units the decode wrote itself (one
// partition) cost only the screening load, so a ragged batch whose rows
// mostly fit one partition launches no CTA per (row, head).  Rows with up to
// 16 partials take all dims per unit; rows with more take 32 dims per unit
// and 32 partitions per warp in flight, so a few long rows still spread over
// the SMs and need one round trip for their partials.
template <int EPL, int BATCH>
__global__ void __launch_bounds__(kRedThreads)
splitk_reduce_kernel(const DecodeArgs a, int D, int n_units) {
  __shared__ float s_red[8];
  __shared__ float s_o[kReduceWarps][32 * EPL];
  __shared__ int s_unit[kRedThreads], s_npp[kRedThreads];
  __shared__ int s_n;
  // The partition kernels' partial counts follow from the contexts alone, so
  // the first screening round runs before griddepcontrol.wait; the balanced
  // split's counts are written by the decode and are read after it.
  bool waited = false;
  auto wait_decode = [&]() {
    if (!waited) {
      pdl_wait();     // every partial of the decode kernel is written
      pdl_trigger();  // the next step's kernel may start launching (it waits too)
      waited = true;
    }
  };
  if (a.part_count != nullptr) wait_decode();
  const int tid = threadIdx.x;
  const int H = a.num_q_heads;
  const int dch = (D + 32 * EPL - 1) / (32 * EPL);  // dim chunks per (row, head)
  for (int64_t round = 0;; ++round) {
    const int64_t first = (int64_t)blockIdx.x + round * kRedThreads * gridDim.x;
    if (first >= n_units) break;
    if (tid == 0) s_n = 0;
    __syncthreads();
    const int64_t uu = first + (int64_t)tid * gridDim.x;
    if (uu < n_units) {
      const int u = (int)uu;
      const int rh = u / dch;
      const int r = rh / H, h = rh - r * H;
      const int npp = partial_count(a, r, h, __ldg(a.ctx + r));
      // Single-partition rows were written by the decode kernel, and so were
      // the empty rows of the partition kernels; the stream kernel leaves
      // those here.
      if (npp > 1 || (npp == 0 && a.part_count != nullptr)) {
        const int i = atomicAdd(&s_n, 1);
        s_unit[i] = u;
        s_npp[i] = npp;
      }
    }
    __syncthreads();
    const int n = s_n;
    if (n > 0) wait_decode();
    for (int i = 0; i < n; ++i) {
      const int u = s_unit[i];
      const int rh = u / dch, dc = u - rh * dch;
      const int r = rh / H, h = rh - r * H;
      reduce_rows_unit<EPL, BATCH>(a, r, h, dc * 32 * EPL, s_npp[i], D, s_red, s_o);
    }
    __syncthreads();  // everyone read s_n before the next round resets it
  }
  wait_decode();  // (a CTA with nothing to reduce still lets the next kernel launch)
}

static int launch_splitk_reduce(const DecodeArgs& a, int D, int n_rows, cudaStream_t s) {
  int sms = 148, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // Few (row, head) pairs with many partials each (one KV head per GPU, long
  // contexts): 32 dims per unit, one lane per dim and 32 partitions per warp
  // in flight, so the pairs spread over the SMs (one rank's share of C3 at 8
  // GPUs: 34.1 against 34.7 us for decode + reduce).  Otherwise every dim of
  // a pair per unit (C3 on one GPU: 175.2 against 178.4 us).
  const bool chunked = a.max_parts > 16 && (int64_t)n_rows * a.num_q_heads < sms;
  const int epl = chunked ? 1 : (D + 31) / 32;
  const int64_t units = (int64_t)n_rows * a.num_q_heads * ((D + 32 * epl - 1) / (32 * epl));
  if (units <= 0) return CLOVER_B200_OK;
  if (units > INT32_MAX) return set_error(CLOVER_B200_ERR_UNSUPPORTED, "splitk_reduce: too many rows");
  const int64_t cap = (int64_t)sms * 16;
  const dim3 grid((unsigned)(units < cap ? units : cap));
  const dim3 block(kRedThreads);
  const int nu = (int)units;
  cudaError_t e;
  if (chunked) {
    e = launch_pdl(splitk_reduce_kernel<1, 32>, grid, block, 0, s, a, D, nu);
  } else {
    switch (epl) {
      case 1: e = launch_pdl(splitk_reduce_kernel<1, 8>, grid, block, 0, s, a, D, nu); break;
      case 2: e = launch_pdl(splitk_reduce_kernel<2, 8>, grid, block, 0, s, a, D, nu); break;
      case 3: e = launch_pdl(splitk_reduce_kernel<3, 8>, grid, block, 0, s, a, D, nu); break;
      case 4: e = launch_pdl(splitk_reduce_kernel<4, 8>, grid, block, 0, s, a, D, nu); break;
      default: e = launch_pdl(splitk_reduce_kernel<8, 8>, grid, block, 0, s, a, D, nu); break;
    }
  }
  return check_cuda(e, "splitk_reduce launch");
}

constexpr int kGatherCtasPerSm = 4;
// (row, head) units of one warp when no pair has more partials than this,
// or when the pairs alone fill the grid's warps.
constexpr int kGatherRowsMaxParts = 16;

__device__ __forceinline__ void st_relaxed_sys_u64(uint64_t* p, uint64_t v) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys_u64(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// One (row, head) of the fused gather's reduce by one warp: lane l merges
// dims l, l + 32, ... (EPL of them) over the partials, 8 partitions' loads
// in flight, and sends each value, tagged with the epoch, to every rank.
template <int EPL>
__device__ __forceinline__ void gather_rows_unit(const DecodeArgs& a, const GatherArgs& g, int r,
                                                 int h, int npp, int D, int64_t orow,
                                                 uint32_t epoch, int lane) {
  constexpr int PB = 8;
  const int64_t base = ((int64_t)r * a.num_q_heads + h) * a.max_parts;
  float m = -INFINITY, l = 0.f, o[EPL];
#pragma unroll
  for (int j = 0; j < EPL; ++j) o[j] = 0.f;
  for (int p0 = 0; p0 < npp; p0 += PB) {
    float lv[PB], ov[PB][EPL];
#pragma unroll
    for (int i = 0; i < PB; ++i) {
      const bool ok = p0 + i < npp;
      lv[i] = ok ? __ldcg(a.part_lse + base + p0 + i) : -INFINITY;
#pragma unroll
      for (int j = 0; j < EPL; ++j) {
        const int d = lane + 32 * j;
        ov[i][j] = (ok && d < D) ? __ldcg(a.part_out + (base + p0 + i) * D + d) : 0.f;
      }
    }
    float mm = m;
#pragma unroll
    for (int i = 0; i < PB; ++i) mm = fmaxf(mm, lv[i]);
    const float u = mm == -INFINITY ? 0.f : mm;
    const float sc = fast_exp2(m - u);
    l *= sc;
#pragma unroll
    for (int j = 0; j < EPL; ++j) o[j] *= sc;
#pragma unroll
    for (int i = 0; i < PB; ++i) {
      const float e = fast_exp2(lv[i] - u);
      l += e;
#pragma unroll
      for (int j = 0; j < EPL; ++j) o[j] = fmaf(e, ov[i][j], o[j]);
    }
    m = mm;
  }
#pragma unroll
  for (int j = 0; j < EPL; ++j) {
    const int d = lane + 32 * j;
    if (d >= D) continue;
    const float v = l > 0.f ? o[j] / l : 0.f;
    const uint64_t word = ((uint64_t)epoch << 32) | (uint64_t)__float_as_uint(v);
    for (int rr = 0; rr < g.n_ranks; ++rr) st_relaxed_sys_u64(g.peer_ll[rr] + orow + d, word);
  }
}

// Split-K reduce with the output all-gather fused in.
// Phase 1: every CTA reduces its units (1 or more partitions; 0 -> zeros) and
// stores each value, tagged with the epoch, into EVERY rank's receive buffer
// over NVLink.  A unit is either (EPL = 0) a (query row, local head, 32-dim
// chunk) whose partitions the CTA's warps split — few (row, head) pairs with
// many partials each — or (EPL > 0) a whole (query row, local head) that one
// warp merges, EPL dims per lane — many pairs with few partials each.
// Phase 2: the grid's threads share out every word of the receive buffer
// (all ranks' heads of all rows), 8 loads in flight per thread, wait
// (bounded) until each carries the epoch and write it to the output
// [rows, total_q_heads, D] in place.  The grid never exceeds the co-resident
// CTA count and each CTA sends before it waits, so no CTA can wait on a CTA
// that has not started.
template <int EPL>
__global__ void __launch_bounds__(kReduceWarps * 32)
reduce_gather_kernel(const DecodeArgs a, const GatherArgs g, int D) {
  __shared__ float s_m[kReduceWarps], s_l[kReduceWarps];
  __shared__ float s_o[kReduceWarps][kReduceDims];
  __shared__ int s_last;
  // The epoch word is written only by this kernel's previous launch, which
  // completed before the decode it waits for began: read it while waiting.
  const int epoch = *(volatile int32_t*)(g.sync + kSyncEpoch) + 1;
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t half = (int64_t)(epoch & 1) * g.ll_half_words;
  const int heads = a.num_q_heads;

  // ---- phase 1: reduce and send
  if (EPL > 0) {
    for (int u = blockIdx.x * kReduceWarps + warp; u < g.units; u += gridDim.x * kReduceWarps) {
      const int h = u % heads, r = u / heads;
      const int npp = partial_count(a, r, h, __ldg(a.ctx + r));
      const int64_t orow = half + ((int64_t)r * g.total_q_heads + g.q_head_offset + h) * D;
      gather_rows_unit<(EPL > 0 ? EPL : 1)>(a, g, r, h, npp, D, orow, (uint32_t)epoch, lane);
    }
  } else {
    const int dchunks = (D + kReduceDims - 1) / kReduceDims;
    for (int u = blockIdx.x; u < g.units; u += gridDim.x) {
      const int dc = u % dchunks;
      const int h = (u / dchunks) % heads;
      const int r = u / (dchunks * heads);
      const int dim = dc * kReduceDims + lane;
      const int npp = partial_count(a, r, h, __ldg(a.ctx + r));
      const float v = reduce_unit<kGatherPartsPerWarp>(a, r, h, dim, D, npp, s_m, s_l, s_o);
      if (warp == 0 && dim < D) {
        const uint64_t word = ((uint64_t)(uint32_t)epoch << 32) | (uint64_t)__float_as_uint(v);
        const int64_t idx = half + ((int64_t)r * g.total_q_heads + g.q_head_offset + h) * D + dim;
        for (int rr = 0; rr < g.n_ranks; ++rr) st_relaxed_sys_u64(g.peer_ll[rr] + idx, word);
      }
    }
  }

  // ---- phase 2: receive every word of the buffer (all ranks' heads)
  bool timed_out = false;
  const uint64_t t0 = global_timer_ns();
  const int64_t n_words = (int64_t)g.rows * g.total_q_heads * D;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const uint64_t* rb = g.peer_ll[g.rank] + half;
  constexpr int kInFlight = 8;
  for (int64_t i0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i0 < n_words;
       i0 += kInFlight * stride) {
    uint64_t w[kInFlight];
#pragma unroll
    for (int k = 0; k < kInFlight; ++k) {
      const int64_t i = i0 + k * stride;
      w[k] = i < n_words ? ld_relaxed_sys_u64(rb + i) : 0;
    }
#pragma unroll
    for (int k = 0; k < kInFlight; ++k) {
      const int64_t i = i0 + k * stride;
      if (i >= n_words) break;
      while ((uint32_t)(w[k] >> 32) != (uint32_t)epoch && !timed_out) {
        if (global_timer_ns() - t0 > a.wait_ns) {
          timed_out = true;
          break;
        }
        w[k] = ld_relaxed_sys_u64(rb + i);
      }
      const int64_t rh = i / D;
      const int dim = (int)(i - rh * D);
      const int64_t r = rh / g.total_q_heads;
      const int head = (int)(rh - r * g.total_q_heads);
      store_out(a, r * a.out_stride + (int64_t)head * D + dim,
                timed_out ? 0.f : __uint_as_float((uint32_t)w[k]));
    }
  }
  if (timed_out) raise_status(a.status, CLOVER_B200_DEV_TIMEOUT);

  // ---- the last CTA advances this rank's epoch
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(g.sync + kSyncDone, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    g.sync[kSyncDone] = 0;
    *(volatile int32_t*)(g.sync + kSyncEpoch) = epoch;
  }
}

// ------------------------------------------------------------------ host side
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::mutex g_mu;

struct TmapEntry {
  const void* ptr;
  int dtype, head_dim, heads, block_size;
  int64_t num_blocks;
  CUtensorMap map;
  bool used;
};
static TmapEntry g_tmaps[64];
static int g_tmap_next = 0;

static int get_tmap(const void* ptr, int dtype, int D, int H, int BS, int64_t nb,
                    CUtensorMap* out) {
  std::lock_guard<std::mutex> lock(g_mu);
  for (auto& e : g_tmaps) {
    if (e.used && e.ptr == ptr && e.dtype == dtype && e.head_dim == D && e.heads == H &&
        e.block_size == BS && e.num_blocks == nb) {
      *out = e.map;
      return CLOVER_B200_OK;
    }
  }
  if (g_encode == nullptr) {
    cudaDriverEntryPointQueryResult q;
    void* fn = nullptr;
    cudaError_t err = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
    if (err != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
      return set_error(CLOVER_B200_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  CUtensorMap m;
  const cuuint64_t dims[3] = {(cuuint64_t)D, (cuuint64_t)H, (cuuint64_t)(nb * BS)};
  // 128-byte rows of the swizzle: 64 two-byte values or 128 fp8 values
  const cuuint64_t esz = dtype == CLOVER_B200_FP8_E4M3 ? 1 : 2;
  const cuuint64_t strides[2] = {(cuuint64_t)D * esz, (cuuint64_t)H * D * esz};
  const cuuint32_t box[3] = {(cuuint32_t)(128 / esz), 1, (cuuint32_t)BS};
  const cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == CLOVER_B200_BF16      ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
      : dtype == CLOVER_B200_FP8_E4M3 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                      : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  CUresult r = g_encode(&m, dt, 3, const_cast<void*>(ptr), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(CLOVER_B200_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  TmapEntry& e = g_tmaps[g_tmap_next];
  g_tmap_next = (g_tmap_next + 1) % 64;
  e = TmapEntry{ptr, dtype, D, H, BS, nb, m, true};
  *out = m;
  return CLOVER_B200_OK;
}

static bool mma_supported(int kv_dtype, int q_dtype, int D, int BS) {
  if (kv_dtype == CLOVER_B200_FP8_E4M3)  // read as fp16: fp32 or fp16 queries
    return (q_dtype == CLOVER_B200_F32 || q_dtype == CLOVER_B200_F16) && (D == 128 || D == 256) &&
           (BS == 16 || BS == 32);
  return (kv_dtype == CLOVER_B200_BF16 || kv_dtype == CLOVER_B200_F16) &&
         (q_dtype == CLOVER_B200_F32 || q_dtype == kv_dtype) && (D == 64 || D == 128 || D == 256) &&
         (BS == 16 || BS == 32);
}

static int MmaGeomBps(int BS) {
  return (CLOVER_MMA_STAGE_TOKENS > BS ? CLOVER_MMA_STAGE_TOKENS : BS) / BS;
}
// one lane per stage group and warp holds the group's block ids
static int max_mma_partition(int BS) { return 32 * kMmaWarps * MmaGeomBps(BS) * BS; }

static int choose_partition(int max_ctx, int BS, int rows_x_kvh, bool mma) {
  if (max_ctx <= 0) return BS * 4;
  if (!mma) {
    // SIMT path: 512-token partitions, finer when there are few (row, head) units
    int pt = 512;
    while (pt > 64 && (int64_t)rows_x_kvh * ((max_ctx + pt - 1) / pt) < 2 * 148 * 4) pt /= 2;
    while ((max_ctx + pt - 1) / pt > kReduceMaxParts) pt *= 2;
    return (pt + BS - 1) / BS * BS;
  }
  // Tensor-core path: the longest partition (fewest partials) whose CTA count
  // fills the resident CTA slots in near-whole waves (>= 90 % of the last
  // wave busy); contexts are assumed as long as the longest one.
  const int64_t slots = 148LL * CLOVER_MMA_MIN_CTAS;
  const int hi = max_mma_partition(BS) < 1024 ? max_mma_partition(BS) : 1024;
  const int lo = BS * kMmaWarps * MmaGeomBps(BS);
  int best = -1;
  double best_eff = 0.0;
  for (int pt = hi; pt >= lo; pt -= BS) {
    const int64_t parts = (max_ctx + pt - 1) / pt;
    if (parts > kReduceMaxParts) break;
    const int64_t ctas = (int64_t)rows_x_kvh * parts;
    const double waves = (double)ctas / (double)slots;
    const double eff = waves / std::ceil(waves);
    if (eff >= 0.9) return pt;
    if (eff > best_eff) {
      best_eff = eff;
      best = pt;
    }
  }
  if (best > 0) return best;
  int pt = lo;
  while ((max_ctx + pt - 1) / pt > kReduceMaxParts) pt *= 2;
  return pt;
}


template <typename T, bool QF32, int D, int BS, int NT, bool F8 = false, int CW = 1>
static int launch_mma(const DecodeArgs& a, const CUtensorMap& tk, const CUtensorMap& tv,
                      dim3 grid, cudaStream_t s) {
  using G = MmaGeom<D, BS, NT, F8, CW>;
  static uint64_t configured = 0;  // one bit per device ordinal
  auto kern = paged_decode_mma_kernel<T, QF32, D, BS, NT, F8, CW>;
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  if (dev >= 64 || !(configured >> dev & 1)) {
    rc = set_smem(kern, G::kSmem);
    if (rc) return rc;
    if (dev < 64) configured |= 1ull << dev;
  }
  return check_cuda(launch_pdl(kern, grid, dim3(G::kThreads), G::kSmem, s, tk, tv, a),
                    "paged_decode_mma launch");
}

template <typename T, bool QF32, int D, int NT, int CW = 1>
static int dispatch_bs(int BS, const DecodeArgs& a, const CUtensorMap& tk, const CUtensorMap& tv,
                       dim3 grid, cudaStream_t s) {
  return BS == 16 ? launch_mma<T, QF32, D, 16, NT, false, CW>(a, tk, tv, grid, s)
                  : launch_mma<T, QF32, D, 32, NT, false, CW>(a, tk, tv, grid, s);
}

// 16-column CTAs exist for head_dim 64 and 128: two column warps of one
// n-tile per token warp (CLOVER_B200_COLSPLIT=0: one warp of two n-tiles).
static bool colsplit_enabled() {
  static const bool on = [] {
    const char* e = getenv("CLOVER_B200_COLSPLIT");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename T, bool QF32>
static int dispatch_d(int D, int BS, const DecodeArgs& a, const CUtensorMap& tk,
                      const CUtensorMap& tv, dim3 grid, cudaStream_t s) {
  const bool wide = a.cols_per_cta > kMmaCols;
  const bool split = colsplit_enabled();
  switch (D) {
    case 64:
      return !wide ? dispatch_bs<T, QF32, 64, 1>(BS, a, tk, tv, grid, s)
             : split ? dispatch_bs<T, QF32, 64, 1, 2>(BS, a, tk, tv, grid, s)
                     : dispatch_bs<T, QF32, 64, 2>(BS, a, tk, tv, grid, s);
    case 128:
      return !wide ? dispatch_bs<T, QF32, 128, 1>(BS, a, tk, tv, grid, s)
             : split ? dispatch_bs<T, QF32, 128, 1, 2>(BS, a, tk, tv, grid, s)
                     : dispatch_bs<T, QF32, 128, 2>(BS, a, tk, tv, grid, s);
    default: return dispatch_bs<T, QF32, 256, 1>(BS, a, tk, tv, grid, s);
  }
}

// fp8 cache: fp16 tensor-core step on the expanded stages (head_dim 128, 8 or
// 16 columns, or 256).
template <bool QF32, int D, int NT>
static int dispatch_bs_f8(int BS, const DecodeArgs& a, const CUtensorMap& tk,
                          const CUtensorMap& tv, dim3 grid, cudaStream_t s) {
  return BS == 16 ? launch_mma<__half, QF32, D, 16, NT, true>(a, tk, tv, grid, s)
                  : launch_mma<__half, QF32, D, 32, NT, true>(a, tk, tv, grid, s);
}

template <bool QF32>
static int dispatch_d_f8(int D, int BS, const DecodeArgs& a, const CUtensorMap& tk,
                         const CUtensorMap& tv, dim3 grid, cudaStream_t s) {
  if (D == 256) return dispatch_bs_f8<QF32, 256, 1>(BS, a, tk, tv, grid, s);
  return a.cols_per_cta > kMmaCols ? dispatch_bs_f8<QF32, 128, 2>(BS, a, tk, tv, grid, s)
                                   : dispatch_bs_f8<QF32, 128, 1>(BS, a, tk, tv, grid, s);
}

template <typename KT, int EPL>
static int launch_simt_nc(int nc, int D, const DecodeArgs& a, dim3 grid, cudaStream_t s) {
  cudaError_t e;
  switch (nc) {
    case 1: e = launch_pdl(paged_decode_simt_kernel<KT, EPL, 1>, grid, dim3(kThreads), 0, s, a, D); break;
    case 2: e = launch_pdl(paged_decode_simt_kernel<KT, EPL, 2>, grid, dim3(kThreads), 0, s, a, D); break;
    case 4: e = launch_pdl(paged_decode_simt_kernel<KT, EPL, 4>, grid, dim3(kThreads), 0, s, a, D); break;
    default: e = launch_pdl(paged_decode_simt_kernel<KT, EPL, 8>, grid, dim3(kThreads), 0, s, a, D); break;
  }
  return check_cuda(e, "paged_decode_simt launch");
}

template <typename KT>
static int launch_simt(int D, int nc, const DecodeArgs& a, dim3 grid, cudaStream_t s) {
  if (D <= 32) return launch_simt_nc<KT, 1>(nc, D, a, grid, s);
  if (D <= 64) return launch_simt_nc<KT, 2>(nc, D, a, grid, s);
  if (D <= 128) return launch_simt_nc<KT, 4>(nc, D, a, grid, s);
  return launch_simt_nc<KT, 8>(nc, D, a, grid, s);
}

static int64_t align256(int64_t x) { return (x + 255) / 256 * 256; }

static int64_t split_workspace_bytes(int64_t rows, int64_t hq, int64_t D, int64_t parts) {
  if (parts < 1) parts = 1;
  return align256(rows * hq * parts * D * 4) + align256(rows * hq * parts * 4);
}

static int64_t workspace_bytes(int64_t rows, int64_t hq, int64_t D, int64_t parts) {
  return parts <= 1 ? 0 : split_workspace_bytes(rows, hq, D, parts);
}

struct DecodePlan {
  bool mma;
  bool stream;  // balanced decomposition (paged_decode_stream.cu)
  int cols_per_cta, col_chunks, part_tokens, max_parts;
  int64_t workspace_bytes;         // paged_decode / decode_step
  int64_t gather_workspace_bytes;  // decode_step_gather (every row through the workspace)
};


// The launch shape of one paged_decode call; shared by the workspace query so
// callers size the workspace for exactly what the launch will use.
static int make_plan(int n_seqs, int n_rows, int max_q, int max_ctx, int hq, int hkv, int D,
                     int BS, int kv_dtype, int q_dtype, int partition_tokens, DecodePlan* pl) {
  if (n_seqs < 0 || n_rows < 0 || hq <= 0 || hkv <= 0 || D <= 0 || BS <= 0 || max_ctx < 0 ||
      max_q < 0)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "paged_decode: bad sizes");
  if (hq % hkv != 0)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "paged_decode: num_q_heads %% num_kv_heads != 0");
  if (q_dtype != CLOVER_B200_F32 && q_dtype != CLOVER_B200_F16 && q_dtype != CLOVER_B200_BF16)
    return set_error(CLOVER_B200_ERR_UNSUPPORTED, "paged_decode: q dtype %d", q_dtype);
  if (kv_dtype != CLOVER_B200_F32 && kv_dtype != CLOVER_B200_F16 && kv_dtype != CLOVER_B200_BF16 &&
      kv_dtype != CLOVER_B200_FP8_E4M3)
    return set_error(CLOVER_B200_ERR_UNSUPPORTED, "paged_decode: kv dtype %d", kv_dtype);
  if (max_q == 0) max_q = 1;
  const int group = hq / hkv;
  pl->mma = mma_supported(kv_dtype, q_dtype, D, BS);
  if (kv_dtype == CLOVER_B200_FP8_E4M3 && !pl->mma)
    return set_error(CLOVER_B200_ERR_UNSUPPORTED,
                     "paged_decode: an fp8 cache needs head_dim 128/256, block 16/32 and fp32 or "
                     "fp16 queries (got D=%d, block %d, q dtype %d)", D, BS, q_dtype);
  if (!pl->mma && D > 256)
    return set_error(CLOVER_B200_ERR_UNSUPPORTED, "paged_decode: head_dim %d > 256", D);
  const int ncols_seq = max_q * group;
  if (pl->mma) {
    // two n-tiles when a sequence has more than 8 columns (multi-token GQA
    // rows): every KV block is then read once for up to 16 columns
    pl->cols_per_cta = ncols_seq > kMmaCols && D <= 128 ? 2 * kMmaCols : kMmaCols;
  } else {
    pl->cols_per_cta = ncols_seq >= 8 ? 8 : ncols_seq >= 4 ? 4 : ncols_seq >= 2 ? 2 : 1;
  }
  pl->col_chunks = (ncols_seq + pl->cols_per_cta - 1) / pl->cols_per_cta;
  int pt = partition_tokens;
  const bool want_stream = partition_tokens == CLOVER_B200_PARTITION_BALANCED;
  if (pt <= 0) {
    pt = choose_partition(max_ctx, BS, n_seqs * hkv * pl->col_chunks, pl->mma);
  } else {
    if (pt % BS != 0)
      return set_error(CLOVER_B200_ERR_INVALID_ARG, "paged_decode: partition_tokens %% block_size != 0");
    if (pl->mma && pt > max_mma_partition(BS))
      return set_error(CLOVER_B200_ERR_INVALID_ARG, "paged_decode: partition_tokens > %d",
                       max_mma_partition(BS));
  }
  pl->part_tokens = pt;
  pl->max_parts = max_ctx > 0 ? (max_ctx + pt - 1) / pt : 1;
  pl->stream = false;
  if (want_stream && pl->mma && kv_dtype != CLOVER_B200_FP8_E4M3 && MmaGeomBps(BS) == 1 &&
      n_seqs <= kStreamMaxSeqs) {
    // Stream decomposition: units of one block; a segment of n units spread
    // over `per`-unit worker ranges has at most min(n, workers / segments
    // per sequence + 1) parts.  Unit keys pack (segment << 16 | block).
    const int64_t units = max_ctx > 0 ? ((int64_t)max_ctx + BS - 1) / BS : 1;
    const int64_t hc = (int64_t)hkv * pl->col_chunks;
    int grid = 0;
    if (units < 65536 && (int64_t)(n_seqs + 1) * hc < 32768 &&
        (int64_t)n_seqs * hc * units < INT32_MAX &&
        stream_decode(kv_dtype, q_dtype, D, BS, pl->cols_per_cta, nullptr, nullptr, nullptr, nullptr,
                      &grid) ==
            CLOVER_B200_OK &&
        grid > 0) {
      const int64_t workers = (int64_t)grid * kMmaWarps;
      const int64_t bound = (workers + hc - 1) / hc + 1;
      pl->stream = true;
      pl->part_tokens = 0;
      pl->max_parts = (int)(bound < units ? bound : units);
      pl->workspace_bytes = split_workspace_bytes(n_rows, hq, D, pl->max_parts) +
                            align256((int64_t)n_rows * hq * 4);
      pl->gather_workspace_bytes = pl->workspace_bytes;
      return CLOVER_B200_OK;
    }
  }
  if (pl->max_parts > kReduceMaxParts)
    return set_error(CLOVER_B200_ERR_UNSUPPORTED,
                     "paged_decode: %d partitions > %d (raise partition_tokens)", pl->max_parts,
                     kReduceMaxParts);
  pl->workspace_bytes = workspace_bytes(n_rows, hq, D, pl->max_parts);
  pl->gather_workspace_bytes = split_workspace_bytes(n_rows, hq, D, pl->max_parts);
  return CLOVER_B200_OK;
}

// The sharded step (decode + the reduce with the NVLink all-gather) runs on
// fixed partitions: a request for the balanced split becomes the library's
// fixed-partition choice there.
static int gather_partition(int partition_tokens) {
  return partition_tokens == CLOVER_B200_PARTITION_BALANCED ? 0 : partition_tokens;
}

}  // namespace clover

using namespace clover;

extern "C" int clover_b200_decode_partition_tokens(
    int32_t n_seqs, int32_t n_query_rows, int32_t max_queries_per_seq, int32_t max_ctx_len,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    int32_t kv_dtype, int32_t q_dtype, int32_t partition_tokens) {
  DecodePlan pl;
  const int rc = make_plan(n_seqs, n_query_rows, max_queries_per_seq, max_ctx_len, num_q_heads,
                           num_kv_heads, head_dim, block_size, kv_dtype, q_dtype,
                           partition_tokens, &pl);
  return rc ? rc : pl.part_tokens;
}

extern "C" int64_t clover_b200_decode_workspace_bytes(
    int32_t n_seqs, int32_t n_query_rows, int32_t max_queries_per_seq, int32_t max_ctx_len,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    int32_t kv_dtype, int32_t q_dtype, int32_t partition_tokens) {
  DecodePlan pl;
  if (make_plan(n_seqs, n_query_rows, max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads,
                head_dim, block_size, kv_dtype, q_dtype, partition_tokens, &pl) != CLOVER_B200_OK)
    return -1;
  return pl.workspace_bytes;
}

// Shared body of paged_decode (k_new == nullptr) and decode_step (fused or
// preceding KV append of every row's new token).
static int decode_impl(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, int32_t q_dtype,
    const void* k_cache, const void* v_cache, int32_t kv_dtype, int64_t num_blocks,
    int32_t block_size, const void* k_new, const void* v_new, int64_t new_token_stride,
    const int32_t* block_tables, int32_t table_stride,
    const int32_t* seq_rows, const int32_t* query_start_loc, const int32_t* ctx_lens,
    int32_t n_seqs, int32_t n_query_rows, int32_t max_queries_per_seq, int32_t max_ctx_len,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, float score_scale,
    int32_t partition_tokens, void* workspace, int64_t workspace_bytes_, int32_t* dev_status,
    void* stream, const GatherArgs* gather, int32_t out_dtype) {
  if (out_dtype != CLOVER_B200_F32 && out_dtype != CLOVER_B200_F16 && out_dtype != CLOVER_B200_BF16)
    return set_error(CLOVER_B200_ERR_UNSUPPORTED, "paged_decode: out dtype %d", out_dtype);
  if (table_stride <= 0 || num_blocks <= 0)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "paged_decode: bad sizes");
  DecodePlan pl;
  int rc = make_plan(n_seqs, n_query_rows, max_queries_per_seq, max_ctx_len, num_q_heads,
                     num_kv_heads, head_dim, block_size, kv_dtype, q_dtype, partition_tokens, &pl);
  if (rc) return rc;
  if (n_seqs == 0 || n_query_rows == 0) return CLOVER_B200_OK;
  if ((!out && !gather) || !q || !k_cache || !v_cache || !block_tables || !query_start_loc ||
      !ctx_lens)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "paged_decode: null pointer");
  if (q_row_stride < (int64_t)num_q_heads * head_dim ||
      (!gather && out_row_stride < (int64_t)num_q_heads * head_dim))
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "paged_decode: row stride < heads*head_dim");
  if (n_seqs > 65535 || (int64_t)num_kv_heads * pl.col_chunks > 65535)
    return set_error(CLOVER_B200_ERR_UNSUPPORTED, "paged_decode: grid too large");
  if (pl.mma) {
    if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15))
      return set_error(CLOVER_B200_ERR_INVALID_ARG, "paged_decode: cache not 16-byte aligned");
    if (num_blocks * (int64_t)block_size > INT32_MAX)
      return set_error(CLOVER_B200_ERR_UNSUPPORTED, "paged_decode: cache exceeds 2^31 slots");
  }
  const int64_t need = gather ? pl.gather_workspace_bytes : pl.workspace_bytes;
  if (need > 0 && (workspace == nullptr || workspace_bytes_ < need))
    return set_error(CLOVER_B200_ERR_WORKSPACE, "paged_decode: workspace needs %lld bytes",
                     (long long)need);
  const int group = num_q_heads / num_kv_heads;
  const int pt = pl.part_tokens;
  const int max_parts = pl.max_parts;
  const int cols_per_cta = pl.cols_per_cta;
  const int col_chunks = pl.col_chunks;
  const bool mma = pl.mma;

  DecodeArgs a;
  a.out = out;
  a.out_stride = out_row_stride;
  a.q = q;
  a.q_stride = q_row_stride;
  a.q_dtype = q_dtype;
  a.out_dtype = out_dtype;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.tables = block_tables;
  a.table_stride = table_stride;
  a.seq_rows = seq_rows;
  a.qsl = query_start_loc;
  a.ctx = ctx_lens;
  a.num_q_heads = num_q_heads;
  a.num_kv_heads = num_kv_heads;
  a.group = group;
  a.block_size = block_size;
  a.num_blocks = num_blocks;
  a.scale_log2 = score_scale * 1.4426950408889634f;
  a.part_tokens = pt;
  a.max_parts = max_parts;
  a.cols_per_cta = cols_per_cta;
  a.col_chunks = col_chunks;
  a.part_out = need > 0 ? static_cast<float*>(workspace) : nullptr;
  a.part_lse = need > 0 ? reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                                   align256((int64_t)n_query_rows * num_q_heads *
                                                            max_parts * head_dim * 4))
                        : nullptr;
  a.status = dev_status;
  a.k_new = nullptr;
  a.v_new = nullptr;
  a.new_stride = new_token_stride;
  a.kv_esz = kv_dtype == CLOVER_B200_F32 ? 4 : (kv_dtype == CLOVER_B200_FP8_E4M3 ? 1 : 2);
  a.force_split = gather != nullptr;
  a.n_seqs = n_seqs;
  a.max_ctx = max_ctx_len;
  a.max_q = max_queries_per_seq > 0 ? max_queries_per_seq : 1;
  a.rows_identity = a.max_q == 1 && n_query_rows == n_seqs;
  a.min_units = kStreamMinUnits;
  a.part_count = nullptr;
  a.wait_ns = wait_limit_ns();
  if (pl.stream) {
    // Stream workspace: partials, their log-sum-exp, then the part counts.
    a.part_tokens = block_size;
    a.part_out = static_cast<float*>(workspace);
    a.part_lse = reinterpret_cast<float*>(static_cast<char*>(workspace) +
                                          align256((int64_t)n_query_rows * num_q_heads *
                                                   max_parts * head_dim * 4));
    a.part_count = reinterpret_cast<int32_t*>(
        static_cast<char*>(workspace) +
        split_workspace_bytes(n_query_rows, num_q_heads, head_dim, max_parts));
  }

  cudaStream_t s = (cudaStream_t)stream;
  if (k_new != nullptr) {
    if (!v_new || new_token_stride < (int64_t)num_kv_heads * head_dim)
      return set_error(CLOVER_B200_ERR_INVALID_ARG, "decode_step: bad new K/V");
    a.k_new = k_new;
    a.v_new = v_new;
    const bool fusable = col_chunks == 1 && (head_dim * a.kv_esz) % 16 == 0 &&
                         (new_token_stride * a.kv_esz) % 16 == 0 &&
                         !(reinterpret_cast<uintptr_t>(k_new) & 15) &&
                         !(reinterpret_cast<uintptr_t>(v_new) & 15) &&
                         !(reinterpret_cast<uintptr_t>(k_cache) & 15) &&
                         !(reinterpret_cast<uintptr_t>(v_cache) & 15);
    if (!fusable) {
      // Several column chunks would read a new token's block before its one
      // writer wrote it: append first in a kernel of its own.
      append_at_ctx_kernel<<<n_seqs, 128, 0, s>>>(a, head_dim);
      rc = check_cuda(cudaGetLastError(), "append_at_ctx launch");
      if (rc) return rc;
      a.k_new = nullptr;
      a.v_new = nullptr;
    }
  }
  const dim3 grid(max_parts, num_kv_heads * col_chunks, n_seqs);
  if (pl.stream) {
    CUtensorMap tk, tv;
    rc = get_tmap(k_cache, kv_dtype, head_dim, num_kv_heads, block_size, num_blocks, &tk);
    if (rc) return rc;
    rc = get_tmap(v_cache, kv_dtype, head_dim, num_kv_heads, block_size, num_blocks, &tv);
    if (rc) return rc;
    rc = stream_decode(kv_dtype, q_dtype, head_dim, block_size, cols_per_cta, &a, &tk, &tv, s,
                       nullptr);
  } else if (mma) {
    CUtensorMap tk, tv;
    rc = get_tmap(k_cache, kv_dtype, head_dim, num_kv_heads, block_size, num_blocks, &tk);
    if (rc) return rc;
    rc = get_tmap(v_cache, kv_dtype, head_dim, num_kv_heads, block_size, num_blocks, &tv);
    if (rc) return rc;
    if (kv_dtype == CLOVER_B200_FP8_E4M3) {
      rc = q_dtype == CLOVER_B200_F32
               ? dispatch_d_f8<true>(head_dim, block_size, a, tk, tv, grid, s)
               : dispatch_d_f8<false>(head_dim, block_size, a, tk, tv, grid, s);
    } else if (kv_dtype == CLOVER_B200_BF16) {
      rc = q_dtype == CLOVER_B200_F32
               ? dispatch_d<__nv_bfloat16, true>(head_dim, block_size, a, tk, tv, grid, s)
               : dispatch_d<__nv_bfloat16, false>(head_dim, block_size, a, tk, tv, grid, s);
    } else {
      rc = q_dtype == CLOVER_B200_F32
               ? dispatch_d<__half, true>(head_dim, block_size, a, tk, tv, grid, s)
               : dispatch_d<__half, false>(head_dim, block_size, a, tk, tv, grid, s);
    }
  } else {
    switch (kv_dtype) {
      case CLOVER_B200_F32: rc = launch_simt<float>(head_dim, cols_per_cta, a, grid, s); break;
      case CLOVER_B200_F16: rc = launch_simt<__half>(head_dim, cols_per_cta, a, grid, s); break;
      default: rc = launch_simt<__nv_bfloat16>(head_dim, cols_per_cta, a, grid, s); break;
    }
  }
  if (rc) return rc;
  if (gather != nullptr) {
    GatherArgs g = *gather;
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    // Many (row, head) pairs, or few partials each (ragged and multi-token
    // batches): a warp per pair.  Few pairs with many partials each (long
    // contexts over short partitions): 32-dim units whose partitions the
    // CTA's warps split.
    const int64_t pairs = (int64_t)n_query_rows * num_q_heads;
    const bool rows = max_parts <= kGatherRowsMaxParts ||
                      pairs >= (int64_t)sms * kGatherCtasPerSm * kReduceWarps;
    const int64_t units = rows ? pairs : pairs * ((head_dim + kReduceDims - 1) / kReduceDims);
    if (units > INT32_MAX) return set_error(CLOVER_B200_ERR_UNSUPPORTED, "reduce_gather: too many rows");
    g.units = (int)units;
    g.rows = n_query_rows;
    const int epl = (head_dim + 31) / 32;
    auto kern = !rows ? reduce_gather_kernel<0>
                : epl <= 1 ? reduce_gather_kernel<1>
                : epl <= 2 ? reduce_gather_kernel<2>
                : epl <= 4 ? reduce_gather_kernel<4>
                           : reduce_gather_kernel<8>;
    // Every CTA waits for words that any CTA of any rank sends: the whole
    // grid must be resident at once (at most kGatherCtasPerSm per SM, and
    // no more than the kernel's registers allow).
    int per_sm = 0;
    rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kReduceWarps * 32, 0),
                    "reduce_gather occupancy");
    if (rc) return rc;
    if (per_sm <= 0) return set_error(CLOVER_B200_ERR_UNSUPPORTED, "reduce_gather: no resident CTA");
    const int64_t cap = (int64_t)sms * (per_sm < kGatherCtasPerSm ? per_sm : kGatherCtasPerSm);
    const int64_t want = rows ? (units + kReduceWarps - 1) / kReduceWarps : units;
    const int grid = (int)(want < cap ? (want > 0 ? want : 1) : cap);
    return check_cuda(launch_pdl(kern, dim3(grid), dim3(kReduceWarps * 32), 0, s, a, g, head_dim),
                      "reduce_gather launch");
  }
  if (max_parts > 1 || pl.stream) {
    // Rows with several partitions are combined here; single-partition rows
    // were written by the decode kernel and return at once (the stream
    // kernel also leaves the empty rows' zeros to this kernel).
    rc = launch_splitk_reduce(a, head_dim, n_query_rows, s);
  }
  return rc;
}

extern "C" int clover_b200_paged_decode(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, int32_t q_dtype,
    const void* k_cache, const void* v_cache, int32_t kv_dtype, int64_t num_blocks,
    int32_t block_size, const int32_t* block_tables, int32_t table_stride,
    const int32_t* seq_rows, const int32_t* query_start_loc, const int32_t* ctx_lens,
    int32_t n_seqs, int32_t n_query_rows, int32_t max_queries_per_seq, int32_t max_ctx_len,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, float score_scale,
    int32_t partition_tokens, void* workspace, int64_t workspace_bytes_, int32_t* dev_status,
    void* stream) {
  return decode_impl(out, out_row_stride, q, q_row_stride, q_dtype, k_cache, v_cache, kv_dtype,
                     num_blocks, block_size, nullptr, nullptr, 0, block_tables, table_stride,
                     seq_rows, query_start_loc, ctx_lens, n_seqs, n_query_rows,
                     max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads, head_dim,
                     score_scale, partition_tokens, workspace, workspace_bytes_, dev_status, stream,
                     nullptr, q_dtype);
}

extern "C" int clover_b200_decode_step(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, int32_t q_dtype,
    void* k_cache, void* v_cache, int32_t kv_dtype, int64_t num_blocks, int32_t block_size,
    const void* k_new, const void* v_new, int64_t new_token_stride,
    const int32_t* block_tables, int32_t table_stride, const int32_t* seq_rows,
    const int32_t* query_start_loc, const int32_t* ctx_lens, int32_t n_seqs,
    int32_t n_query_rows, int32_t max_queries_per_seq, int32_t max_ctx_len, int32_t num_q_heads,
    int32_t num_kv_heads, int32_t head_dim, float score_scale, int32_t partition_tokens,
    void* workspace, int64_t workspace_bytes_, int32_t* dev_status, void* stream) {
  if (!k_new || !v_new)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "decode_step: null new K/V");
  return decode_impl(out, out_row_stride, q, q_row_stride, q_dtype, k_cache, v_cache, kv_dtype,
                     num_blocks, block_size, k_new, v_new, new_token_stride, block_tables,
                     table_stride, seq_rows, query_start_loc, ctx_lens, n_seqs, n_query_rows,
                     max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads, head_dim,
                     score_scale, partition_tokens, workspace, workspace_bytes_, dev_status, stream,
                     nullptr, q_dtype);
}

extern "C" int64_t clover_b200_decode_gather_workspace_bytes(
    int32_t n_seqs, int32_t n_query_rows, int32_t max_queries_per_seq, int32_t max_ctx_len,
    int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim, int32_t block_size,
    int32_t kv_dtype, int32_t q_dtype, int32_t partition_tokens) {
  DecodePlan pl;
  if (make_plan(n_seqs, n_query_rows, max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads,
                head_dim, block_size, kv_dtype, q_dtype, gather_partition(partition_tokens),
                &pl) != CLOVER_B200_OK)
    return -1;
  return pl.gather_workspace_bytes;
}

extern "C" int64_t clover_b200_gather_sync_bytes(void) { return (int64_t)kSyncInts * 4; }

static int step_gather_impl(
    void* out, int64_t out_row_stride, int32_t out_dtype, const void* q, int64_t q_row_stride,
    int32_t q_dtype, void* k_cache, void* v_cache, int32_t kv_dtype, int64_t num_blocks,
    int32_t block_size, const void* k_new, const void* v_new, int64_t new_token_stride,
    const int32_t* block_tables, int32_t table_stride, const int32_t* seq_rows,
    const int32_t* query_start_loc, const int32_t* ctx_lens, int32_t n_seqs, int32_t n_query_rows,
    int32_t max_queries_per_seq, int32_t max_ctx_len, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, float score_scale, int32_t partition_tokens, void* const* peer_recv,
    int32_t* sync, int32_t n_ranks, int32_t rank, int64_t recv_half_words, void* workspace,
    int64_t workspace_bytes_, int32_t* dev_status, void* stream) {
  const int64_t total_q_heads = (int64_t)num_q_heads * n_ranks;
  if (!out || !peer_recv || !sync || n_ranks <= 0 || rank < 0 || rank >= n_ranks ||
      out_row_stride < total_q_heads * head_dim ||
      recv_half_words < (int64_t)n_query_rows * total_q_heads * head_dim)
    return set_error(CLOVER_B200_ERR_INVALID_ARG, "decode_step_gather: bad gather arguments");
  GatherArgs g;
  g.peer_ll = reinterpret_cast<uint64_t* const*>(peer_recv);
  g.sync = sync;
  g.n_ranks = n_ranks;
  g.rank = rank;
  g.q_head_offset = rank * num_q_heads;
  g.total_q_heads = (int32_t)total_q_heads;
  g.ll_half_words = recv_half_words;
  g.units = 0;
  g.rows = 0;
  return decode_impl(out, out_row_stride, q, q_row_stride, q_dtype, k_cache, v_cache, kv_dtype,
                     num_blocks, block_size, k_new, v_new, new_token_stride, block_tables,
                     table_stride, seq_rows, query_start_loc, ctx_lens, n_seqs, n_query_rows,
                     max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads, head_dim,
                     score_scale, gather_partition(partition_tokens), workspace, workspace_bytes_,
                     dev_status, stream, &g, out_dtype);
}

extern "C" int clover_b200_decode_step_gather(
    void* out, int64_t out_row_stride, const void* q, int64_t q_row_stride, int32_t q_dtype,
    void* k_cache, void* v_cache, int32_t kv_dtype, int64_t num_blocks, int32_t block_size,
    const void* k_new, const void* v_new, int64_t new_token_stride, const int32_t* block_tables,
    int32_t table_stride, const int32_t* seq_rows, const int32_t* query_start_loc,
    const int32_t* ctx_lens, int32_t n_seqs, int32_t n_query_rows, int32_t max_queries_per_seq,
    int32_t max_ctx_len, int32_t num_q_heads, int32_t num_kv_heads, int32_t head_dim,
    float score_scale, int32_t partition_tokens, void* const* peer_recv, int32_t* sync,
    int32_t n_ranks, int32_t rank, int64_t recv_half_words, void* workspace,
    int64_t workspace_bytes_, int32_t* dev_status, void* stream) {
  return step_gather_impl(out, out_row_stride, q_dtype, q, q_row_stride, q_dtype, k_cache, v_cache,
                          kv_dtype, num_blocks, block_size, k_new, v_new, new_token_stride,
                          block_tables, table_stride, seq_rows, query_start_loc, ctx_lens, n_seqs,
                          n_query_rows, max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads,
                          head_dim, score_scale, partition_tokens, peer_recv, sync, n_ranks, rank,
                          recv_half_words, workspace, workspace_bytes_, dev_status, stream);
}

extern "C" int clover_b200_decode_step_gather_into(
    void* out, int64_t out_row_stride, int32_t out_dtype, const void* q, int64_t q_row_stride,
    int32_t q_dtype, void* k_cache, void* v_cache, int32_t kv_dtype, int64_t num_blocks,
    int32_t block_size, const void* k_new, const void* v_new, int64_t new_token_stride,
    const int32_t* block_tables, int32_t table_stride, const int32_t* seq_rows,
    const int32_t* query_start_loc, const int32_t* ctx_lens, int32_t n_seqs, int32_t n_query_rows,
    int32_t max_queries_per_seq, int32_t max_ctx_len, int32_t num_q_heads, int32_t num_kv_heads,
    int32_t head_dim, float score_scale, int32_t partition_tokens, void* const* peer_recv,
    int32_t* sync, int32_t n_ranks, int32_t rank, int64_t recv_half_words, void* workspace,
    int64_t workspace_bytes_, int32_t* dev_status, void* stream) {
  return step_gather_impl(out, out_row_stride, out_dtype, q, q_row_stride, q_dtype, k_cache,
                          v_cache, kv_dtype, num_blocks, block_size, k_new, v_new,
                          new_token_stride, block_tables, table_stride, seq_rows, query_start_loc,
                          ctx_lens, n_seqs, n_query_rows, max_queries_per_seq, max_ctx_len,
                          num_q_heads, num_kv_heads, head_dim, score_scale, partition_tokens,
                          peer_recv, sync, n_ranks, rank, recv_half_words, workspace,
                          workspace_bytes_, dev_status, stream);
}
