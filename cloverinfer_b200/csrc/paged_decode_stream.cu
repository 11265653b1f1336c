// Balanced ("stream") paged decode for B200 (sm_100a): the tensor-core decode
// with the work of the whole step split evenly over every resident warp.
//
// Same math and outputs as paged_decode_mma_kernel (the attention of
// CpuAttentionBackend.decode_layer, src/core/attention_backend.py:113-118, and
// of KVCacheManager.attention / paged_attention,
// src/core/memory_manager.py:175-239, src/kernels/csrc/attention.cu:16-115),
// with a different decomposition:
//
//   * a unit is one KV block (TOK = block_size tokens) of one segment; a
//     segment is (sequence, KV head, column chunk) and holds
//     ceil(ctx / TOK) units, ctx = the sequence's longest row context;
//   * units are numbered sequence-major, then segment, then block; the grid
//     is the resident CTA count and every warp is one worker that owns the
//     contiguous range [w * per, (w + 1) * per) with per = ceil(U / workers):
//     ragged batches cost no empty CTAs and every worker streams the same
//     number of KV bytes;
//   * each warp runs one TMA ring over its whole range — the ring crosses
//     block, head and sequence boundaries without draining, so the
//     table-load / first-copy latency is paid once per worker, not once per
//     partition;
//   * a worker that covers a whole segment writes the output directly;
//     otherwise it writes its normalised partial (O / l, m + log2 l) as part
//     `w - first worker of the segment`, and the worker that owns the
//     segment's first unit records the number of parts, which the split-K
//     reduce reads (DecodeArgs::part_count).
//
// Block ids are fetched 32 units ahead per warp: lane j resolves unit
// (32 t + j) to its (sequence, segment, block) through a 32-sequence window
// held one sequence per lane, and the table load stays in flight until the
// ring reaches that batch.
#include <cudaTypedefs.h>

#include "decode_common.cuh"

namespace clover {

constexpr int kStreamEntries = 64;  // two 32-unit batches per warp

struct StreamEntry {
  int32_t blk;   // KV block id; -1: invalid (block 0 is fetched, status flagged)
  int32_t key;   // (segment << 16) | unit index within the segment
  int32_t n;     // units of the segment
  int32_t seg0;  // flat index of the segment's first unit
};

// Units of each of sequence b's segments: its last row's context (the
// longest, rows being in causal order), rounded up to whole blocks.
template <int TOK>
__device__ __forceinline__ int seq_units(const DecodeArgs& a, int b) {
  const int r0 = __ldg(a.qsl + b), r1 = __ldg(a.qsl + b + 1);
  if (r1 <= r0) return 0;
  int c = __ldg(a.ctx + r1 - 1);
  if (c > a.max_ctx) {
    raise_status(a.status, CLOVER_B200_DEV_CTX_RANGE);
    c = a.max_ctx;
  }
  return c > 0 ? (c + TOK - 1) / TOK : 0;
}

// 32 consecutive sequences, one per lane: the flat index of the sequence's
// first unit, its units per segment and its table row.
struct SeqWindow {
  int wb;   // first sequence of the window
  int S, n, trow;
  int end;  // flat index just past the window (uniform)
};

template <int TOK>
__device__ __forceinline__ void load_window(const DecodeArgs& a, SeqWindow& w, int wb, int p0,
                                            int hc, int lane) {
  const int b = wb + lane;
  int n = 0, trow = 0;
  if (b < a.n_seqs) {
    n = seq_units<TOK>(a, b);
    trow = a.seq_rows ? __ldg(a.seq_rows + b) : b;
  }
  int incl = n;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  w.wb = wb;
  w.n = n;
  w.trow = trow;
  w.S = (p0 + incl - n) * hc;
  w.end = __shfl_sync(0xffffffffu, (p0 + incl) * hc, 31);
}

// Resolve this lane's unit of batch t (local units 32 t + lane) and store its
// entry; the block-id load is left in flight in `pend` (committed later).
template <int TOK>
__device__ __forceinline__ void fill_batch(const DecodeArgs& a, SeqWindow& w, StreamEntry* ent,
                                           int t, int u0, int u1, int hc, int lane, int& pend) {
  const int u = u0 + t * 32 + lane;
  const bool valid = u < u1;
  bool done = !valid;
  int64_t tab_idx = -1;
  int key = 0, n = 0, seg0 = 1;
  // Every unit below U lies in some sequence, so the window reaches it within
  // n_seqs / 32 slides; the bound only guards against inconsistent inputs.
  for (int slides = 0;; ++slides) {
    const bool here = !done && u < w.end;
    // largest window lane i with S_i <= u (S is non-decreasing over lanes)
    int i = 0;
#pragma unroll
    for (int step = 16; step >= 1; step >>= 1) {
      const int s = __shfl_sync(0xffffffffu, w.S, i + step);
      if (here && s <= u) i += step;
    }
    const int ni = __shfl_sync(0xffffffffu, w.n, i);
    const int si = __shfl_sync(0xffffffffu, w.S, i);
    const int ti = __shfl_sync(0xffffffffu, w.trow, i);
    if (here) {
      if (ni > 0 && u >= si) {
        const int off = u - si;
        const int h = off / ni;
        const int jj = off - h * ni;
        key = (((w.wb + i) * hc + h) << 16) | jj;
        n = ni;
        seg0 = si + h * ni;
        tab_idx = jj < a.table_stride ? (int64_t)ti * a.table_stride + jj : -1;
      } else {
        raise_status(a.status, CLOVER_B200_DEV_CTX_RANGE);  // inconsistent inputs
      }
      done = true;
    }
    if (__all_sync(0xffffffffu, done)) break;
    if (slides > (a.n_seqs >> 5) + 1) {
      if (!done) raise_status(a.status, CLOVER_B200_DEV_CTX_RANGE);
      break;  // unresolved lanes keep key 0 (sequence 0, block 0) and block id -1
    }
    load_window<TOK>(a, w, w.wb + 32, w.end / hc, hc, lane);  // slide to the next 32
  }
  StreamEntry& e = ent[(t & 1) * 32 + lane];
  if (valid) {
    e.key = key;
    e.n = n;
    e.seg0 = seg0;
  }
  pend = (valid && tab_idx >= 0) ? __ldg(a.tables + tab_idx) : -1;
}

__device__ __forceinline__ void commit_batch(const DecodeArgs& a, StreamEntry* ent, int t,
                                             int u0, int u1, int lane, int pend) {
  if (u0 + t * 32 + lane < u1) {
    int id = pend;
    if (id < 0 || id >= a.num_blocks) {
      raise_status(a.status, CLOVER_B200_DEV_BAD_BLOCK);
      id = -1;
    }
    ent[(t & 1) * 32 + lane].blk = id;
  }
  __syncwarp();
}

// Fused KV append for one unit: the rows of sequence b whose new token falls
// in this block are written (KV head kvh) before the block is fetched.  Only
// the worker that owns the unit reads it for this head, so the token has one
// writer and no earlier reader.
template <int D, int BS>
__device__ __forceinline__ void append_unit(const DecodeArgs& a, int b, int kvh, int blk, int jj,
                                            int lane) {
  constexpr int kVecs = D * 2 / 16;  // 16-byte vectors of one head row (2-byte types)
  const int row0 = __ldg(a.qsl + b), nq = __ldg(a.qsl + b + 1) - row0;
  for (int j = 0; j < nq; ++j) {
    const int pos = __ldg(a.ctx + row0 + j) - 1;
    if (pos < 0 || pos / BS != jj) continue;
    const int64_t slot = (int64_t)blk * BS + (pos - jj * BS);
    const int64_t src = (((int64_t)(row0 + j)) * a.new_stride + (int64_t)kvh * D) * 2 / 16;
    const int64_t dst = ((slot * a.num_kv_heads + kvh) * D) * 2 / 16;
    const uint4* ks = static_cast<const uint4*>(a.k_new) + src;
    const uint4* vs = static_cast<const uint4*>(a.v_new) + src;
    uint4* kd = static_cast<uint4*>(const_cast<void*>(a.k_cache)) + dst;
    uint4* vd = static_cast<uint4*>(const_cast<void*>(a.v_cache)) + dst;
    for (int v = lane; v < 2 * kVecs; v += 32) {
      if (v < kVecs) kd[v] = __ldg(ks + v);
      else vd[v - kVecs] = __ldg(vs + (v - kVecs));
    }
  }
  fence_proxy_async_global();
  __syncwarp();
}

template <typename T, bool QF32, int D, int BS, int NT>
__global__ void __launch_bounds__(kMmaThreads, mma_min_ctas<D, NT>())
paged_decode_stream_kernel(const __grid_constant__ CUtensorMap tmK,
                           const __grid_constant__ CUtensorMap tmV, const DecodeArgs a) {
  using G = MmaGeom<D, BS, NT>;
  static_assert(G::kBps == 1, "one KV block per stage");
  constexpr int NW = kMmaWarps;
  constexpr int NTH = kMmaThreads;
  constexpr int STAGES = G::kStages;
  constexpr int TOK = G::kTok;
  constexpr int KK = D / 16;
  constexpr int E = kStreamSeqsPerThread;
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t bars[NW * STAGES];
  __shared__ int s_wsum[E][NW];
  __shared__ int s_start[NW][2];

  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  // The plan and the first batches of block ids read only the step's
  // metadata (rows, contexts, block tables), which no kernel that triggers
  // this launch early writes: they run before griddepcontrol.wait, under the
  // previous kernel's tail.  Queries, new K/V, cache contents and workspace
  // are read, and every write made, after it.
  // After a bounded wait gave up anywhere, later launches stop at once.
  // (Every CTA waits before it ends, early exits too: a grid that finished
  // before its predecessor would let the next kernel's wait pass early.)
  if (a.status != nullptr && (*(volatile int32_t*)a.status & CLOVER_B200_DEV_TIMEOUT)) {
    pdl_wait();
    pdl_trigger();
    return;
  }

  // ---- plan: units per sequence, their prefix sums and each warp's range
  const int HC = a.num_kv_heads * a.col_chunks;
  int nreg[E], pre[E];
#pragma unroll
  for (int it = 0; it < E; ++it) {
    const int b = it * NTH + threadIdx.x;
    nreg[it] = b < a.n_seqs ? seq_units<TOK>(a, b) : 0;
    // the warps' windows read the table rows next: bring them into L1 now
    if (b < a.n_seqs && a.seq_rows != nullptr)
      asm volatile("prefetch.global.L1 [%0];" ::"l"(a.seq_rows + b));
  }
#pragma unroll
  for (int it = 0; it < E; ++it) {
    int x = nreg[it];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, x, off);
      if (lane >= off) x += y;
    }
    pre[it] = x - nreg[it];
    if (lane == 31) s_wsum[it][warp] = x;
  }
  if (threadIdx.x < NW) s_start[threadIdx.x][0] = -1;
  __syncthreads();
  int run = 0;
#pragma unroll
  for (int it = 0; it < E; ++it) {
    int before = run;
#pragma unroll
    for (int w2 = 0; w2 < NW; ++w2) {
      const int v = s_wsum[it][w2];
      if (w2 < warp) before += v;
      run += v;
    }
    pre[it] += before;
  }
  const int U = run * HC;
  const int workers = gridDim.x * NW;
  int weff = (U + a.min_units - 1) / a.min_units;
  weff = weff < 1 ? 1 : (weff > workers ? workers : weff);
  const int per = U > 0 ? (U + weff - 1) / weff : 1;
#pragma unroll
  for (int k = 0; k < NW; ++k) {
    const int u0k = (blockIdx.x * NW + k) * per;
#pragma unroll
    for (int it = 0; it < E; ++it) {
      if (nreg[it] > 0 && pre[it] * HC <= u0k && u0k < (pre[it] + nreg[it]) * HC) {
        s_start[k][0] = it * NTH + threadIdx.x;
        s_start[k][1] = pre[it];
      }
    }
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < NW * STAGES; ++i) mbar_init(smem_addr(&bars[i]), 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmK);
    tma_prefetch_desc(&tmV);
  }
  __syncthreads();  // the last CTA-wide barrier: warps are independent from here

  const int wid = blockIdx.x * NW + warp;
  const int u0 = wid * per;
  const int n_units = u0 < U ? (U - u0 < per ? U - u0 : per) : 0;
  if (n_units == 0 || s_start[warp][0] < 0) {
    pdl_wait();
    pdl_trigger();
    return;
  }
  const int u1 = u0 + n_units;

  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t ring = smem_addr(smem) + warp * STAGES * G::kStage;
  const uint32_t bar0 = smem_addr(&bars[warp * STAGES]);
  StreamEntry* ent =
      reinterpret_cast<StreamEntry*>(smem + NW * STAGES * G::kStage) + warp * kStreamEntries;

  SeqWindow win;
  load_window<TOK>(a, win, s_start[warp][0], s_start[warp][1], HC, lane);
  int pend;
  fill_batch<TOK>(a, win, ent, 0, u0, u1, HC, lane, pend);
  commit_batch(a, ent, 0, u0, u1, lane, pend);
  if (n_units > 32) fill_batch<TOK>(a, win, ent, 1, u0, u1, HC, lane, pend);
  const int new_tail = (a.max_q + TOK - 2) / TOK;  // blocks past the last that hold new tokens

  // Fetch local unit p into ring slot p % STAGES (all lanes call).
  auto issue = [&](int p) {
    const int t = p >> 5;
    if ((p & 31) == 0 && t > 0) commit_batch(a, ent, t, u0, u1, lane, pend);
    if ((p & 31) == STAGES && t > 0 && (t + 1) * 32 < n_units)
      fill_batch<TOK>(a, win, ent, t + 1, u0, u1, HC, lane, pend);
    const StreamEntry e = ent[p & (kStreamEntries - 1)];
    const int seg = e.key >> 16, jj = e.key & 0xffff;
    const int kvh = (seg % HC) / a.col_chunks;
    if (a.k_new != nullptr && e.blk >= 0 && jj >= e.n - 1 - new_tail)
      append_unit<D, BS>(a, seg / HC, kvh, e.blk, jj, lane);
    if (lane == 0) {
      const int s = p % STAGES;
      const uint32_t bar = bar0 + s * 8;
      const uint32_t kd = ring + s * G::kStage;
      const uint32_t vd = kd + G::kTile;
      const int blk = e.blk < 0 ? 0 : e.blk;
      mbar_arrive_expect_tx(bar, 2 * BS * D * 2);
#pragma unroll
      for (int c = 0; c < G::kChunks; ++c) {
        tma_load_3d(kd + c * TOK * 128, &tmK, c * 64, kvh, blk * BS, bar);
        tma_load_3d(vd + c * TOK * 128, &tmV, c * 64, kvh, blk * BS, bar);
      }
    }
  };

  // Current piece: the part of one segment this worker covers.
  int cur_seg = -1, first_jj = 0, last_jj = 0, seg_n = 0, seg_first = 0;
  int row0 = 0, nq = 0, kvh = 0, chunk = 0, tok_end = 0;
  MmaCols<D, NT> c;
  const int ca = (lane & 3) * 2;

  // Write the piece: the output when it is the whole segment (and the output
  // is not gathered through the workspace), else a partial; the owner of the
  // segment's first unit also records the segment's number of parts.
  auto finish = [&]() {
    const bool whole = first_jj == 0 && last_jj == seg_n - 1;
    const int first_w = seg_first / per;
    const int part = wid - first_w;
    const int count = (seg_first + seg_n - 1) / per - first_w + 1;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        c.l[nt][0] += __shfl_xor_sync(0xffffffffu, c.l[nt][0], off);
        c.l[nt][1] += __shfl_xor_sync(0xffffffffu, c.l[nt][1], off);
      }
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const ColInfo ci = col_info(a, row0, nq, kvh, chunk * G::kCols + nt * kMmaCols + ca + e);
        if (!ci.valid) continue;
        const float l = c.l[nt][e];
        const float m = c.m[nt][e];
        const float inv = l > 0.f ? 1.f / l : 0.f;
        const int64_t rh = (int64_t)ci.qrow * a.num_q_heads + ci.qhead;
        if (whole && !a.force_split) {
          const int64_t ob = (int64_t)ci.qrow * a.out_stride + (int64_t)ci.qhead * D;
#pragma unroll
          for (int dm = 0; dm < KK; ++dm) {
            const int d = dm * 16 + (lane >> 2);
            store_out(a, ob + d, c.acc[nt][dm][e] * inv);
            store_out(a, ob + d + 8, c.acc[nt][dm][2 + e] * inv);
          }
        } else if (part < a.max_parts) {
          const int64_t base = rh * a.max_parts + part;
          float* po = a.part_out + base * D;
#pragma unroll
          for (int dm = 0; dm < KK; ++dm) {
            const int d = dm * 16 + (lane >> 2);
            po[d] = c.acc[nt][dm][e] * inv;
            po[d + 8] = c.acc[nt][dm][2 + e] * inv;
          }
          if (lane < 4) a.part_lse[base] = l > 0.f ? m + fast_log2(l) : -INFINITY;
        } else if (lane < 4) {
          raise_status(a.status, CLOVER_B200_DEV_CTX_RANGE);
        }
        if (first_jj == 0 && lane < 4) a.part_count[rh] = whole ? 1 : count;
      }
    }
  };

  // Start a piece of segment `seg`: its rows, columns, queries and limits.
  auto start = [&](int seg, int jj, int n, int s0) {
    cur_seg = seg;
    first_jj = jj;
    seg_n = n;
    seg_first = s0;
    const int b = seg / HC;
    const int hcix = seg - b * HC;
    kvh = hcix / a.col_chunks;
    chunk = hcix - kvh * a.col_chunks;
    row0 = __ldg(a.qsl + b);
    nq = __ldg(a.qsl + b + 1) - row0;
    tok_end = nq > 0 ? __ldg(a.ctx + row0 + nq - 1) : 0;
    tok_end = tok_end < a.max_ctx ? tok_end : a.max_ctx;
    load_cols<T, QF32, D, NT>(a, row0, nq, kvh, chunk * G::kCols, c, lane);
    // a row past its sequence's last row context is not covered by the units
    bool past = false;
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) past |= c.lim[nt][0] > n * TOK || c.lim[nt][1] > n * TOK;
    if (past && (lane & ~3) == 0) raise_status(a.status, CLOVER_B200_DEV_CTX_RANGE);
    c.reset();
  };

  pdl_wait();  // queries, new K/V, cache contents and workspace are final from here
  // First copies in flight, then the first piece's queries and limits load
  // while they land.
  const int npre = n_units < STAGES ? n_units : STAGES;
  for (int p = 0; p < npre; ++p) issue(p);
  int issued = npre;
  int consumed = 0;
  {
    const StreamEntry e = ent[0];
    start(e.key >> 16, e.key & 0xffff, e.n, e.seg0);
  }

  bool timed_out = false;
  for (int k = 0; k < n_units; ++k) {
    const int s = k % STAGES;
    if (!mbar_wait_bounded(bar0 + s * 8, (k / STAGES) & 1, a.wait_ns)) {
      timed_out = true;
      break;
    }
    consumed = k + 1;
    const StreamEntry e = ent[k & (kStreamEntries - 1)];
    const int seg = e.key >> 16, jj = e.key & 0xffff;
    if (seg != cur_seg) {
      if (cur_seg >= 0) finish();
      start(seg, jj, e.n, e.seg0);
    }
    last_jj = jj;
    const uint32_t ks = ring + s * G::kStage;
    const uint32_t vs = ks + G::kTile;
    const int tok0 = jj * TOK;
    const int nvalid = tok_end - tok0 > 0 ? tok_end - tok0 : 0;
    mma_stage<T, QF32, D, TOK, NT>(ks, vs, smem + (vs - smem_addr(smem)), tok0, nvalid,
                                   a.scale_log2, c, lane);
    __syncwarp();
    if (k + STAGES < n_units) {
      issue(k + STAGES);
      ++issued;
    }
  }
  if (timed_out) {
    // Drain this warp's copies still in flight (bounded) before giving up.
    for (int k = consumed; k < issued; ++k)
      mbar_wait_bounded(bar0 + (k % STAGES) * 8, (k / STAGES) & 1, kWaitLimitNs);
    if (lane == 0) raise_status(a.status, CLOVER_B200_DEV_TIMEOUT);
  } else if (cur_seg >= 0) {
    finish();
  }
  pdl_trigger();  // the split-K reduce may launch once every CTA got here
}

// ------------------------------------------------------------------ host side
template <typename T, bool QF32, int D, int BS, int NT>
static int stream_config(int dev, int* grid, int* smem_out) {
  using G = MmaGeom<D, BS, NT>;
  constexpr int kSmem = G::kPipeBytes + kMmaWarps * kStreamEntries * (int)sizeof(StreamEntry) + 1024;
  static int cached[64] = {0};  // CTAs per device ordinal (0 = not queried)
  static std::mutex mu;
  *smem_out = kSmem;
  if (dev >= 0 && dev < 64 && cached[dev] > 0) {
    *grid = cached[dev];
    return CLOVER_B200_OK;
  }
  std::lock_guard<std::mutex> lock(mu);
  auto kern = paged_decode_stream_kernel<T, QF32, D, BS, NT>;
  int rc = set_smem(kern, kSmem);
  if (rc) return rc;
  int per_sm = 0, sms = 0;
  rc = check_cuda(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kMmaThreads, kSmem),
                  "cudaOccupancyMaxActiveBlocksPerMultiprocessor");
  if (rc) return rc;
  rc = check_cuda(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev),
                  "cudaDeviceGetAttribute");
  if (rc) return rc;
  if (per_sm < 1)
    return set_error(CLOVER_B200_ERR_UNSUPPORTED, "stream decode: kernel does not fit on an SM");
  *grid = per_sm * sms;
  if (dev >= 0 && dev < 64) cached[dev] = *grid;
  return CLOVER_B200_OK;
}

template <typename T, bool QF32, int D, int BS, int NT>
static int stream_launch(const DecodeArgs* a, const CUtensorMap* tk, const CUtensorMap* tv,
                         cudaStream_t s, int* grid_out) {
  int dev = 0;
  int rc = check_cuda(cudaGetDevice(&dev), "cudaGetDevice");
  if (rc) return rc;
  int grid = 0, smem = 0;
  rc = stream_config<T, QF32, D, BS, NT>(dev, &grid, &smem);
  if (rc || a == nullptr) {
    *grid_out = grid;
    return rc;
  }
  return check_cuda(launch_pdl(paged_decode_stream_kernel<T, QF32, D, BS, NT>, dim3(grid),
                               dim3(kMmaThreads), smem, s, *tk, *tv, *a),
                    "paged_decode_stream launch");
}

template <typename T, bool QF32, int NT>
static int stream_dispatch_nt(int D, int BS, const DecodeArgs* a, const CUtensorMap* tk,
                              const CUtensorMap* tv, cudaStream_t s, int* grid) {
  if (BS == 16) {
    switch (D) {
      case 64: return stream_launch<T, QF32, 64, 16, NT>(a, tk, tv, s, grid);
      case 128: return stream_launch<T, QF32, 128, 16, NT>(a, tk, tv, s, grid);
      default: return stream_launch<T, QF32, 256, 16, 1>(a, tk, tv, s, grid);
    }
  }
  switch (D) {
    case 64: return stream_launch<T, QF32, 64, 32, NT>(a, tk, tv, s, grid);
    case 128: return stream_launch<T, QF32, 128, 32, NT>(a, tk, tv, s, grid);
    default: return stream_launch<T, QF32, 256, 32, 1>(a, tk, tv, s, grid);
  }
}

template <typename T, bool QF32>
static int stream_dispatch(int D, int BS, int cols, const DecodeArgs* a, const CUtensorMap* tk,
                           const CUtensorMap* tv, cudaStream_t s, int* grid) {
  return cols > kMmaCols ? stream_dispatch_nt<T, QF32, 2>(D, BS, a, tk, tv, s, grid)
                         : stream_dispatch_nt<T, QF32, 1>(D, BS, a, tk, tv, s, grid);
}

// Launch (a != null) or only size (a == null: *grid receives the CTA count)
// the stream decode for these types, shape and columns per warp (8 or 16) on
// the current device.
int stream_decode(int kv_dtype, int q_dtype, int D, int BS, int cols, const DecodeArgs* a,
                  const CUtensorMap* tk, const CUtensorMap* tv, cudaStream_t s, int* grid) {
  int g = 0;
  int rc;
  if (kv_dtype == CLOVER_B200_BF16) {
    rc = q_dtype == CLOVER_B200_F32
             ? stream_dispatch<__nv_bfloat16, true>(D, BS, cols, a, tk, tv, s, &g)
             : stream_dispatch<__nv_bfloat16, false>(D, BS, cols, a, tk, tv, s, &g);
  } else {
    rc = q_dtype == CLOVER_B200_F32 ? stream_dispatch<__half, true>(D, BS, cols, a, tk, tv, s, &g)
                                    : stream_dispatch<__half, false>(D, BS, cols, a, tk, tv, s, &g);
  }
  if (grid) *grid = g;
  return rc;
}

}  // namespace clover
