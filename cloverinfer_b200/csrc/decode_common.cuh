// Definitions shared by the paged decode kernels: launch-shape knobs, the
// kernel argument blocks, column mapping, q/out access, the tensor-core stage
// geometry and the launch helpers.
#pragma once

#include <stdlib.h>

#include <mutex>
#include <utility>

#include <cuda_fp8.h>

#include "common.cuh"

namespace clover {

constexpr int kNumWarps = 4;  // SIMT path
constexpr int kThreads = kNumWarps * 32;
constexpr int kMmaCols = 8;

// Tensor-core path launch shape (compile-time knobs).
#ifndef CLOVER_MMA_WARPS
#define CLOVER_MMA_WARPS 2
#endif
#ifndef CLOVER_MMA_STAGES
#define CLOVER_MMA_STAGES 2
#endif
#ifndef CLOVER_MMA_STAGE_TOKENS
#define CLOVER_MMA_STAGE_TOKENS 16
#endif
#ifndef CLOVER_MMA_MIN_CTAS
#define CLOVER_MMA_MIN_CTAS 6
#endif
constexpr int kMmaWarps = CLOVER_MMA_WARPS;
constexpr int kMmaThreads = kMmaWarps * 32;
// Stream kernel: each CTA scans up to kStreamSeqsPerThread sequences per
// thread; a worker's range is at least kStreamMinUnits blocks when there is
// less work than workers.
constexpr int kStreamSeqsPerThread = 16;
constexpr int kStreamMaxSeqs = kMmaThreads * kStreamSeqsPerThread;
constexpr int kStreamMinUnits = 8;

struct DecodeArgs {
  void* out;
  int64_t out_stride;
  const void* q;
  int64_t q_stride;
  int32_t q_dtype;
  int32_t out_dtype;  // the output's type (the query's, except for a gather into a consumer buffer)
  const void* k_cache;
  const void* v_cache;
  const int32_t* tables;
  int32_t table_stride;
  const int32_t* seq_rows;
  const int32_t* qsl;
  const int32_t* ctx;
  int32_t num_q_heads;
  int32_t num_kv_heads;
  int32_t group;
  int32_t block_size;
  int64_t num_blocks;
  float scale_log2;
  int32_t part_tokens;
  int32_t max_parts;
  int32_t cols_per_cta;
  int32_t col_chunks;
  float* part_out;
  float* part_lse;
  int32_t* status;
  // Fused KV append (decode_step): row r's new token k_new/v_new[r] (all local
  // KV heads, token stride new_stride elements) is written to position
  // ctx[r] - 1 before attending.  Null when the caller appended already.
  const void* k_new;
  const void* v_new;
  int64_t new_stride;
  int32_t kv_esz;
  // Gathered output (decode_step_gather): every row goes through the split-K
  // workspace, even a single-partition one, and the reduce writes the output.
  int32_t force_split;
  // Balanced (stream) decomposition: the units (one KV block of one KV head
  // and column chunk) of all sequences are split evenly over every resident
  // warp.  part_count[row * num_q_heads + head] holds how many partials the
  // row's (sequence, head) was split into; null for the partition kernels.
  int32_t n_seqs;
  int32_t max_ctx;
  int32_t max_q;
  // One query row per sequence (max_q == 1 and as many rows as sequences):
  // query_start_loc is then the identity and the kernels do not load it.
  int32_t rows_identity;
  int32_t min_units;
  int32_t* part_count;
  // Limit of this launch's bounded waits (wait_limit_ns() at launch).
  uint64_t wait_ns;
};

// Fused output all-gather over peer memory, LL style: every value travels as
// one 8-byte word (epoch << 32 | fp32 bits) written with a single 64-bit
// store, so a reader that sees the current epoch in a word also sees its
// value — no fences and no global barrier.  Words live in each rank's receive
// buffer, [2 parities][rows, total_q_heads, D] (parity = epoch & 1).  The
// local sync words: kSyncDone counts finished reduce CTAs of this launch;
// kSyncEpoch is the number of completed calls.
constexpr int kSyncDone = 0;
constexpr int kSyncEpoch = 1;
constexpr int kSyncInts = 64;

struct GatherArgs {
  uint64_t* const* peer_ll;  // [n_ranks] receive buffers (own one at [rank])
  int32_t* sync;             // this rank's sync words
  int32_t n_ranks, rank, q_head_offset, total_q_heads;
  int64_t ll_half_words;     // words per parity half (>= rows * total_q_heads * D)
  int32_t units;             // reduce units: (row, local head[, 32-dim chunk])
  int32_t rows;              // query rows of the step
};

struct ColInfo {
  int32_t qrow, qhead, limit;
  bool valid;
};

__device__ __forceinline__ ColInfo col_info(const DecodeArgs& a, int row0, int nq, int kvh,
                                            int cglob) {
  ColInfo c{0, 0, 0, false};
  if (cglob < nq * a.group) {
    const int j = cglob / a.group;
    c.qrow = row0 + j;
    c.qhead = kvh * a.group + (cglob - j * a.group);
    c.limit = __ldg(a.ctx + c.qrow);
    c.valid = true;
  }
  return c;
}

__device__ __forceinline__ float load_q(const DecodeArgs& a, int64_t idx) {
  switch (a.q_dtype) {
    case CLOVER_B200_F32: return __ldg(static_cast<const float*>(a.q) + idx);
    case CLOVER_B200_F16: return __half2float(static_cast<const __half*>(a.q)[idx]);
    default: return __bfloat162float(static_cast<const __nv_bfloat16*>(a.q)[idx]);
  }
}

__device__ __forceinline__ void store_out(const DecodeArgs& a, int64_t idx, float v) {
  switch (a.out_dtype) {
    case CLOVER_B200_F32: static_cast<float*>(a.out)[idx] = v; break;
    case CLOVER_B200_F16: static_cast<__half*>(a.out)[idx] = __float2half_rn(v); break;
    default: static_cast<__nv_bfloat16*>(a.out)[idx] = __float2bfloat16_rn(v); break;
  }
}

// ------------------------------------------------------------------ tensor-core path
// One pipeline stage holds BPS consecutive KV blocks (K and V tiles) of one KV
// head: kTok = BPS * BS token rows of D values, stored per 128-byte chunk of
// a row (64 bf16/fp16 values, or 128 fp8 values) with the TMA 128-byte
// swizzle.  An fp8 cache (F8) adds one fp16 staging stage (K and V) per warp
// that each landed stage is converted into before the tensor-core step.
//
// CW > 1 (column warps): CW warps share each token warp's ring, each holding
// its own NT n-tiles of the CTA's columns, so a CTA of kMmaWarps * CW warps
// carries kCols * CW columns with the ring of kMmaWarps warps.
template <int D, int BS, int NT = 1, bool F8 = false, int CW = 1>
struct MmaGeom {
  static constexpr int kEsz = F8 ? 1 : 2;            // bytes per cached value
  static constexpr int kChunkVals = 128 / kEsz;       // values per 128-byte chunk
  static constexpr int kChunks = D / kChunkVals;      // TMA boxes per tile
  static constexpr int kBps = (CLOVER_MMA_STAGE_TOKENS > BS ? CLOVER_MMA_STAGE_TOKENS : BS) / BS;
  static constexpr int kTok = kBps * BS;   // tokens per stage
  static constexpr int kTile = kTok * D * kEsz;
  static constexpr int kStage = 2 * kTile;  // K + V
  static constexpr int kConv = F8 ? 2 * kTok * D * 2 : 0;  // fp16 staging (K + V)
  // keep the ring within the per-CTA shared memory limit; fp8 rings are
  // deeper (their stages are half the bytes)
  static constexpr int kWant = F8 ? 3 * CLOVER_MMA_STAGES / 2 : CLOVER_MMA_STAGES;
  static constexpr int kStages = kMmaWarps * (kWant * kStage + kConv) <= 200 * 1024
                                     ? kWant
                                     : (kMmaWarps * (2 * kStage + kConv) <= 200 * 1024 ? 2 : 1);
  static constexpr int kWarpBytes = kStages * kStage + kConv;
  static constexpr int kPipeBytes = kMmaWarps * kWarpBytes;
  static constexpr int kCols = kMmaCols * NT;  // columns per warp (NT n-tiles)
  static constexpr int kCtaCols = kCols * CW;  // columns per CTA
  static constexpr int kThreads = kMmaWarps * CW * 32;
  static constexpr int kRedBytes = kMmaWarps * kCtaCols * (D + 4) * 4 + 2 * kMmaWarps * kCtaCols * 4;
  static constexpr int kSmem = (kPipeBytes > kRedBytes ? kPipeBytes : kRedBytes) + 1024;
};

// byte offset of 16-byte chunk `cg` (along head_dim) of stage row `r`
template <int TOK>
__device__ __forceinline__ uint32_t swz(int r, int cg) {
  const int c64 = cg >> 3, c = cg & 7;
  return (uint32_t)(c64 * TOK * 128 + r * 128 + ((c ^ (r & 7)) << 4));
}

// Expand one landed fp8 (e4m3) tile — TOK rows of D bytes, 128-byte
// swizzled per 128-value chunk — into the fp16 layout the tensor-core step
// reads (swz).  e4m3 values are exact in fp16.  One warp; 16 values per
// lane and step.
template <int D, int TOK>
__device__ __forceinline__ void expand_fp8_tile(const uint8_t* src, uint8_t* dst, int lane) {
  constexpr int kUnits = D / 16;  // 16-byte fp8 units per row
#pragma unroll 4
  for (int i = lane; i < TOK * kUnits; i += 32) {
    const int r = i / kUnits, u = i - r * kUnits;
    const int c8 = u >> 3, uu = u & 7;
    const uint4 raw = *reinterpret_cast<const uint4*>(src + c8 * TOK * 128 + r * 128 + ((uu ^ (r & 7)) << 4));
    const uint32_t w[4] = {raw.x, raw.y, raw.z, raw.w};
    uint32_t h[8];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const __half2_raw lo = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[j] & 0xffffu), __NV_E4M3);
      const __half2_raw hi = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[j] >> 16), __NV_E4M3);
      h[2 * j] = (uint32_t)lo.x | ((uint32_t)lo.y << 16);
      h[2 * j + 1] = (uint32_t)hi.x | ((uint32_t)hi.y << 16);
    }
    const int cg = u * 2;  // 8-value fp16 units of this row
    *reinterpret_cast<uint4*>(dst + swz<TOK>(r, cg)) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(dst + swz<TOK>(r, cg + 1)) = make_uint4(h[4], h[5], h[6], h[7]);
  }
}

// Per-warp column state of the tensor-core path: NT n-tiles of 8 columns.
// Lane l holds, for every n-tile, the query B-operand fragments of column
// l / 4, and the accumulators of columns (l % 4) * 2 and (l % 4) * 2 + 1
// (O^T rows d = 16 dm + l / 4 and d + 8) with their running max m (base-2
// domain, uniform over the lanes of a column), partial sum l and causal
// limit (tokens [0, lim) are attended).
template <int D, int NT>
struct MmaCols {
  uint32_t qh[NT][D / 16][2], ql[NT][D / 16][2];
  float acc[NT][D / 16][4];
  float m[NT][2], l[NT][2];
  int lim[NT][2];

  __device__ __forceinline__ void reset() {
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      m[nt][0] = m[nt][1] = -INFINITY;
      l[nt][0] = l[nt][1] = 0.f;
#pragma unroll
      for (int i = 0; i < D / 16; ++i) acc[nt][i][0] = acc[nt][i][1] = acc[nt][i][2] = acc[nt][i][3] = 0.f;
    }
  }
};

// One pipeline stage of the tensor-core path for one warp: scores
// S[tokens x columns] = K . Q^T with mma.sync m16n8k16 (tokens = M, one
// n-tile of 8 columns per MMA, fp32 accumulate; fp32 queries as hi + lo
// 16-bit halves; each K fragment is loaded once for all n-tiles), scale to
// the base-2 domain and causal mask (token position tok0 of the stage's
// first row), online-softmax update of (m, l), then
// O^T[dims x cols] += V^T . P^T with V^T from ldmatrix.trans (loaded once for
// all n-tiles) and P^T from movmatrix.trans (P split hi + lo).  ks / vs:
// shared addresses of the stage's K and V tiles (vgen: generic pointer to the
// V tile).  Rows at and past nvalid hold no context token: they are zeroed in
// V so that P = 0 never multiplies a non-finite value.
template <typename T, bool QF32, int D, int TOK, int NT>
__device__ __forceinline__ void mma_stage(uint32_t ks, uint32_t vs, uint8_t* vgen, int tok0,
                                          int nvalid, float scale_log2, MmaCols<D, NT>& c,
                                          int lane) {
  constexpr int MT = TOK / 16;  // token m-tiles per stage
  constexpr int KK = D / 16;    // k-steps (QK) / m-tiles (PV) over head_dim
  if (nvalid < TOK) {
    for (int idx = lane; idx < (TOK - nvalid) * (D / 8); idx += 32) {
      const int r = nvalid + idx / (D / 8);
      *reinterpret_cast<uint4*>(vgen + swz<TOK>(r, idx % (D / 8))) = make_uint4(0, 0, 0, 0);
    }
    __syncwarp();
  }

  // ---- S = K . Q^T (tokens x columns): independent accumulator chains
  // (even/odd k-steps, hi/lo query halves) summed at the end.
  float sc[NT][MT][4];
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    float ch[NT][QF32 ? 4 : 2][4];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int q = 0; q < (QF32 ? 4 : 2); ++q) ch[nt][q][0] = ch[nt][q][1] = ch[nt][q][2] = ch[nt][q][3] = 0.f;
    const int r = mt * 16 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
    for (int kk = 0; kk < KK; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(ks + swz<TOK>(r, kk * 2 + (lane >> 4)), a0, a1, a2, a3);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        MmaOp<T>::run(ch[nt][kk & 1], a0, a1, a2, a3, c.qh[nt][kk][0], c.qh[nt][kk][1]);
        if (QF32)
          MmaOp<T>::run(ch[nt][2 + (kk & 1)], a0, a1, a2, a3, c.ql[nt][kk][0], c.ql[nt][kk][1]);
      }
    }
#pragma unroll
    for (int nt = 0; nt < NT; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        sc[nt][mt][e] = QF32 ? (ch[nt][0][e] + ch[nt][1][e]) + (ch[nt][2][e] + ch[nt][3][e])
                             : ch[nt][0][e] + ch[nt][1][e];
  }
  // ---- scale (base-2 domain), causal mask, stage max per column, rescale
  float u[NT][2];
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = tok0 + mt * 16 + (lane >> 2) + h * 8;
        const float sa = t < c.lim[nt][0] ? sc[nt][mt][2 * h] * scale_log2 : -INFINITY;
        const float sb = t < c.lim[nt][1] ? sc[nt][mt][2 * h + 1] * scale_log2 : -INFINITY;
        sc[nt][mt][2 * h] = sa;
        sc[nt][mt][2 * h + 1] = sb;
        mx_a = fmaxf(mx_a, sa);
        mx_b = fmaxf(mx_b, sb);
      }
    }
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
    }
    const float nm_a = fmaxf(c.m[nt][0], mx_a), nm_b = fmaxf(c.m[nt][1], mx_b);
    u[nt][0] = nm_a == -INFINITY ? 0.f : nm_a;
    u[nt][1] = nm_b == -INFINITY ? 0.f : nm_b;
    const float al_a = fast_exp2(c.m[nt][0] - u[nt][0]), al_b = fast_exp2(c.m[nt][1] - u[nt][1]);
    c.m[nt][0] = nm_a;
    c.m[nt][1] = nm_b;
    c.l[nt][0] *= al_a;
    c.l[nt][1] *= al_b;
#pragma unroll
    for (int i = 0; i < KK; ++i) {
      c.acc[nt][i][0] *= al_a;
      c.acc[nt][i][1] *= al_b;
      c.acc[nt][i][2] *= al_a;
      c.acc[nt][i][3] *= al_b;
    }
  }
  // ---- O^T += V^T . P^T  (P split hi + lo; V^T via ldmatrix.trans)
#pragma unroll
  for (int mt = 0; mt < MT; ++mt) {
    uint32_t bh[NT][2], bl[NT][2];
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
      const float p0 = fast_exp2(sc[nt][mt][0] - u[nt][0]), p1 = fast_exp2(sc[nt][mt][1] - u[nt][1]);
      const float p2 = fast_exp2(sc[nt][mt][2] - u[nt][0]), p3 = fast_exp2(sc[nt][mt][3] - u[nt][1]);
      c.l[nt][0] += p0 + p2;
      c.l[nt][1] += p1 + p3;
      uint32_t h_top, l_top, h_bot, l_bot;
      split_pack<T>(p0, p1, h_top, l_top);
      split_pack<T>(p2, p3, h_bot, l_bot);
      bh[nt][0] = movm_trans(h_top);
      bh[nt][1] = movm_trans(h_bot);
      bl[nt][0] = movm_trans(l_top);
      bl[nt][1] = movm_trans(l_bot);
    }
    const int grp = lane >> 3;
    const int r = mt * 16 + (lane & 7) + (grp >> 1) * 8;
    uint32_t va[KK][4];
#pragma unroll
    for (int dm = 0; dm < KK; ++dm)
      ldsm_x4_trans(vs + swz<TOK>(r, dm * 2 + (grp & 1)), va[dm][0], va[dm][1], va[dm][2], va[dm][3]);
#pragma unroll
    for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
      for (int dm = 0; dm < KK; ++dm)
        MmaOp<T>::run(c.acc[nt][dm], va[dm][0], va[dm][1], va[dm][2], va[dm][3], bh[nt][0], bh[nt][1]);
#pragma unroll
      for (int dm = 0; dm < KK; ++dm)
        MmaOp<T>::run(c.acc[nt][dm], va[dm][0], va[dm][1], va[dm][2], va[dm][3], bl[nt][0], bl[nt][1]);
    }
  }
}

// Query values (fp32, as loaded) and causal limits of n-tile columns
// [col0, col0 + 8 NT) of (query rows row0 .. row0 + nq - 1, KV head kvh):
// the loads are issued here and first used by pack_cols, so other loads and
// copies can be issued in between.
template <int D, int NT>
struct QRaw {
  float x[NT][D / 16][4];
  int lim[NT][2];
};

template <int D, int NT>
__device__ __forceinline__ void load_cols_raw(const DecodeArgs& a, int row0, int nq, int kvh,
                                              int col0, QRaw<D, NT>& r, int lane) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
    const ColInfo ci = col_info(a, row0, nq, kvh, col0 + nt * kMmaCols + (lane >> 2));
    const int64_t qbase = (int64_t)ci.qrow * a.q_stride + (int64_t)ci.qhead * D;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const int d0 = kk * 16 + (lane & 3) * 2;
      r.x[nt][kk][0] = ci.valid ? load_q(a, qbase + d0) : 0.f;
      r.x[nt][kk][1] = ci.valid ? load_q(a, qbase + d0 + 1) : 0.f;
      r.x[nt][kk][2] = ci.valid ? load_q(a, qbase + d0 + 8) : 0.f;
      r.x[nt][kk][3] = ci.valid ? load_q(a, qbase + d0 + 9) : 0.f;
    }
    const int ca = col0 + nt * kMmaCols + (lane & 3) * 2;
    const ColInfo c0 = col_info(a, row0, nq, kvh, ca);
    const ColInfo c1 = col_info(a, row0, nq, kvh, ca + 1);
    r.lim[nt][0] = c0.valid ? c0.limit : 0;
    r.lim[nt][1] = c1.valid ? c1.limit : 0;
  }
}

// MMA B-operand fragments (columns = lane / 4 of each n-tile) from the raw
// query values: hi + lo 16-bit halves for fp32 queries.
template <typename T, bool QF32, int D, int NT>
__device__ __forceinline__ void pack_cols(const QRaw<D, NT>& r, MmaCols<D, NT>& c) {
#pragma unroll
  for (int nt = 0; nt < NT; ++nt) {
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      if (QF32) {
        split_pack<T>(r.x[nt][kk][0], r.x[nt][kk][1], c.qh[nt][kk][0], c.ql[nt][kk][0]);
        split_pack<T>(r.x[nt][kk][2], r.x[nt][kk][3], c.qh[nt][kk][1], c.ql[nt][kk][1]);
      } else {
        c.qh[nt][kk][0] = Pack<T>::pack(r.x[nt][kk][0], r.x[nt][kk][1]);
        c.qh[nt][kk][1] = Pack<T>::pack(r.x[nt][kk][2], r.x[nt][kk][3]);
      }
    }
    c.lim[nt][0] = r.lim[nt][0];
    c.lim[nt][1] = r.lim[nt][1];
  }
}

template <typename T, bool QF32, int D, int NT>
__device__ __forceinline__ void load_cols(const DecodeArgs& a, int row0, int nq, int kvh, int col0,
                                          MmaCols<D, NT>& c, int lane) {
  QRaw<D, NT> r;
  load_cols_raw<D, NT>(a, row0, nq, kvh, col0, r, lane);
  pack_cols<T, QF32, D, NT>(r, c);
}

// ------------------------------------------------------------------ host launch helpers
// Programmatic dependent launch: on by default; CLOVER_B200_PDL=0 turns it off.
static bool pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("CLOVER_B200_PDL");
    return !(e && e[0] == '0');
  }();
  return on;
}

template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

template <typename Kern>
static int set_smem(Kern k, int bytes) {
  static std::mutex mu;
  std::lock_guard<std::mutex> lock(mu);
  return check_cuda(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                    "cudaFuncSetAttribute");
}

struct DecodeArgs;
// Balanced decode (paged_decode_stream.cu): launches when `a` is set, else
// only reports the grid (resident CTAs on the current device) in *grid.
int stream_decode(int kv_dtype, int q_dtype, int D, int BS, int cols, const DecodeArgs* a,
                  const CUtensorMap* tk, const CUtensorMap* tv, cudaStream_t s, int* grid);

// CTAs per SM the tensor-core kernels are compiled for: 16-column warps keep
// twice the accumulators (and run 3 CTAs per SM at block 32, whose stages
// are twice as large); an fp8 cache's warps hold a deeper ring plus an fp16
// staging stage (5 CTAs per SM).
// Column-split CTAs (CW = 2: four warps) run 3 per SM, 12 warps.
template <int D, int NT, bool F8 = false, int CW = 1>
constexpr int mma_min_ctas() {
  return D >= 256 ? 1 : ((NT > 1 || CW > 1) ? 3 : (F8 ? 5 : CLOVER_MMA_MIN_CTAS));
}

}  // namespace clover
