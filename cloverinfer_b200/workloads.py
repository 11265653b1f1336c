"""Seeded synthetic workloads for the five reference configurations.

Shapes and value distributions follow the configurations the upstream metric
is quoted on (no dataset is involved; synthetic inputs stand in):

  c1  OPT-125m shape, CPU-reference case: 12 layers, 12 heads (MHA), D=64, fp32,
      batch 4, contexts U[128, 512], block 16, tables from a 256-block pool.
  c2  Qwen2.5-7B GQA: 28 q / 4 KV heads, D=128, bf16, block 16, batch 32,
      contexts U[1024, 4096], values N(0,1)*0.5, random non-contiguous tables.
  c3  Llama-3-8B long context: 32 q / 8 KV heads, D=128, bf16, block 16,
      batch 8, every context 32768, split-K with 512-token partitions.
  c4  mixed continuous batching, Llama-3-8B shape, fp16, batch 256, contexts
      log-uniform [16, 16384], 1-4 new tokens per sequence, block 32,
      2M-block pool (head-sharded over 8 GPUs), 30 % of blocks churned per step.
  c5  Llama-3-70B shape: 64 q / 8 KV heads, D=128, bf16, block 16, batch 64,
      contexts U[8192, 65536], one KV head per GPU on 8 GPUs.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field
from typing import List

import torch


@dataclass
class Config:
    name: str
    num_layers: int
    num_q_heads: int
    num_kv_heads: int
    head_dim: int
    dtype: torch.dtype
    block_size: int
    batch: int
    ctx_lo: int
    ctx_hi: int
    ctx_dist: str = "uniform"      # uniform | loguniform | fixed
    new_lo: int = 1
    new_hi: int = 1
    pool_blocks: int = 0           # 0: just enough (+ slack)
    value_scale: float = 1.0
    partition_tokens: int = 0
    churn: float = 0.0
    score_scale: float = field(default=0.0)

    def __post_init__(self):
        if not self.score_scale:
            self.score_scale = 1.0 / math.sqrt(self.head_dim)

    @property
    def group(self) -> int:
        return self.num_q_heads // self.num_kv_heads


CONFIGS = {
    "c1": Config("c1-opt125m-fp32", 12, 12, 12, 64, torch.float32, 16, 4, 128, 512,
                 pool_blocks=256, score_scale=1.0 / 8.0),
    "c2": Config("c2-qwen2.5-7b-gqa-bf16", 1, 28, 4, 128, torch.bfloat16, 16, 32, 1024, 4096,
                 value_scale=0.5),
    "c3": Config("c3-llama3-8b-32k-bf16", 1, 32, 8, 128, torch.bfloat16, 16, 8, 32768, 32768,
                 ctx_dist="fixed", partition_tokens=512),
    "c4": Config("c4-mixed-cb-llama3-8b-fp16", 1, 32, 8, 128, torch.float16, 32, 256, 16, 16384,
                 ctx_dist="loguniform", new_lo=1, new_hi=4, pool_blocks=2 * 1024 * 1024, churn=0.3),
    "c5": Config("c5-llama3-70b-bf16", 1, 64, 8, 128, torch.bfloat16, 16, 64, 8192, 65536),
}


def context_lengths(cfg: Config, seed: int, batch: int = 0) -> List[int]:
    g = torch.Generator().manual_seed(seed)
    b = batch or cfg.batch
    if cfg.ctx_dist == "fixed":
        return [cfg.ctx_hi] * b
    if cfg.ctx_dist == "loguniform":
        u = torch.rand(b, generator=g, dtype=torch.float64)
        lo, hi = math.log(cfg.ctx_lo), math.log(cfg.ctx_hi)
        return [int(round(math.exp(lo + (hi - lo) * float(x)))) for x in u]
    return torch.randint(cfg.ctx_lo, cfg.ctx_hi + 1, (b,), generator=g).tolist()


def new_tokens(cfg: Config, seed: int, batch: int = 0) -> List[int]:
    g = torch.Generator().manual_seed(seed + 1)
    b = batch or cfg.batch
    return torch.randint(cfg.new_lo, cfg.new_hi + 1, (b,), generator=g).tolist()


def randn(shape, seed: int, scale: float, dtype: torch.dtype, device="cpu") -> torch.Tensor:
    """N(0,1)*scale rounded to ``dtype`` (generated in fp32 from a seed)."""
    g = torch.Generator(device=device).manual_seed(seed)
    return (torch.randn(shape, generator=g, device=device, dtype=torch.float32) * scale).to(dtype)


def kv_bytes(ctx_per_seq: List[int], num_kv_heads: int, head_dim: int, dtype: torch.dtype) -> int:
    """Algorithmic KV bytes one decode step reads: sum_s ctx_s * Hkv * D * 2 * e."""
    e = torch.empty((), dtype=dtype).element_size()
    return sum(ctx_per_seq) * num_kv_heads * head_dim * 2 * e


def build_decode_step(cfg, rank, world, lens, device, seed=0, gather=None, n_new=None,
                      partition_tokens=0, pool_blocks=None):
    """Pool + static buffers for one decode step: sequence b holds lens[b]
    tokens after the step, n_new[b] of them (default 1) appended by it and
    attended causally.  ``partition_tokens``: 0 leaves the split to the
    library, -1 asks for the balanced split, None takes the configuration's
    fixed partition length on one GPU (the library's choice on several).
    ``pool_blocks``: None takes the configuration's pool size (capped at half
    the device's free memory), 0 just the blocks the tables need."""
    from . import _lib
    from .head_groups import kv_head_shards
    from .kv_cache import PagedKVPool, auto_partition

    lo, hi = kv_head_shards(cfg.num_kv_heads, world)[rank]
    hkv_l = hi - lo
    hq_l = hkv_l * cfg.group
    B, bs, D, dt = len(lens), cfg.block_size, cfg.head_dim, cfg.dtype
    n_new = [1] * B if n_new is None else list(n_new)
    T = sum(n_new)
    blocks = sum(-(-n // bs) for n in lens) + 64
    want = cfg.pool_blocks if pool_blocks is None else pool_blocks
    if want > blocks and torch.device(device).type == "cuda":
        # the configured pool (C4: 2M blocks), as far as half the free memory
        # holds it; the shuffled free stack spreads the tables over all of it
        esz = torch.empty((), dtype=dt).element_size()
        per_block = 2 * bs * hkv_l * D * esz
        free, _ = torch.cuda.mem_get_info(device)
        blocks = max(blocks, min(want, int(0.5 * free) // per_block))
    pool = PagedKVPool(blocks, bs, hkv_l, D, num_layers=1, dtype=dt, device=device,
                       max_seqs=B, max_blocks_per_seq=max(-(-n // bs) for n in lens) + 1)
    pool.shuffle_free_stack(1234 + seed)
    pool.reserve(list(range(B)), list(lens))
    g = torch.Generator(device=device).manual_seed(4321 + rank)
    chunk = 1 << 28
    for t in (pool.k, pool.v):  # fill the whole pool: every block holds N(0,1)*scale data
        flat = t.view(-1)
        for i in range(0, flat.numel(), chunk):
            part = flat[i:i + chunk]
            if dt == torch.float32:
                part.normal_(0.0, cfg.value_scale, generator=g)
            else:
                part.copy_(torch.randn(part.numel(), generator=g, device=device).mul_(cfg.value_scale).to(dt))
    q = (torch.randn((T, hq_l, D), generator=g, device=device) * cfg.value_scale).to(dt).float()
    kn = (torch.randn((T, hkv_l, D), generator=g, device=device) * cfg.value_scale).to(dt)
    vn = (torch.randn((T, hkv_l, D), generator=g, device=device) * cfg.value_scale).to(dt)
    max_q = max(n_new)
    pt = partition_tokens
    if pt is None:
        pt = cfg.partition_tokens if world == 1 else 0
    if pt == 0:
        pt = auto_partition(lens, max(n_new), world > 1)
    pt = _lib.decode_partition_tokens(B, T, max_q, max(lens), hq_l, hkv_l, D, bs, dt, torch.float32, pt)
    if pt == 0:
        pt = _lib.PARTITION_BALANCED  # the library took the balanced split
    offs, ctx = [0], []
    for n, k in zip(lens, n_new):
        offs.append(offs[-1] + k)
        ctx += list(range(n - k + 1, n + 1))
    meta = torch.tensor(list(range(B)) + offs + ctx, dtype=torch.int32, device=device)
    rows, offs_d, ctx_d = meta[:B], meta[B:2 * B + 1], meta[2 * B + 1:]
    out = torch.empty_like(q)
    if gather is not None:
        nbytes = _lib.decode_gather_workspace_bytes(B, T, max_q, max(lens), hq_l, hkv_l, D, bs, dt,
                                                    q.dtype, pt)
    else:
        nbytes = _lib.decode_workspace_bytes(B, T, max_q, max(lens), hq_l, hkv_l, D, bs, dt, q.dtype, pt)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=device)
    # Table row b belongs to sequence b (reserved in order above): the tables are
    # per sequence, as the reference's get_kernel_inputs lays them out
    # (memory_manager.py:145-173), so the launches take no row indirection.
    common = dict(max_queries_per_seq=max_q, max_ctx_len=max(lens), score_scale=cfg.score_scale,
                  seq_rows=None, partition_tokens=pt, workspace=ws, status=pool.status)

    def decode_only():
        _lib.paged_decode(out, q, pool.k[0], pool.v[0], pool.tables, offs_d, ctx_d, **common)

    def step():
        if gather is not None:
            # fused append + decode, then reduce with the all-gather fused in
            _lib.decode_step_gather(q, pool.k[0], pool.v[0], kn, vn, pool.tables, offs_d, ctx_d,
                                    gather, **common)
            return
        # append each row's new token at position ctx-1 and attend (fused)
        _lib.decode_step(out, q, pool.k[0], pool.v[0], kn, vn, pool.tables, offs_d, ctx_d, **common)

    return dict(pool=pool, q=q, out=out, step=step, decode_only=decode_only, hkv_local=hkv_l,
                hq_local=hq_l, kv_range=(lo, hi), partition_tokens=pt, workspace_bytes=nbytes,
                rows=T, max_q=max_q, k_new=kn, v_new=vn, n_new=n_new, ctx_rows=ctx,
                pool_blocks=pool.num_blocks)

