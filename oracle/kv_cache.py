"""CPU restatement of CloverInfer's ``KVCacheManager`` (test oracle).

Follows src/core/memory_manager.py:

* __init__        :19-53   caches ``[num_blocks, block_size, num_heads, head_dim]`` (zeros);
                           free stack ``list(range(num_blocks))``.
* allocate        :55-72   duplicate id -> ValueError; reserves ``ceil((seq_len+1)/bs)``
                           blocks (at least 1) by ``pop()`` from the END of the stack;
                           not enough -> RuntimeError("OOM: Not enough blocks").
* load_initial_kv :74-93   allocate if needed, then copy token ``t`` to
                           ``(table[t // bs], t % bs)``.
* append_slot     :95-121  one ``pop()`` when ``len == len(table) * bs``; returns
                           ``(physical_block, offset)`` of the new token; empty stack ->
                           RuntimeError("OOM during append").
* write_new_kv    :123-132 append_slot then write ``[H, D]`` into that slot.
* free            :134-143 unknown id ignored; blocks pushed back in table order.
* get_kernel_inputs :145-173 int32 tables padded with -1, int32 lengths, max length.
* _paged_attention_ref :192-239 gather + fp32 matmul with the FIXED ``1/sqrt(D)`` scale.

Test infrastructure only: the product never imports this module.
"""

from __future__ import annotations

import math
from typing import Dict, List, Tuple

import torch


class KVCacheOracle:
    def __init__(self, num_blocks: int, block_size: int, num_heads: int, head_dim: int,
                 dtype=torch.float32, with_storage: bool = True) -> None:
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.dtype = dtype
        shape = (num_blocks, block_size, num_heads, head_dim)
        self.k_cache = torch.zeros(shape, dtype=dtype) if with_storage else None
        self.v_cache = torch.zeros(shape, dtype=dtype) if with_storage else None
        self.free_blocks: List[int] = list(range(num_blocks))
        self.block_tables: Dict[str, List[int]] = {}
        self.context_lens: Dict[str, int] = {}

    def allocate(self, request_id: str, seq_len: int = 0) -> None:
        if request_id in self.block_tables:
            raise ValueError(f"Request {request_id} already exists")
        need = max(1, math.ceil((seq_len + 1) / self.block_size))
        if len(self.free_blocks) < need:
            raise RuntimeError("OOM: Not enough blocks")
        self.block_tables[request_id] = [self.free_blocks.pop() for _ in range(need)]
        self.context_lens[request_id] = seq_len

    def load_initial_kv(self, request_id: str, k_data: torch.Tensor, v_data: torch.Tensor) -> None:
        n = int(k_data.shape[0])
        if request_id not in self.block_tables:
            self.allocate(request_id, n)
        table = self.block_tables[request_id]
        for t in range(0, n, self.block_size):
            blk = table[t // self.block_size]
            m = min(self.block_size, n - t)
            self.k_cache[blk, :m] = k_data[t:t + m].to(self.dtype)
            self.v_cache[blk, :m] = v_data[t:t + m].to(self.dtype)
        self.context_lens[request_id] = n

    def append_slot(self, request_id: str) -> Tuple[int, int]:
        cur = self.context_lens[request_id]
        table = self.block_tables[request_id]
        if cur >= len(table) * self.block_size:
            if not self.free_blocks:
                raise RuntimeError("OOM during append")
            table.append(self.free_blocks.pop())
        self.context_lens[request_id] = cur + 1
        return table[cur // self.block_size], cur % self.block_size

    def write_new_kv(self, request_id: str, k: torch.Tensor, v: torch.Tensor) -> None:
        k = k.squeeze(0) if k.dim() == 3 else k
        v = v.squeeze(0) if v.dim() == 3 else v
        blk, off = self.append_slot(request_id)
        self.k_cache[blk, off] = k.to(self.dtype)
        self.v_cache[blk, off] = v.to(self.dtype)

    def free(self, request_id: str) -> None:
        if request_id not in self.block_tables:
            return
        self.free_blocks.extend(self.block_tables.pop(request_id))
        del self.context_lens[request_id]

    def slot(self, request_id: str, position: int) -> int:
        """Flat slot index ``block * block_size + offset`` of a token position."""
        table = self.block_tables[request_id]
        return table[position // self.block_size] * self.block_size + position % self.block_size

    def get_kernel_inputs(self, request_ids: List[str]):
        lens = [self.context_lens[r] for r in request_ids]
        tabs = [self.block_tables[r] for r in request_ids]
        width = max((len(t) for t in tabs), default=0)
        padded = torch.full((len(request_ids), width), -1, dtype=torch.int32)
        for i, t in enumerate(tabs):
            padded[i, :len(t)] = torch.tensor(t, dtype=torch.int32)
        return padded, torch.tensor(lens, dtype=torch.int32), max(lens, default=0)

    def paged_attention_ref(self, q: torch.Tensor, request_ids: List[str]) -> torch.Tensor:
        """memory_manager.py:192-239: per-sequence gather, scale fixed at 1/sqrt(D)."""
        n, h, d = q.shape
        out = torch.empty_like(q)
        scale = 1.0 / math.sqrt(d)
        for i, rid in enumerate(request_ids):
            idx = torch.tensor(self.block_tables[rid])
            L = self.context_lens[rid]
            k = self.k_cache[idx].reshape(-1, h, d)[:L].permute(1, 0, 2)
            v = self.v_cache[idx].reshape(-1, h, d)[:L].permute(1, 0, 2)
            s = torch.matmul(q[i].unsqueeze(1), k.transpose(-2, -1)) * scale
            out[i] = torch.matmul(torch.softmax(s, dim=-1), v).squeeze(1)
        return out
