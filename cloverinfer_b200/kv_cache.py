"""Device-resident paged KV cache: block pool, LIFO allocator and block tables.

``PagedKVPool`` owns, in HBM:

* per-layer caches ``k[layer]``/``v[layer]`` of shape
  ``[num_blocks, block_size, num_kv_heads, head_dim]`` — the layout of
  ``KVCacheManager`` (src/core/memory_manager.py:35-46), zero-initialised;
* the free-block stack ``free_stack[num_blocks]`` + ``free_top`` (LIFO, the
  upstream ``list(range(num_blocks))`` with ``pop()``/``append``, :49);
* block tables ``tables[max_seqs, max_blocks_per_seq]`` (-1 padded, :167) and
  ``table_len[max_seqs]``, shared by every layer (all layers of a sequence
  hold the same number of tokens).

The host keeps only counters (free blocks, blocks per row) so it can raise the
upstream errors (``RuntimeError`` on exhaustion, :64-65, :108-109) before any
kernel runs; block ids never leave the GPU on the hot path.

``KVCacheManager`` is the drop-in for the upstream class of the same name:
same constructor, methods, return values and errors, backed by the pool.
"""

from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch

from . import _lib


def to_device_i32(values: Sequence[int], device: torch.device) -> torch.Tensor:
    """One pinned, stream-ordered H2D copy of a small int32 array."""
    h = torch.tensor(list(values), dtype=torch.int32)
    if device.type != "cuda":
        return h
    return h.pin_memory().to(device, non_blocking=True)


def auto_partition(contexts: Sequence[int], max_q: int, sharded: bool = False) -> int:
    """The split for a batch whose caller left it to the library (0): the
    balanced split (``_lib.PARTITION_BALANCED``) for ragged batches of
    single-token rows — the longest context at least 1.25x the mean, where
    fixed partitions sized for the longest leave most CTAs short or empty —
    else 0 (fixed partitions chosen by the library from the longest context).
    Sharded steps keep 0."""
    n = len(contexts)
    if sharded or max_q != 1 or n == 0 or n > 1024:
        return 0
    longest = max(contexts)
    return _lib.PARTITION_BALANCED if longest * n >= 1.25 * sum(contexts) and longest > 0 else 0


class PagedKVPool:
    def __init__(self, num_blocks: int, block_size: int, num_kv_heads: int, head_dim: int, *,
                 num_layers: int = 1, dtype: torch.dtype = torch.bfloat16,
                 device="cuda", max_seqs: int = 256, max_blocks_per_seq: Optional[int] = None) -> None:
        if num_blocks <= 0 or block_size <= 0 or num_kv_heads <= 0 or head_dim <= 0:
            raise ValueError("PagedKVPool: sizes must be positive")
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise RuntimeError("PagedKVPool lives in GPU memory; a CUDA device is required")
        _lib.lib()  # fail loudly now if the CUDA library is missing
        self.num_blocks = int(num_blocks)
        self.block_size = int(block_size)
        self.num_kv_heads = int(num_kv_heads)
        self.head_dim = int(head_dim)
        self.num_layers = int(num_layers)
        self.dtype = dtype
        self.max_seqs = int(max_seqs)
        width = max_blocks_per_seq if max_blocks_per_seq is not None else min(num_blocks, 8192)
        self.max_blocks_per_seq = int(width)
        shape = (self.num_layers, self.num_blocks, self.block_size, self.num_kv_heads, self.head_dim)
        dev = self.device
        self.k = torch.zeros(shape, dtype=dtype, device=dev)
        self.v = torch.zeros(shape, dtype=dtype, device=dev)
        self.free_stack = torch.arange(self.num_blocks, dtype=torch.int32, device=dev)
        self.free_top = torch.tensor([self.num_blocks], dtype=torch.int32, device=dev)
        self.tables = torch.full((self.max_seqs, self.max_blocks_per_seq), -1, dtype=torch.int32, device=dev)
        self.table_len = torch.zeros(self.max_seqs, dtype=torch.int32, device=dev)
        self.status = torch.zeros(1, dtype=torch.int32, device=dev)
        # host mirror: counters only
        self.free_count = self.num_blocks
        self.row_blocks = [0] * self.max_seqs
        self._free_rows = list(range(self.max_seqs - 1, -1, -1))
        self._workspace: Optional[torch.Tensor] = None

    def shuffle_free_stack(self, seed: int) -> None:
        """Permute the initial free stack (a workload knob: random,
        non-contiguous block tables).  Only valid while no block is in use."""
        if self.free_count != self.num_blocks:
            raise RuntimeError("shuffle_free_stack: blocks are in use")
        g = torch.Generator().manual_seed(seed)
        perm = torch.randperm(self.num_blocks, generator=g).to(torch.int32)
        self.free_stack.copy_(perm.to(self.device))

    # ------------------------------------------------------------ rows
    def acquire_row(self) -> int:
        if not self._free_rows:
            raise RuntimeError(f"PagedKVPool: more than max_seqs={self.max_seqs} live sequences")
        return self._free_rows.pop()

    def release_row(self, row: int) -> None:
        self.release([row])
        self._free_rows.append(row)

    # ------------------------------------------------------------ allocator
    def blocks_for(self, tokens: int) -> int:
        return 0 if tokens <= 0 else -(-tokens // self.block_size)

    def demand(self, rows: Sequence[int], targets: Sequence[int]) -> int:
        need = 0
        for r, t in zip(rows, targets):
            want = self.blocks_for(t)
            if want > self.max_blocks_per_seq:
                raise RuntimeError(
                    f"sequence needs {want} blocks > max_blocks_per_seq={self.max_blocks_per_seq}")
            need += max(0, want - self.row_blocks[r])
        return need

    def reserve(self, rows: Sequence[int], targets: Sequence[int], oom_message: str = "OOM: Not enough blocks") -> int:
        """Grow each row to hold ``targets[i]`` tokens (item order = pop order)."""
        if len(set(rows)) != len(rows):
            raise ValueError("reserve: duplicate rows in one batch")
        need = self.demand(rows, targets)
        if need > self.free_count:
            raise RuntimeError(oom_message)
        if need == 0:
            return 0
        self.commit_reserve(rows, targets, need, to_device_i32(rows, self.device),
                            to_device_i32(targets, self.device))
        return need

    def commit_reserve(self, rows: Sequence[int], targets: Sequence[int], need: int,
                       rows_d: torch.Tensor, targets_d: torch.Tensor) -> None:
        """The reserve kernel for a batch already checked with ``demand`` (``need``
        blocks, at most ``free_count``), reading rows and targets from device
        int32 tensors the caller staged; then the host counters."""
        _lib.block_reserve(self.free_stack, self.free_top, self.tables, self.table_len, rows_d,
                           targets_d, self.block_size, self.status)
        for r, t in zip(rows, targets):
            self.row_blocks[r] = max(self.row_blocks[r], self.blocks_for(t))
        self.free_count -= need

    def release(self, rows: Sequence[int]) -> None:
        rows = [r for r in rows if self.row_blocks[r] > 0]
        if not rows:
            return
        if len(set(rows)) != len(rows):
            raise ValueError("release: duplicate rows in one batch")
        rd = to_device_i32(rows, self.device)
        _lib.block_free(self.free_stack, self.free_top, self.tables, self.table_len, rd, self.status)
        for r in rows:
            self.free_count += self.row_blocks[r]
            self.row_blocks[r] = 0

    def slots(self, rows_d: torch.Tensor, positions_d: torch.Tensor, offsets_d: torch.Tensor,
              n_tokens: int) -> torch.Tensor:
        out = torch.empty(n_tokens, dtype=torch.int64, device=self.device)
        _lib.compute_slots(self.tables, rows_d, positions_d, offsets_d, self.block_size,
                           self.num_blocks, out, self.status)
        return out

    # ------------------------------------------------------------ data path
    def append(self, layer: int, k_new: torch.Tensor, v_new: torch.Tensor, slots: torch.Tensor) -> None:
        _lib.kv_append(self.k[layer], self.v[layer], k_new, v_new, slots, self.status)

    def workspace(self, nbytes: int) -> Optional[torch.Tensor]:
        """A reusable device workspace of at least ``nbytes`` (grown, never shrunk)."""
        if nbytes <= 0:
            return None
        if self._workspace is None or self._workspace.numel() < nbytes:
            self._workspace = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=self.device)
        return self._workspace

    def decode(self, layer: int, q: torch.Tensor, query_start_loc: torch.Tensor, ctx_lens: torch.Tensor,
               seq_rows: Optional[torch.Tensor], max_q: int, max_ctx: int, score_scale: float,
               out: Optional[torch.Tensor] = None, partition_tokens: int = 0) -> torch.Tensor:
        if out is None:
            out = torch.empty_like(q)
        n_seqs = query_start_loc.numel() - 1
        nbytes = _lib.decode_workspace_bytes(n_seqs, q.shape[0], max_q, max_ctx, q.shape[1],
                                             self.num_kv_heads, self.head_dim, self.block_size,
                                             self.dtype, q.dtype, partition_tokens)
        _lib.paged_decode(out, q, self.k[layer], self.v[layer], self.tables, query_start_loc,
                          ctx_lens, max_queries_per_seq=max_q, max_ctx_len=max_ctx,
                          score_scale=score_scale, seq_rows=seq_rows,
                          partition_tokens=partition_tokens, workspace=self.workspace(nbytes),
                          status=self.status)
        return out

    def decode_step(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                    query_start_loc: torch.Tensor, ctx_lens: torch.Tensor,
                    seq_rows: Optional[torch.Tensor], max_q: int, max_ctx: int, score_scale: float,
                    out: Optional[torch.Tensor] = None, partition_tokens: int = 0,
                    check: bool = True) -> torch.Tensor:
        """Append every query row's new token at ctx - 1 and attend (one fused
        launch for a plain decode step).  Capacity must be reserved first."""
        if out is None:
            out = torch.empty_like(q)
        n_seqs = query_start_loc.numel() - 1
        nbytes = _lib.decode_workspace_bytes(n_seqs, q.shape[0], max_q, max_ctx, q.shape[1],
                                             self.num_kv_heads, self.head_dim, self.block_size,
                                             self.dtype, q.dtype, partition_tokens)
        _lib.decode_step(out, q, self.k[layer], self.v[layer], k_new, v_new, self.tables,
                         query_start_loc, ctx_lens, max_queries_per_seq=max_q, max_ctx_len=max_ctx,
                         score_scale=score_scale, seq_rows=seq_rows,
                         partition_tokens=partition_tokens, workspace=self.workspace(nbytes),
                         status=self.status, check=check)
        return out

    def decode_step_gather(self, layer: int, q: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor,
                           query_start_loc: torch.Tensor, ctx_lens: torch.Tensor,
                           seq_rows: Optional[torch.Tensor], max_q: int, max_ctx: int,
                           score_scale: float, gather, partition_tokens: int = 0,
                           out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """decode_step for a head-sharded group: the all-gathered output of
        every rank lands in ``out`` ([rows, Hq_total, D] view of a consumer
        buffer, any f32/f16/bf16) or in ``gather.out`` (returned view, valid
        until the next call)."""
        n_seqs = query_start_loc.numel() - 1
        nbytes = _lib.decode_gather_workspace_bytes(n_seqs, q.shape[0], max_q, max_ctx, q.shape[1],
                                                    self.num_kv_heads, self.head_dim,
                                                    self.block_size, self.dtype, q.dtype,
                                                    partition_tokens)
        _lib.decode_step_gather(q, self.k[layer], self.v[layer], k_new, v_new, self.tables,
                                query_start_loc, ctx_lens, gather, max_queries_per_seq=max_q,
                                max_ctx_len=max_ctx, score_scale=score_scale, seq_rows=seq_rows,
                                partition_tokens=partition_tokens, workspace=self.workspace(nbytes),
                                status=self.status, out=out)
        return gather.out[:q.shape[0]] if out is None else out

    # ------------------------------------------------------------ checks / views
    def check_status(self) -> None:
        """Raise if any kernel flagged a bad index since the last check (syncs)."""
        code = int(self.status.item())
        if code:
            self.status.zero_()
            self.raise_status(code)

    @staticmethod
    def raise_status(code: int) -> None:
        """Raise the RuntimeError that names the CLOVER_B200_DEV_* bits of ``code``."""
        names = [n for n, bit in [("bad slot", _lib.DEV_BAD_SLOT), ("bad block id", _lib.DEV_BAD_BLOCK),
                                  ("table full", _lib.DEV_TABLE_FULL), ("out of blocks", _lib.DEV_OOM),
                                  ("wait timeout", _lib.DEV_TIMEOUT), ("context > max_ctx_len", _lib.DEV_CTX_RANGE)]
                 if code & bit]
        raise RuntimeError(f"libclover_b200 device status 0x{code:x}: {', '.join(names)}")

    def row_table(self, row: int) -> List[int]:
        n = self.row_blocks[row]
        return self.tables[row, :n].tolist() if n else []

    def free_list(self) -> List[int]:
        top = int(self.free_top.item())
        return self.free_stack[:top].tolist()


class KVCacheManager:
    """Drop-in for CloverInfer's ``KVCacheManager`` (src/core/memory_manager.py:18-239)
    with the block pool, free stack and block tables in GPU memory and the
    paged attention on the sm_100a kernel.

    Differences, all deliberate: ``attention`` computes in fp32 and returns
    q's dtype (the upstream CUDA op accumulated the output in fp16,
    attention.cu:101-106); bf16 is supported; there is no CPU path — the
    manager requires a CUDA device.
    """

    def __init__(self, num_blocks: int, block_size: int, num_heads: int, head_dim: int,
                 dtype=torch.float32, device="cuda", max_seqs: int = 256,
                 max_blocks_per_seq: Optional[int] = None) -> None:
        self.num_blocks = num_blocks
        self.block_size = block_size
        self.num_heads = num_heads
        self.head_dim = head_dim
        self.dtype = dtype
        self.device = device
        self.pool = PagedKVPool(num_blocks, block_size, num_heads, head_dim, num_layers=1,
                                dtype=dtype, device=device, max_seqs=max_seqs,
                                max_blocks_per_seq=max_blocks_per_seq)
        self.k_cache = self.pool.k[0]
        self.v_cache = self.pool.v[0]
        self.context_lens: Dict[str, int] = {}
        self._rows: Dict[str, int] = {}

    # memory_manager.py:55-72
    def allocate(self, request_id: str, seq_len: int = 0) -> None:
        if request_id in self._rows:
            raise ValueError(f"Request {request_id} already exists")
        row = self.pool.acquire_row()
        try:
            self.pool.reserve([row], [max(seq_len + 1, 1)], "OOM: Not enough blocks")
        except Exception:
            self.pool._free_rows.append(row)
            raise
        self._rows[request_id] = row
        self.context_lens[request_id] = seq_len

    # memory_manager.py:74-93
    def load_initial_kv(self, request_id: str, k_data: torch.Tensor, v_data: torch.Tensor) -> None:
        n = int(k_data.shape[0])
        if request_id not in self._rows:
            self.allocate(request_id, n)
        row = self._rows[request_id]
        if n > 0:
            dev = self.pool.device
            rd = to_device_i32([row], dev)
            pd = to_device_i32([0], dev)
            od = to_device_i32([0, n], dev)
            slots = self.pool.slots(rd, pd, od, n)
            k = k_data.to(device=dev, dtype=self.dtype).contiguous()
            v = v_data.to(device=dev, dtype=self.dtype).contiguous()
            self.pool.append(0, k, v, slots)
        self.context_lens[request_id] = n

    # memory_manager.py:95-121
    def _grow_for_append(self, request_id: str) -> int:
        cur = self.context_lens[request_id]
        row = self._rows[request_id]
        self.pool.reserve([row], [cur + 1], "OOM during append")
        self.context_lens[request_id] = cur + 1
        return cur

    def append_slot(self, request_id: str) -> Tuple[int, int]:
        pos = self._grow_for_append(request_id)
        blk = int(self.pool.tables[self._rows[request_id], pos // self.block_size].item())
        return blk, pos % self.block_size

    # memory_manager.py:123-132
    def write_new_kv(self, request_id: str, k: torch.Tensor, v: torch.Tensor) -> None:
        k = k.squeeze(0) if k.dim() == 3 else k
        v = v.squeeze(0) if v.dim() == 3 else v
        pos = self._grow_for_append(request_id)
        dev = self.pool.device
        row = self._rows[request_id]
        slots = self.pool.slots(to_device_i32([row], dev), to_device_i32([pos], dev),
                                to_device_i32([0, 1], dev), 1)
        self.pool.append(0, k.to(device=dev, dtype=self.dtype).reshape(1, self.num_heads, self.head_dim).contiguous(),
                         v.to(device=dev, dtype=self.dtype).reshape(1, self.num_heads, self.head_dim).contiguous(),
                         slots)

    # memory_manager.py:134-143
    def free(self, request_id: str) -> None:
        if request_id not in self._rows:
            return
        row = self._rows.pop(request_id)
        self.pool.release_row(row)
        del self.context_lens[request_id]

    @property
    def block_tables(self) -> Dict[str, List[int]]:
        return {rid: self.pool.row_table(row) for rid, row in self._rows.items()}

    @property
    def free_blocks(self) -> List[int]:
        return self.pool.free_list()

    # memory_manager.py:145-173
    def get_kernel_inputs(self, request_ids: List[str]):
        rows = [self._rows[r] for r in request_ids]
        width = max((self.pool.row_blocks[r] for r in rows), default=0)
        idx = torch.tensor(rows, dtype=torch.long, device=self.pool.device)
        tables = self.pool.tables.index_select(0, idx)[:, :width].contiguous()
        lens = [self.context_lens[r] for r in request_ids]
        return tables, torch.tensor(lens, dtype=torch.int32, device=self.pool.device), max(lens, default=0)

    # memory_manager.py:175-190 (scale fixed at 1/sqrt(D), memory_manager.py:199)
    def attention(self, q: torch.Tensor, request_ids: List[str]) -> torch.Tensor:
        dev = self.pool.device
        qd = q.to(dev)
        if qd.dtype not in (torch.float32, self.dtype):
            qd = qd.to(torch.float32)
        qd = qd.contiguous()
        n = len(request_ids)
        lens = [self.context_lens[r] for r in request_ids]
        rows = to_device_i32([self._rows[r] for r in request_ids], dev)
        qsl = to_device_i32(list(range(n + 1)), dev)
        ctx = to_device_i32(lens, dev)
        out = self.pool.decode(0, qd, qsl, ctx, rows, 1, max(lens, default=0),
                               1.0 / math.sqrt(self.head_dim))
        return out.to(q.dtype) if out.dtype != q.dtype else out
