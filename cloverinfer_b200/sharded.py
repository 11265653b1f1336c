"""Head-sharded multi-GPU attention: one process per GPU, KV heads split.

Rank ``r`` of ``world`` owns the KV heads ``kv_head_shards(Hkv, world)[r]``
(balanced contiguous ranges, identity placement — the upstream head-grouping
split, src/core/attention_backend.py:429-438, :400) and the query heads of
those groups.  Every rank replays the same allocator operations, so block
tables are identical everywhere with no communication.  The only exchange is
one all-gather of the per-rank attention outputs ``[T, Hq_local, D]`` into the
``[T, Hq, D]`` the dense node consumes (src/core/scheduler.py:1058-1059).

Two implementations of that gather:

* ``HeadShardGroup.gather`` — NCCL ``all_gather_into_tensor`` (any backend);
* ``PeerGather`` — fused into the split-K reduce kernel
  (``clover_b200_decode_step_gather``): each rank stores its rows straight into
  every rank's receive buffer over NVLink (CUDA IPC peer mappings) as
  epoch-tagged 8-byte words and waits, bounded, for every rank's words of its
  own rows: the exchange needs no fence, barrier or extra launch.
"""

from __future__ import annotations

from typing import List, Tuple

import torch
import torch.distributed as dist

from .head_groups import kv_head_shards


class HeadShardGroup:
    def __init__(self, process_group=None) -> None:
        if not dist.is_available() or not dist.is_initialized():
            raise RuntimeError("HeadShardGroup needs an initialised torch.distributed process group")
        self.pg = process_group
        self.rank = dist.get_rank(process_group)
        self.world = dist.get_world_size(process_group)
        self._bufs = {}

    def ranges(self, num_kv_heads: int) -> List[Tuple[int, int]]:
        return kv_head_shards(num_kv_heads, self.world)

    def kv_range(self, num_kv_heads: int) -> Tuple[int, int]:
        return self.ranges(num_kv_heads)[self.rank]

    def gather(self, out_local: torch.Tensor, num_kv_heads: int, group: int) -> torch.Tensor:
        """All-gather [T, Hq_local, D] from every rank into [T, Hq, D]."""
        if self.world == 1:
            return out_local
        ranges = self.ranges(num_kv_heads)
        widths = [(hi - lo) * group for lo, hi in ranges]
        wmax = max(widths)
        T, hl, D = out_local.shape
        send = out_local
        if hl != wmax:  # uneven split: pad to the widest shard
            send = torch.zeros((T, wmax, D), dtype=out_local.dtype, device=out_local.device)
            send[:, :hl] = out_local
        recv = torch.empty((self.world * T, wmax, D), dtype=out_local.dtype, device=out_local.device)
        dist.all_gather_into_tensor(recv, send.contiguous(), group=self.pg)
        recv = recv.view(self.world, T, wmax, D)
        if all(w == wmax for w in widths):
            return recv.permute(1, 0, 2, 3).reshape(T, self.world * wmax, D)
        return torch.cat([recv[r, :, :w] for r, w in enumerate(widths)], dim=1)


class PeerGather:
    """Buffers of the fused output gather (``clover_b200_decode_step_gather``)
    for one head-sharded group, one process per GPU.

    Every rank allocates a receive buffer of 2 x [max_rows, total_q_heads,
    head_dim] 8-byte words (CUDA IPC memory, zeroed), exchanges the IPC
    handles over the process group and maps every peer's; ``out`` is the
    local all-gathered output ``[max_rows, total_q_heads, head_dim]``.
    """

    def __init__(self, shard: "HeadShardGroup", max_rows: int, total_q_heads: int,
                 head_dim: int, dtype: torch.dtype, device) -> None:
        from . import _lib
        if total_q_heads % shard.world:
            raise ValueError("fused gather needs equal head shards")
        self.device = torch.device(device)
        self.world, self.rank = shard.world, shard.rank
        self.half_words = max_rows * total_q_heads * head_dim
        with torch.cuda.device(self.device):
            self.recv_ptr, handle = _lib.ipc_alloc(2 * self.half_words * 8)
        handles = [None] * self.world
        dist.all_gather_object(handles, handle, group=shard.pg)
        self._opened: List[int] = []
        ptrs = []
        with torch.cuda.device(self.device):
            for r, h in enumerate(handles):
                if r == self.rank:
                    ptrs.append(self.recv_ptr)
                else:
                    p = _lib.ipc_open(h)
                    self._opened.append(p)
                    ptrs.append(p)
        self.peer_recv_d = torch.tensor(ptrs, dtype=torch.int64, device=self.device)
        self.sync = torch.zeros(_lib.gather_sync_bytes() // 4, dtype=torch.int32, device=self.device)
        self.out = torch.zeros((max_rows, total_q_heads, head_dim), dtype=dtype, device=self.device)
        self._shard = shard
        dist.barrier(group=shard.pg)

    def close(self) -> None:
        """Unmap peers and free the own buffer (collective: every rank calls it)."""
        from . import _lib
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self._shard.pg)
        with torch.cuda.device(self.device):
            for p in self._opened:
                _lib.ipc_close(p)
            self._opened = []
        dist.barrier(group=self._shard.pg)
        if self.recv_ptr:
            with torch.cuda.device(self.device):
                _lib.ipc_free(self.recv_ptr)
            self.recv_ptr = 0
