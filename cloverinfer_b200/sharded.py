"""Head-sharded multi-GPU attention: one process per GPU, KV heads split.

Rank ``r`` of ``world`` owns the KV heads ``kv_head_shards(Hkv, world)[r]``
(balanced contiguous ranges, identity placement — the upstream head-grouping
split, src/core/attention_backend.py:429-438, :400) and the query heads of
those groups.  Every rank replays the same allocator operations, so block
tables are identical everywhere with no communication.  The only exchange is
one all-gather of the per-rank attention outputs ``[T, Hq_local, D]`` into the
``[T, Hq, D]`` the dense node consumes (src/core/scheduler.py:1058-1059).
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
