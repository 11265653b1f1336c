"""cloverinfer_b200 — B200-native paged decode attention for CloverInfer.

A drop-in for the attention node's backend interface
(``CpuAttentionBackend``: src/core/attention_backend.py:56-144) and for the
``KVCacheManager`` paged block layout (src/core/memory_manager.py), computed by
hand-written sm_100a CUDA kernels in ``libclover_b200.so`` (C ABI:
``include/clover_b200.h``).  There is no CPU path: without a CUDA device or the
library, constructing a backend raises.
"""

from .backend import B200AttentionBackend  # noqa: F401
from .kv_cache import KVCacheManager, PagedKVPool  # noqa: F401
from .head_groups import (build_head_groups, effective_group_count, group_ranges,  # noqa: F401
                          kv_head_shards, place_group, placement_rotation)
from .sharded import HeadShardGroup  # noqa: F401
from ._lib import CloverB200Error, lib, lib_path  # noqa: F401

__all__ = [
    "B200AttentionBackend", "KVCacheManager", "PagedKVPool", "HeadShardGroup",
    "CloverB200Error", "build_head_groups", "effective_group_count", "group_ranges",
    "kv_head_shards", "place_group", "placement_rotation", "lib", "lib_path",
]
