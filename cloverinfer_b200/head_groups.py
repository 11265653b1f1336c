"""Head-grouping policy: how attention heads are split into groups and placed.

Restates the upstream policy (src/core/attention_backend.py:320-471,
docs/head_grouping_policy_universal.md) as pure functions, so the same rule
that split heads across PIM devices splits KV heads across B200 ranks:

* ``effective_group_count``  — ``_effective_head_group_count`` (:320-381),
  policies ``legacy | balanced | coarse | segment_aware | universal``;
* ``group_ranges``           — the contiguous ranges of ``_build_head_groups``
  (:413-438): ``legacy`` uses ceil-sized groups, every other policy balanced
  groups where the first ``num_heads % n`` groups take one extra head;
* ``placement_rotation`` / ``place_group`` — ``dpu_rotation`` (:417-418) and
  ``_choose_group_physical_dpu`` (:383-400), placements
  ``identity | rotated | rank_spread``.

``kv_head_shards`` is the multi-GPU use: balanced ranges over ``world`` ranks
with identity placement, i.e. rank ``r`` owns the ``r``-th range.  Identity
placement is required there because the output all-gather assumes a fixed
rank -> head map.
"""

from __future__ import annotations

import math
from typing import List, Tuple

POLICIES = ("legacy", "balanced", "coarse", "segment_aware", "universal")
PLACEMENTS = ("identity", "rotated", "rank_spread")


def effective_group_count(policy: str, seq_len: int, num_heads: int, head_dim: int,
                          num_devices: int) -> int:
    """Number of head groups a layer is split into (attention_backend.py:320-381)."""
    cap = max(1, min(num_devices, num_heads))
    if cap <= 1:
        return 1
    if policy == "coarse":
        return max(1, min(cap, max(1, math.ceil(num_heads / 32))))
    if policy == "segment_aware":
        per_group = 4 if seq_len >= 192 else 2
        return max(1, min(cap, max(1, math.ceil(num_heads / per_group))))
    if policy == "universal":
        by_shape = max(1, math.ceil(num_heads / 32))
        work = max(1, seq_len * head_dim)
        if work <= 4_096:
            per_group = 16
        elif work <= 16_384:
            per_group = 8
        elif work <= 65_536:
            per_group = 4
        else:
            per_group = 2
        by_heads = max(1, math.ceil(num_heads / per_group))
        return max(1, min(cap, max(by_shape, by_heads)))
    # "legacy" and "balanced" share the work-based count.
    work = max(1, seq_len * head_dim)
    if work <= 8_192:
        min_per_group = 4
    elif work <= 32_768:
        min_per_group = 2
    else:
        min_per_group = 1
    by_heads = max(1, math.ceil(num_heads / min_per_group))
    by_work = max(1, math.ceil(work * num_heads / 32_768))
    return max(1, min(cap, by_heads, by_work))


def group_ranges(policy: str, num_heads: int, num_groups: int) -> List[Tuple[int, int]]:
    """Contiguous [start, end) head ranges (attention_backend.py:421-438)."""
    if num_heads <= 0:
        raise ValueError("no attention heads")
    out: List[Tuple[int, int]] = []
    if policy == "legacy":
        size = math.ceil(num_heads / num_groups)
        for g in range(num_groups):
            lo, hi = g * size, min(num_heads, g * size + size)
            if lo >= hi:
                break
            out.append((lo, hi))
        return out
    base, extra = divmod(num_heads, num_groups)
    lo = 0
    for g in range(num_groups):
        hi = min(num_heads, lo + base + (1 if g < extra else 0))
        if lo >= hi:
            break
        out.append((lo, hi))
        lo = hi
    return out


def placement_rotation(request_id: str, layer_idx: int, num_devices: int) -> int:
    """``(sum(ord(c)) + layer) % n`` (attention_backend.py:417-418)."""
    return (sum(ord(c) for c in request_id) + int(layer_idx)) % max(num_devices, 1)


def place_group(placement: str, group_idx: int, num_groups: int, rotation: int,
                num_devices: int) -> int:
    """Physical device of a group (attention_backend.py:383-400)."""
    if num_devices <= 0:
        return 0
    if placement == "rotated":
        return (group_idx + rotation) % num_devices
    if placement == "rank_spread":
        stride = max(1, math.ceil(num_devices / max(1, num_groups)))
        return (rotation + group_idx * stride) % num_devices
    return group_idx % num_devices


def build_head_groups(policy: str, placement: str, request_id: str, layer_idx: int,
                      seq_len: int, num_heads: int, head_dim: int,
                      num_devices: int) -> List[Tuple[int, int, int]]:
    """(head_start, head_end, device) for every group of one layer."""
    n = effective_group_count(policy, seq_len, num_heads, head_dim, num_devices)
    rot = placement_rotation(request_id, layer_idx, num_devices)
    ranges = group_ranges(policy, num_heads, n)
    return [(lo, hi, place_group(placement, g, len(ranges), rot, num_devices))
            for g, (lo, hi) in enumerate(ranges)]


def kv_head_shards(num_kv_heads: int, world: int) -> List[Tuple[int, int]]:
    """KV-head range of every rank: balanced contiguous split, identity placement."""
    if world > num_kv_heads:
        raise ValueError(f"cannot shard {num_kv_heads} KV heads over {world} ranks")
    return group_ranges("balanced", num_kv_heads, world)


def select_kv_heads(x, kv_range: Tuple[int, int], num_kv_heads: int):
    """View of K or V [T, H, D] with KV heads [lo, hi) only.  H may be Hkv
    (native) or Hq = Hkv * g (repeat_kv-expanded, model_adapter.py:504-507:
    one head per group kept)."""
    h = x.shape[1]
    if h != num_kv_heads:
        if h % num_kv_heads:
            raise ValueError(f"K/V has {h} heads; expected {num_kv_heads} (or a multiple)")
        x = x[:, :: h // num_kv_heads]
    lo, hi = kv_range
    return x if (lo, hi) == (0, num_kv_heads) else x[:, lo:hi]


def local_inputs(query, key, value, kv_range: Tuple[int, int], num_kv_heads: int):
    """A sharded rank's part of a step's inputs, as views: the query heads of
    KV heads [lo, hi) (each KV head's GQA group is contiguous in query
    [T, Hq, D]) and those KV heads of key/value."""
    hq = query.shape[1]
    if hq % num_kv_heads:
        raise ValueError(f"{hq} query heads do not fit {num_kv_heads} KV heads")
    g = hq // num_kv_heads
    lo, hi = kv_range
    q = query if (lo, hi) == (0, num_kv_heads) else query[:, lo * g:hi * g]
    return q, select_kv_heads(key, kv_range, num_kv_heads), select_kv_heads(value, kv_range, num_kv_heads)
