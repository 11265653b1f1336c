"""Head-grouping policy == the upstream policy on its own recorded outputs
(tests/golden/head_groups.json, generated from src/core/attention_backend.py:320-471)."""

from __future__ import annotations

import json
import os

import pytest

from conftest import GOLDEN
from cloverinfer_b200.head_groups import (build_head_groups, effective_group_count,
                                          group_ranges, kv_head_shards)


@pytest.fixture(scope="module")
def golden():
    with open(os.path.join(GOLDEN, "head_groups.json")) as f:
        return json.load(f)


def test_group_counts(golden):
    for policy, ndev, heads, seq, hd, n in golden["counts"]:
        assert effective_group_count(policy, seq, heads, hd, ndev) == n, (policy, ndev, heads, seq, hd)


def test_build_head_groups(golden):
    for policy, placement, ndev, heads, seq, hd, n, ranges, dpus in golden["build"]:
        got = build_head_groups(policy, placement, "req-xyz", 3, seq, heads, hd, ndev)
        assert [[lo, hi] for lo, hi, _ in got] == ranges, (policy, ndev, heads, seq)
        assert [d for _, _, d in got] == dpus, (policy, placement, ndev, heads, seq)
        assert len(got) <= n


def test_kv_head_shards():
    assert kv_head_shards(8, 1) == [(0, 8)]
    assert kv_head_shards(8, 2) == [(0, 4), (4, 8)]
    assert kv_head_shards(8, 8) == [(i, i + 1) for i in range(8)]
    assert kv_head_shards(7, 3) == [(0, 3), (3, 5), (5, 7)]  # earlier groups take the extra head
    with pytest.raises(ValueError):
        kv_head_shards(4, 8)
    assert group_ranges("legacy", 7, 3) == [(0, 3), (3, 6), (6, 7)]
