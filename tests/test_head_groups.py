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


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_local_inputs_partition_every_head(world):
    """Each rank's part of a step's inputs (what a sharded decode_batch copies
    from host memory): the query heads of its KV heads, and those KV heads of
    native or repeat_kv-expanded K/V; the parts cover every head once."""
    import torch
    from cloverinfer_b200.head_groups import kv_head_shards, local_inputs
    T, hkv, g, D = 5, 8, 4, 16
    q = torch.randn(T, hkv * g, D)
    k = torch.randn(T, hkv, D)
    v = torch.randn(T, hkv, D)
    k_exp = k.repeat_interleave(g, dim=1)  # repeat_kv: each KV head repeated g times in place
    qs, ks, vs = [], [], []
    for lo, hi in kv_head_shards(hkv, world):
        ql, kl, vl = local_inputs(q, k, v, (lo, hi), hkv)
        _, kx, vx = local_inputs(q, k_exp, v.repeat_interleave(g, dim=1), (lo, hi), hkv)
        assert ql.shape == (T, (hi - lo) * g, D) and kl.shape == (T, hi - lo, D)
        assert torch.equal(kx, kl) and torch.equal(vx, vl)
        assert ql.data_ptr() >= q.data_ptr()  # views, no copies
        qs.append(ql)
        ks.append(kl)
        vs.append(vl)
    assert torch.equal(torch.cat(qs, 1), q) and torch.equal(torch.cat(ks, 1), k)
    assert torch.equal(torch.cat(vs, 1), v)


def test_local_inputs_reject_bad_head_counts():
    import torch
    from cloverinfer_b200.head_groups import local_inputs
    with pytest.raises(ValueError):
        local_inputs(torch.zeros(1, 6, 4), torch.zeros(1, 4, 4), torch.zeros(1, 4, 4), (0, 4), 4)
    with pytest.raises(ValueError):
        local_inputs(torch.zeros(1, 8, 4), torch.zeros(1, 6, 4), torch.zeros(1, 6, 4), (0, 4), 4)
