"""The backend's captured fast path (CUDA graph per batch shape, layer, scale
and 512-token context bucket) against the eager path and the CPU oracle.

``decode_layer_batch`` with host tensors runs its first call for a batch
shape eagerly, then replays a captured graph (H2D of the staging buffer,
fused append + decode + reduce, D2H of output and status).  The steps here
cross a context bucket, so a graph is re-captured mid-run.
"""

from __future__ import annotations

import pytest
import torch

from conftest import assert_attn_close, gpu
from oracle import attend, repeat_kv

pytestmark = gpu


def _run(cuda_graphs: bool, steps: int = 24):
    from cloverinfer_b200 import B200AttentionBackend
    hq, hkv, D, L = 16, 4, 128, 2
    lens = [500, 505, 1019]  # 505 + 24 and 1019 + 24 cross a 512-token bucket
    be = B200AttentionBackend(num_blocks=256, block_size=16, num_kv_heads=hkv,
                              kv_dtype=torch.bfloat16, device="cuda", max_seqs=4,
                              shuffle_seed=3, cuda_graphs=cuda_graphs)
    g = torch.Generator().manual_seed(11)
    kv = {}
    for i, n in enumerate(lens):
        layers = [{"key": torch.randn(n, hkv, D, generator=g).bfloat16(),
                   "value": torch.randn(n, hkv, D, generator=g).bfloat16()} for _ in range(L)]
        be.init_request(f"s{i}", layers)
        kv[f"s{i}"] = layers
    outs = []
    for step in range(steps):
        for layer in range(L):
            items = [{"request_id": f"s{i}", "layer_idx": layer,
                      "query": torch.randn(1, hq, D, generator=g).pin_memory(),
                      "key": torch.randn(1, hkv, D, generator=g).bfloat16().pin_memory(),
                      "value": torch.randn(1, hkv, D, generator=g).bfloat16().pin_memory(),
                      "score_scale": 0.088} for i in range(len(lens))]
            res = be.decode_layer_batch(items)
            outs.append(torch.cat(res))
            for i, it in enumerate(items):
                lay = kv[f"s{i}"][layer]
                lay["key"] = torch.cat([lay["key"], it["key"][0:1].reshape(1, hkv, D)])
                lay["value"] = torch.cat([lay["value"], it["value"][0:1].reshape(1, hkv, D)])
            last = (items, res)
    n_graphs = sum(len(p.graphs) for p in be._fast.values())
    return outs, last, kv, n_graphs, be


def test_graph_path_matches_eager_and_oracle():
    eager, _, _, n0, _ = _run(False)
    graphed, (items, res), kv, n1, be = _run(True)
    assert n0 == 0 and n1 >= 2  # one graph per layer in the last bucket
    for a, b in zip(eager, graphed):
        assert float((a - b).abs().max()) < 2e-5
    for i, it in enumerate(items):
        lay = kv[f"s{i}"][it["layer_idx"]]
        ref = attend(it["query"][0].float(), repeat_kv(lay["key"], 4), repeat_kv(lay["value"], 4), 0.088)
        assert_attn_close(res[i][0], ref, what=f"seq {i}")
    assert be.get_context_len("s0") == 500 + 24


def test_plan_cache_is_bounded_and_stays_correct():
    """Continuous batching changes the batch size every step: only the most
    recent ``max_fast_plans`` shapes keep staging buffers and graphs."""
    from cloverinfer_b200 import B200AttentionBackend
    hq, hkv, D = 8, 2, 128
    be = B200AttentionBackend(num_blocks=128, block_size=16, num_kv_heads=hkv,
                              kv_dtype=torch.bfloat16, device="cuda", max_seqs=4,
                              max_fast_plans=2)
    g = torch.Generator().manual_seed(5)
    kv = {}
    for i, n in enumerate([30, 200, 64]):
        k = torch.randn(n, hkv, D, generator=g).bfloat16()
        v = torch.randn(n, hkv, D, generator=g).bfloat16()
        be.init_request(f"r{i}", [{"key": k, "value": v}])
        kv[f"r{i}"] = [k.float(), v.float()]
    for step, batch in enumerate([[0], [0, 1], [0, 1, 2], [0], [0, 1, 2], [0, 1, 2], [1]]):
        items = [{"request_id": f"r{i}", "layer_idx": 0, "score_scale": 0.09,
                  "query": torch.randn(hq, D, generator=g),
                  "key": torch.randn(hkv, D, generator=g).bfloat16(),
                  "value": torch.randn(hkv, D, generator=g).bfloat16()} for i in batch]
        res = be.decode_layer_batch(items)
        assert len(be._fast) <= 2
        for it, o in zip(items, res):
            k, v = kv[it["request_id"]]
            k = torch.cat([k, it["key"].float()[None]])
            v = torch.cat([v, it["value"].float()[None]])
            kv[it["request_id"]] = [k, v]
            ref = attend(it["query"], repeat_kv(k, hq // hkv), repeat_kv(v, hq // hkv), 0.09)
            assert_attn_close(o[0], ref, what=f"step {step} {it['request_id']}")


def test_mismatched_item_shapes_raise():
    """Items whose query/key shapes differ cannot share the fixed-size host
    gather: the call raises instead of reading past a smaller tensor."""
    from cloverinfer_b200 import B200AttentionBackend
    be = B200AttentionBackend(num_blocks=64, block_size=16, num_kv_heads=2,
                              kv_dtype=torch.bfloat16, device="cuda", max_seqs=4)
    for rid in ("a", "b"):
        be.init_request(rid, [{"key": torch.randn(20, 2, 64).bfloat16(),
                               "value": torch.randn(20, 2, 64).bfloat16()}])
    items = [{"request_id": "a", "layer_idx": 0, "query": torch.randn(8, 64),
              "key": torch.randn(2, 64).bfloat16(), "value": torch.randn(2, 64).bfloat16()},
             {"request_id": "b", "layer_idx": 0, "query": torch.randn(4, 64),
              "key": torch.randn(2, 64).bfloat16(), "value": torch.randn(2, 64).bfloat16()}]
    with pytest.raises(Exception):
        be.decode_layer_batch(items)
