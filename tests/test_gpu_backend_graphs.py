"""The backend's captured fast path (CUDA graph per batch shape, layer, scale
and 512-token context bucket) against the eager path and the CPU oracle.

``decode_layer_batch`` with host tensors runs its first call for a batch
shape eagerly, then replays a captured graph (H2D of the staging buffer,
fused append + decode + reduce, D2H of output and status).  The steps here
cross a context bucket, so a graph is re-captured mid-run.
"""

from __future__ import annotations

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
