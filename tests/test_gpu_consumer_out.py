"""Attention outputs written straight into the consumer's buffer.

The dense node reshapes the gathered contexts into its o_proj input
[rows, Hq * D] in the model's dtype (src/core/model_adapter.py:572, fed by
src/core/scheduler.py:1058-1059).  ``clover_b200_decode_step_gather_into``
writes the all-gathered output there directly, in a dtype of its own and with
any row stride; ``B200AttentionBackend.decode_batch(out=...)`` exposes it.
Checked against the CPU oracle (bf16 output: its half-ulp added to the
bound), with the padding of each consumer row left untouched.  The two-rank
fused gather into a consumer buffer is covered in test_gpu_sharded.py.
"""

from __future__ import annotations

import math
from types import SimpleNamespace

import torch

from conftest import assert_attn_close, gpu
from oracle import CpuAttentionOracle, repeat_kv
from test_gpu_gather_timeout import _oracle, _problem

pytestmark = gpu


def test_gather_into_padded_bf16_consumer_rows():
    from cloverinfer_b200 import _lib
    dev = torch.device("cuda")
    P = _problem(seed=31)
    B, hq_l, D = len(P["lens"]), P["hq_l"], P["D"]
    kc, vc, tables, q = (P[k].to(dev) for k in ("kc", "vc", "tables", "q"))
    qsl = torch.arange(B + 1, dtype=torch.int32, device=dev)
    ctx = torch.tensor(P["lens"], dtype=torch.int32, device=dev)
    half = B * hq_l * D
    recv = torch.zeros(2 * half, dtype=torch.int64, device=dev)
    sync = torch.zeros(_lib.gather_sync_bytes() // 4, dtype=torch.int32, device=dev)
    g1 = SimpleNamespace(world=1, rank=0, half_words=half, sync=sync,
                         peer_recv_d=torch.tensor([recv.data_ptr()], dtype=torch.int64, device=dev),
                         out=torch.zeros(B, hq_l, D, device=dev))
    nbytes = _lib.decode_gather_workspace_bytes(B, B, 1, max(P["lens"]), hq_l, P["hkv_l"], D,
                                                P["bs"], torch.bfloat16, torch.float32)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    pad = 64
    consumer = torch.full((B, 1, hq_l * D + pad), 7.0, dtype=torch.bfloat16, device=dev)
    view = consumer[:, 0, :hq_l * D].as_strided((B, hq_l, D), (hq_l * D + pad, D, 1))
    for _ in range(2):  # both parities of the receive buffer
        _lib.decode_step_gather(q, kc, vc, None, None, tables, qsl, ctx, g1, max_queries_per_seq=1,
                                max_ctx_len=max(P["lens"]), score_scale=1 / math.sqrt(D),
                                workspace=ws, status=st, out=view)
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        got = consumer[:, 0, :hq_l * D].reshape(B, hq_l, D).cpu()
        assert_attn_close(got, _oracle(P), kv_dtype=torch.bfloat16, out_dtype=torch.bfloat16,
                          what="gather into bf16 consumer rows")
        assert bool((consumer[:, 0, hq_l * D:] == 7.0).all()), "row padding must be untouched"


def test_backend_decode_batch_into_consumer_buffer():
    from cloverinfer_b200 import B200AttentionBackend
    g = torch.Generator().manual_seed(41)
    hq, hkv, D = 16, 4, 128
    be = B200AttentionBackend(device="cuda", num_blocks=128, block_size=16, num_kv_heads=hkv,
                              max_seqs=4)
    ref = CpuAttentionOracle()
    for rid, n in [("a", 300), ("b", 1500)]:
        k = torch.randn(n, hkv, D, generator=g).bfloat16()
        v = torch.randn(n, hkv, D, generator=g).bfloat16()
        be.init_request(rid, [{"key": k, "value": v}])
        ref.init_request(rid, [{"key": repeat_kv(k, hq // hkv), "value": repeat_kv(v, hq // hkv)}])
    q = torch.randn(2, hq, D, generator=g).bfloat16().float()
    kn = torch.randn(2, hkv, D, generator=g).bfloat16()
    vn = torch.randn(2, hkv, D, generator=g).bfloat16()
    consumer = torch.zeros(2, 1, hq * D, dtype=torch.bfloat16, device="cuda")  # o_proj input
    res = be.decode_batch(["a", "b"], 0, q.cuda(), kn.cuda(), vn.cuda(), 1 / math.sqrt(D), out=consumer)
    assert res.data_ptr() == consumer.data_ptr() and tuple(res.shape) == (2, hq, D)
    want = torch.stack([ref.decode_layer(r, 0, q[i], repeat_kv(kn[i:i + 1], hq // hkv)[0],
                                         repeat_kv(vn[i:i + 1], hq // hkv)[0], 1 / math.sqrt(D))[0]
                        for i, r in enumerate(["a", "b"])])
    assert_attn_close(consumer.view(2, hq, D).cpu(), want, kv_dtype=torch.bfloat16,
                      out_dtype=torch.bfloat16, what="decode_batch into o_proj input")
    be.pool.check_status()
