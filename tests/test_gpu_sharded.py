"""Head-sharded decode on 2 GPUs (skipped with fewer): the fused peer-store
gather (clover_b200_decode_step_gather) and the NCCL gather both return, on
every rank, the same [rows, Hq, D] as a single GPU holding every KV head.
Ranks run as spawned processes with NCCL (NVLS off) and short timeouts."""

from __future__ import annotations

import datetime
import math
import os
import socket

import pytest
import torch

from conftest import gpu

pytestmark = gpu


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _problem(device, seed=0):
    g = torch.Generator().manual_seed(seed)
    B, hq, hkv, D, bs = 4, 32, 8, 128, 16
    lens = [3000, 777, 4096, 65]
    nblk = [-(-(n + 1) // bs) for n in lens]
    nb = sum(nblk) + 8
    kc = torch.randn(nb, bs, hkv, D, generator=g).bfloat16()
    vc = torch.randn(nb, bs, hkv, D, generator=g).bfloat16()
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    tables = torch.full((B, max(nblk)), -1, dtype=torch.int32)
    o = 0
    for i, k in enumerate(nblk):
        tables[i, :k] = perm[o:o + k]
        o += k
    q = torch.randn(B, hq, D, generator=g).bfloat16().float()
    kn = torch.randn(B, hkv, D, generator=g).bfloat16()
    vn = torch.randn(B, hkv, D, generator=g).bfloat16()
    return dict(kc=kc, vc=vc, tables=tables, q=q, kn=kn, vn=vn, lens=lens, hq=hq, hkv=hkv, D=D, bs=bs)


def _worker(rank, world, port, q_out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=60))
    peer = None
    try:
        from cloverinfer_b200 import _lib
        from cloverinfer_b200.head_groups import kv_head_shards
        from cloverinfer_b200.sharded import HeadShardGroup, PeerGather
        P = _problem(dev)
        B, hq, hkv, D, bs, lens = len(P["lens"]), P["hq"], P["hkv"], P["D"], P["bs"], P["lens"]
        grp = hq // hkv
        ctx = torch.tensor([n + 1 for n in lens], dtype=torch.int32, device=dev)
        qsl = torch.arange(B + 1, dtype=torch.int32, device=dev)
        tables = P["tables"].to(dev)
        st = torch.zeros(1, dtype=torch.int32, device=dev)
        # single-GPU reference on this rank: every head, fused append
        kc, vc = P["kc"].to(dev), P["vc"].to(dev)
        ref = torch.empty(B, hq, D, device=dev)
        nbytes = _lib.decode_workspace_bytes(B, B, 1, max(lens) + 1, hq, hkv, D, bs, torch.bfloat16, torch.float32)
        ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
        _lib.decode_step(ref, P["q"].to(dev), kc, vc, P["kn"].to(dev), P["vn"].to(dev), tables, qsl, ctx,
                         max_queries_per_seq=1, max_ctx_len=max(lens) + 1, score_scale=1 / math.sqrt(D),
                         workspace=ws, status=st)
        # sharded: this rank's KV heads only
        sg = HeadShardGroup()
        lo, hi = sg.kv_range(hkv)
        kcl = P["kc"][:, :, lo:hi].contiguous().to(dev)
        vcl = P["vc"][:, :, lo:hi].contiguous().to(dev)
        ql = P["q"][:, lo * grp:hi * grp].contiguous().to(dev)
        knl = P["kn"][:, lo:hi].contiguous().to(dev)
        vnl = P["vn"][:, lo:hi].contiguous().to(dev)
        peer = PeerGather(sg, B, hq, D, torch.float32, dev)
        nb2 = _lib.decode_gather_workspace_bytes(B, B, 1, max(lens) + 1, ql.shape[1], hi - lo, D, bs,
                                                 torch.bfloat16, torch.float32)
        ws2 = torch.empty(max(nb2, 1), dtype=torch.uint8, device=dev)
        errs = []
        for call in range(3):  # three calls: both halves of the double buffer
            _lib.decode_step_gather(ql, kcl, vcl, knl, vnl, tables, qsl, ctx, peer,
                                    max_queries_per_seq=1, max_ctx_len=max(lens) + 1,
                                    score_scale=1 / math.sqrt(D), workspace=ws2, status=st)
            torch.cuda.synchronize(dev)
            errs.append(float((peer.out[:B] - ref).abs().max()))
        # NCCL gather of a plain local decode
        outl = torch.empty_like(ql)
        nb3 = _lib.decode_workspace_bytes(B, B, 1, max(lens) + 1, ql.shape[1], hi - lo, D, bs,
                                          torch.bfloat16, torch.float32)
        ws3 = torch.empty(max(nb3, 1), dtype=torch.uint8, device=dev)
        _lib.paged_decode(outl, ql, kcl, vcl, tables, qsl, ctx, max_queries_per_seq=1,
                          max_ctx_len=max(lens) + 1, score_scale=1 / math.sqrt(D), workspace=ws3, status=st)
        nccl = sg.gather(outl, hkv, grp)
        torch.cuda.synchronize(dev)
        errs.append(float((nccl - ref).abs().max()))
        # the drop-in backend, sharded, through decode_layer_batch with host items
        from cloverinfer_b200 import B200AttentionBackend
        gen = torch.Generator().manual_seed(9)
        kv = {rid: [{"key": torch.randn(n, hkv, D, generator=gen).bfloat16(),
                     "value": torch.randn(n, hkv, D, generator=gen).bfloat16()} for _ in range(2)]
              for rid, n in [("a", 1200), ("b", 90)]}
        bes = [B200AttentionBackend(device=dev, num_blocks=256, num_kv_heads=hkv, max_seqs=4),
               B200AttentionBackend(device=dev, num_blocks=256, num_kv_heads=hkv, max_seqs=4,
                                    shard=sg, gather="peer")]
        for be in bes:
            for rid, layers in kv.items():
                be.init_request(rid, layers)
        # two steps of two layers: the first call of the batch shape runs eagerly,
        # later ones capture and replay the fused step as a CUDA graph
        for layer in [0, 1, 0, 1]:
            items = [{"request_id": rid, "layer_idx": layer, "score_scale": 1 / math.sqrt(D),
                      "query": torch.randn(hq, D, generator=gen),
                      "key": torch.randn(hkv, D, generator=gen).bfloat16(),
                      "value": torch.randn(hkv, D, generator=gen).bfloat16()} for rid in kv]
            o0 = bes[0].decode_layer_batch(items)
            o1 = bes[1].decode_layer_batch(items)
            errs.append(max(float((x - y).abs().max()) for x, y in zip(o0, o1)))
        assert bes[1]._peer is not None
        assert all(p.graphs for p in bes[1]._fast.values())  # the sharded step was captured
        # the fused gather straight into a bf16 consumer buffer (the o_proj input)
        qd = torch.randn(2, hq, D, generator=gen).bfloat16().float().to(dev)
        knd = torch.randn(2, hkv, D, generator=gen).bfloat16().to(dev)
        vnd = torch.randn(2, hkv, D, generator=gen).bfloat16().to(dev)
        consumer = torch.zeros(2, 1, hq * D, dtype=torch.bfloat16, device=dev)
        o_ref = bes[0].decode_batch(["a", "b"], 0, qd, knd, vnd, 1 / math.sqrt(D))
        o_sh = bes[1].decode_batch(["a", "b"], 0, qd, knd, vnd, 1 / math.sqrt(D), out=consumer)
        torch.cuda.synchronize(dev)
        assert o_sh.data_ptr() == consumer.data_ptr()
        # bf16 output: within half a bf16 ulp of the fp32 single-GPU result (+ the fp32 bound)
        dev_err = (consumer.view(2, hq, D).float() - o_ref).abs() - o_ref.abs() * 2.0 ** -8
        errs.append(max(0.0, float(dev_err.max())))
        bes[1].close()
        q_out.put((rank, int(st.item()), errs))
    except Exception as e:
        q_out.put((rank, -1, repr(e)))
    finally:
        if peer is not None:
            peer.close()
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sharded_gather_matches_single_gpu():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=240) for _ in procs), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=120)
    for rank, status, errs in res:
        assert status == 0, (rank, status, errs)
        assert all(e < 2e-5 for e in errs), (rank, errs)
