"""The fused gather's bounded wait gives up cleanly, on one GPU.

``clover_b200_decode_step_gather`` stores every output value into every rank's
receive buffer and then waits, bounded, for the other ranks' words.  Here a
two-rank call is made by one process on one GPU whose "rank 1" buffer is a
second local buffer that no kernel ever fills for rank 0: the words rank 0
waits for never arrive (a flag that nothing sets), so the wait runs out after
the limit set with ``clover_b200_set_wait_limit_ns``.

Checked: the call returns (the host sees the device status word) with
``CLOVER_B200_DEV_TIMEOUT`` set well inside the default 1 s; rank 1's heads read
0; rank 0's own heads still match the CPU oracle; the pool's status check turns
the bit into the ``RuntimeError`` that AttentionNode surfaces to its callers
(src/core/nodes.py:167-170); and once the caller clears the word, the next
call on the same stream, sync words and buffers runs clean.
"""

from __future__ import annotations

import math
import time
from types import SimpleNamespace

import pytest
import torch

from conftest import assert_attn_close, gpu
from oracle import attend, repeat_kv

pytestmark = gpu


def _problem(seed=11):
    g = torch.Generator().manual_seed(seed)
    hq_l, hkv_l, D, bs = 4, 1, 128, 16
    lens = [700, 33, 2000]
    nblk = [-(-n // bs) for n in lens]
    nb = sum(nblk) + 4
    kc = torch.randn(nb, bs, hkv_l, D, generator=g).bfloat16()
    vc = torch.randn(nb, bs, hkv_l, D, generator=g).bfloat16()
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    tables = torch.full((len(lens), max(nblk)), -1, dtype=torch.int32)
    o = 0
    for i, k in enumerate(nblk):
        tables[i, :k] = perm[o:o + k]
        o += k
    q = torch.randn(len(lens), hq_l, D, generator=g).bfloat16().float()
    return dict(kc=kc, vc=vc, tables=tables, q=q, lens=lens, hq_l=hq_l, hkv_l=hkv_l, D=D, bs=bs)


def _oracle(P):
    """[B, hq_l, D] from oracle.attend over each sequence's blocks."""
    bs, D = P["bs"], P["D"]
    outs = []
    for i, n in enumerate(P["lens"]):
        blocks = P["tables"][i, :-(-n // bs)].long()
        k = P["kc"][blocks].reshape(-1, P["hkv_l"], D)[:n]
        v = P["vc"][blocks].reshape(-1, P["hkv_l"], D)[:n]
        grp = P["hq_l"] // P["hkv_l"]
        outs.append(attend(P["q"][i], repeat_kv(k, grp), repeat_kv(v, grp), 1 / math.sqrt(D),
                           out_dtype=torch.float32))
    return torch.stack(outs)


def _gather(world, recv, sync, B, heads_local, D, dev):
    """A stand-in for sharded.PeerGather whose 'ranks' all live on this GPU."""
    half = B * world * heads_local * D
    return SimpleNamespace(world=world, rank=0, half_words=half, sync=sync,
                           peer_recv_d=torch.tensor([t.data_ptr() for t in recv], dtype=torch.int64,
                                                    device=dev),
                           out=torch.full((B, world * heads_local, D), float("nan"), device=dev))


def test_gather_wait_times_out_and_the_next_call_runs_clean():
    from cloverinfer_b200 import _lib
    from cloverinfer_b200.kv_cache import PagedKVPool

    dev = torch.device("cuda")
    P = _problem()
    B, hq_l, D = len(P["lens"]), P["hq_l"], P["D"]
    kc, vc, tables, q = (P[k].to(dev) for k in ("kc", "vc", "tables", "q"))
    qsl = torch.arange(B + 1, dtype=torch.int32, device=dev)
    ctx = torch.tensor(P["lens"], dtype=torch.int32, device=dev)
    ref = _oracle(P)

    # rank 0's receive buffer, and a second local one standing in for rank 1's
    half = B * 2 * hq_l * D
    recv = [torch.zeros(2 * half, dtype=torch.int64, device=dev) for _ in range(2)]
    sync = torch.zeros(_lib.gather_sync_bytes() // 4, dtype=torch.int32, device=dev)
    common = dict(max_queries_per_seq=1, max_ctx_len=max(P["lens"]), score_scale=1 / math.sqrt(D))
    nbytes = _lib.decode_gather_workspace_bytes(B, B, 1, max(P["lens"]), hq_l, P["hkv_l"], D,
                                                P["bs"], torch.bfloat16, torch.float32)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)

    g2 = _gather(2, recv, sync, B, hq_l, D, dev)
    limit_ns = 20_000_000  # 20 ms
    prev = _lib.set_wait_limit_ns(limit_ns)
    try:
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        _lib.decode_step_gather(q, kc, vc, None, None, tables, qsl, ctx, g2, workspace=ws, status=st,
                                **common)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        _lib.set_wait_limit_ns(prev)
    code = int(st.item())
    assert code & _lib.DEV_TIMEOUT, f"status 0x{code:x}"
    assert code == _lib.DEV_TIMEOUT, f"only the timeout bit: 0x{code:x}"
    assert elapsed < 0.5, f"the 20 ms limit was not honoured ({elapsed:.3f} s)"
    out = g2.out[:B].cpu()
    assert bool((out[:, hq_l:] == 0).all()), "missing rank's heads must read 0"
    assert_attn_close(out[:, :hq_l], ref, kv_dtype=torch.bfloat16, what="own heads after timeout")

    # The pool's status check raises on the bit (and clears the word).
    pool = SimpleNamespace(status=st, raise_status=PagedKVPool.raise_status)
    with pytest.raises(RuntimeError, match="wait timeout"):
        PagedKVPool.check_status(pool)
    assert int(st.item()) == 0

    # The next call on the same stream, sync words and buffers runs clean.
    g1 = _gather(1, recv[:1], sync, B, hq_l, D, dev)
    for _ in range(2):  # both parities of the receive buffer
        _lib.decode_step_gather(q, kc, vc, None, None, tables, qsl, ctx, g1, workspace=ws, status=st,
                                **common)
        torch.cuda.synchronize()
        assert int(st.item()) == 0
        assert_attn_close(g1.out[:B], ref, kv_dtype=torch.bfloat16, what="single rank after timeout")
