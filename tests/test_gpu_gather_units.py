"""Both unit shapes of the fused gather's split-K reduce, on one GPU.

``clover_b200_decode_step_gather`` merges the decode's partials and sends each
value to every rank.  When no (row, head) has more than 16 partials (or the
pairs alone fill the grid's warps) a warp takes a whole (row, head);
otherwise 32-dim units whose partitions the CTA's warps split.  A one-rank
gather (its own receive buffer only) runs the whole kernel, sends and bounded
receives included, with no peer: here a ragged multi-token GQA batch at two partition lengths, one per
unit shape, is held to the CPU oracle (``oracle.attend`` over the sequence's
blocks, each row with its causal limit).
"""

from __future__ import annotations

import math
from types import SimpleNamespace

import pytest
import torch

from conftest import assert_attn_close, gpu
from oracle import attend, repeat_kv

pytestmark = gpu


def _problem(seed=5):
    g = torch.Generator().manual_seed(seed)
    hq_l, hkv_l, D, bs = 8, 2, 128, 16
    lens = [3000, 17, 640, 1, 2049, 96]
    n_new = [3, 1, 4, 1, 2, 1]
    nblk = [-(-n // bs) for n in lens]
    nb = sum(nblk) + 5
    kc = torch.randn(nb, bs, hkv_l, D, generator=g).bfloat16()
    vc = torch.randn(nb, bs, hkv_l, D, generator=g).bfloat16()
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    tables = torch.full((len(lens), max(nblk)), -1, dtype=torch.int32)
    o = 0
    for i, k in enumerate(nblk):
        tables[i, :k] = perm[o:o + k]
        o += k
    T = sum(n_new)
    q = torch.randn(T, hq_l, D, generator=g).bfloat16().float()
    qsl, ctx = [0], []
    for n, k in zip(lens, n_new):
        qsl.append(qsl[-1] + k)
        ctx += list(range(n - k + 1, n + 1))
    return dict(kc=kc, vc=vc, tables=tables, q=q, lens=lens, n_new=n_new, qsl=qsl, ctx=ctx,
                hq_l=hq_l, hkv_l=hkv_l, D=D, bs=bs)


def _oracle(P):
    bs, D, grp = P["bs"], P["D"], P["hq_l"] // P["hkv_l"]
    outs, r = [], 0
    for i, n in enumerate(P["lens"]):
        blocks = P["tables"][i, :-(-n // bs)].long()
        k = P["kc"][blocks].reshape(-1, P["hkv_l"], D)
        v = P["vc"][blocks].reshape(-1, P["hkv_l"], D)
        for _ in range(P["n_new"][i]):
            lim = P["ctx"][r]
            outs.append(attend(P["q"][r], repeat_kv(k[:lim], grp), repeat_kv(v[:lim], grp),
                               1 / math.sqrt(D), out_dtype=torch.float32))
            r += 1
    return torch.stack(outs)


@pytest.mark.parametrize("partition_tokens", [64, 512], ids=["warp-split-units", "row-units"])
def test_gather_reduce_unit_shapes(partition_tokens):
    from cloverinfer_b200 import _lib

    dev = torch.device("cuda")
    P = _problem()
    T, hq_l, D = P["q"].shape[0], P["hq_l"], P["D"]
    parts = -(-max(P["lens"]) // partition_tokens)
    assert (parts > 16) == (partition_tokens == 64)  # one case per unit shape
    kc, vc, tables, q = (P[k].to(dev) for k in ("kc", "vc", "tables", "q"))
    qsl = torch.tensor(P["qsl"], dtype=torch.int32, device=dev)
    ctx = torch.tensor(P["ctx"], dtype=torch.int32, device=dev)
    half = T * hq_l * D
    recv = torch.zeros(2 * half, dtype=torch.int64, device=dev)
    sync = torch.zeros(_lib.gather_sync_bytes() // 4, dtype=torch.int32, device=dev)
    g1 = SimpleNamespace(world=1, rank=0, half_words=half, sync=sync,
                         peer_recv_d=torch.tensor([recv.data_ptr()], dtype=torch.int64, device=dev),
                         out=torch.full((T, hq_l, D), float("nan"), device=dev))
    common = dict(max_queries_per_seq=max(P["n_new"]), max_ctx_len=max(P["lens"]),
                  score_scale=1 / math.sqrt(D), partition_tokens=partition_tokens)
    nbytes = _lib.decode_gather_workspace_bytes(len(P["lens"]), T, max(P["n_new"]), max(P["lens"]),
                                                hq_l, P["hkv_l"], D, P["bs"], torch.bfloat16,
                                                torch.float32, partition_tokens)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    ref = _oracle(P)
    for step in range(3):  # both parities of the receive buffer, and one more
        _lib.decode_step_gather(q, kc, vc, None, None, tables, qsl, ctx, g1, workspace=ws, status=st,
                                **common)
        torch.cuda.synchronize()
        assert int(st.item()) == 0, f"status 0x{int(st.item()):x}"
        assert_attn_close(g1.out.cpu(), ref, kv_dtype=torch.bfloat16,
                          what=f"gather reduce, {partition_tokens}-token partitions, step {step}")
