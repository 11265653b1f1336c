"""Balanced (stream) decode vs the CPU oracle and vs the partition kernels.

The stream kernel is what ``partition_tokens=-1`` (CLOVER_B200_PARTITION_BALANCED)
runs on the tensor-core path (bf16/fp16 cache, head_dim 64/128/256, block
16/32, up to 1024 sequences):
every resident warp owns an equal share of all (sequence, KV head, block)
units and the split-K reduce merges the pieces of each (row, head).  These
cases stress what that decomposition adds: many and ragged sequences (the
32-sequence window slides), empty and one-token rows, tiny problems (few
workers), multi-token causal rows with the KV append fused per unit, and
agreement with the fixed-partition kernels.  Tolerance:
``conftest.assert_attn_close``.
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import assert_attn_close, gpu
from oracle import attend, repeat_kv

pytestmark = gpu


def _case(lens, n_new=None, *, hq=8, hkv=2, D=128, bs=16, dt=torch.bfloat16, q_dt=torch.float32,
          pt=-1, seed=0, step=False, max_ctx=None):
    """One paged_decode (or decode_step when ``step``) call on sequences whose
    last row holds lens[b] tokens, with n_new[b] causal rows each.  Returns the
    output, the oracle reference and the status word."""
    from cloverinfer_b200 import _lib
    dev = "cuda"
    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    n_new = [1] * B if n_new is None else list(n_new)
    nblk = [max(1, -(-n // bs)) for n in lens]
    nb = sum(nblk) + 3
    kc = torch.randn(nb, bs, hkv, D, generator=g).to(dt)
    vc = torch.randn(nb, bs, hkv, D, generator=g).to(dt)
    perm = torch.randperm(nb, generator=g)
    tables = torch.full((B, max(nblk) + 1), -1, dtype=torch.int32)
    o = 0
    for i, k in enumerate(nblk):
        tables[i, :k] = perm[o:o + k].to(torch.int32)
        o += k
    T = sum(n_new)
    q = torch.randn(T, hq, D, generator=g).to(dt).to(q_dt)
    kn = torch.randn(T, hkv, D, generator=g).to(dt)
    vn = torch.randn(T, hkv, D, generator=g).to(dt)
    qsl, ctx = [0], []
    for n, k in zip(lens, n_new):
        qsl.append(qsl[-1] + k)
        ctx += [max(0, n - k + 1 + j) for j in range(k)] if n > 0 else [0] * k
    qsl_t = torch.tensor(qsl, dtype=torch.int32)
    ctx_t = torch.tensor(ctx, dtype=torch.int32)
    out = torch.full((T, hq, D), float("nan"), dtype=q_dt, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    max_q = max(n_new)
    mc = max_ctx or max(lens)
    nbytes = _lib.decode_workspace_bytes(B, T, max_q, mc, hq, hkv, D, bs, dt, q_dt, pt)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    kcd, vcd = kc.to(dev), vc.to(dev)
    common = dict(max_queries_per_seq=max_q, max_ctx_len=mc, score_scale=1 / math.sqrt(D),
                  partition_tokens=pt, workspace=ws, status=status)
    if step:
        _lib.decode_step(out, q.to(dev), kcd, vcd, kn.to(dev), vn.to(dev), tables.to(dev),
                         qsl_t.to(dev), ctx_t.to(dev), **common)
    else:
        _lib.paged_decode(out, q.to(dev), kcd, vcd, tables.to(dev), qsl_t.to(dev), ctx_t.to(dev),
                          **common)
    torch.cuda.synchronize()
    # reference: the cache as the step leaves it (new rows written at ctx - 1)
    kref, vref = kc.clone(), vc.clone()
    if step:
        r = 0
        for b in range(B):
            for j in range(n_new[b]):
                pos = ctx[r] - 1
                if pos >= 0:
                    blk = int(tables[b, pos // bs])
                    kref[blk, pos % bs] = kn[r]
                    vref[blk, pos % bs] = vn[r]
                r += 1
        assert torch.equal(kcd.cpu(), kref) and torch.equal(vcd.cpu(), vref)
    refs = []
    r = 0
    for b, n in enumerate(lens):
        idx = tables[b, :nblk[b]].long()
        keys = kref[idx].reshape(-1, hkv, D)
        vals = vref[idx].reshape(-1, hkv, D)
        for j in range(n_new[b]):
            c = ctx[r]
            if c == 0:
                refs.append(torch.zeros(hq, D))
            else:
                refs.append(attend(q[r].float(), repeat_kv(keys[:c], hq // hkv),
                                   repeat_kv(vals[:c], hq // hkv), 1 / math.sqrt(D)))
            r += 1
    return out.cpu(), torch.stack(refs), int(status.item())


def test_balanced_split_is_chosen_on_request():
    from cloverinfer_b200 import _lib
    bf, f32 = torch.bfloat16, torch.float32
    bal = _lib.PARTITION_BALANCED
    assert _lib.decode_partition_tokens(8, 8, 1, 32768, 32, 8, 128, 16, bf, f32, bal) == 0
    assert _lib.decode_partition_tokens(8, 8, 1, 32768, 32, 8, 128, 16, bf, f32, 0) > 0
    assert _lib.decode_partition_tokens(8, 8, 1, 32768, 32, 8, 128, 16, bf, f32, 512) == 512
    # fp32 caches and more than 1024 sequences keep the partition kernels
    assert _lib.decode_partition_tokens(4, 4, 1, 512, 12, 12, 64, 16, f32, f32, bal) > 0
    assert _lib.decode_partition_tokens(1025, 1025, 1, 512, 8, 2, 128, 16, bf, f32, bal) > 0


@pytest.mark.parametrize("B,seed", [(33, 1), (300, 2), (1024, 3)])
def test_many_ragged_sequences(B, seed):
    g = torch.Generator().manual_seed(seed)
    lens = torch.randint(0, 700, (B,), generator=g).tolist()
    lens[0], lens[B // 2], lens[-1] = 0, 1, 1999
    out, ref, st = _case(lens, seed=seed)
    assert st == 0
    assert_attn_close(out, ref, what=f"B{B}")


def test_more_sequences_than_the_stream_scan_takes_the_partition_kernel():
    lens = [5 + (i * 37) % 200 for i in range(1025)]
    out, ref, st = _case(lens, seed=9)
    assert st == 0
    assert_attn_close(out, ref, what="B1025")


@pytest.mark.parametrize("lens", [[1], [16], [17], [0, 0, 3], [31, 0, 1, 2, 33]])
def test_tiny_problems(lens):
    out, ref, st = _case(lens, seed=len(lens))
    assert st == 0
    assert_attn_close(out, ref, what=str(lens))


@pytest.mark.parametrize("dt,D,bs,hq,hkv", [(torch.bfloat16, 64, 16, 32, 8), (torch.float16, 128, 32, 28, 4),
                                            (torch.bfloat16, 256, 16, 8, 1), (torch.float16, 128, 16, 64, 8)])
def test_shapes_and_one_long_sequence(dt, D, bs, hq, hkv):
    lens = [40000, 3, 900, 0, 17]
    out, ref, st = _case(lens, hq=hq, hkv=hkv, D=D, bs=bs, dt=dt, seed=D + bs)
    assert st == 0
    assert_attn_close(out, ref, kv_dtype=dt, what=f"{dt} D{D} bs{bs} {hq}/{hkv}")


def test_stream_matches_partition_kernel():
    lens = [4096, 3000, 777, 1, 0, 12345]
    a, ref, st_a = _case(lens, pt=-1, seed=5)
    b, _, st_b = _case(lens, pt=512, seed=5)
    assert st_a == 0 and st_b == 0
    assert float((a - b).abs().max()) < 2e-5
    assert_attn_close(a, ref, what="stream")


@pytest.mark.parametrize("hq,hkv,bs", [(8, 4, 16), (32, 8, 32), (16, 8, 16)])
def test_multitoken_causal_step(hq, hkv, bs):
    # group * 4 rows: 8 columns (appended in the decode) or 16 (two chunks,
    # appended by a kernel of its own)
    lens = [1, 2, 5, 17, 33, 64, 900, 2048]
    n_new = [1, 2, 4, 3, 4, 4, 2, 4]
    out, ref, st = _case(lens, n_new, hq=hq, hkv=hkv, bs=bs, dt=torch.float16, step=True,
                         seed=hq + bs)
    assert st == 0
    assert_attn_close(out, ref, kv_dtype=torch.float16, what=f"{hq}/{hkv} bs{bs}")


def test_fused_append_single_token_rows():
    lens = [700, 1, 16, 17, 4097]
    out, ref, st = _case(lens, step=True, seed=21)
    assert st == 0
    assert_attn_close(out, ref, what="append")


def test_bf16_queries_and_outputs():
    out, ref, st = _case([100, 2000, 3], q_dt=torch.bfloat16, seed=4)
    assert out.dtype == torch.bfloat16 and st == 0
    assert_attn_close(out, ref, kv_dtype=torch.bfloat16, out_dtype=torch.bfloat16, what="bf16 q")


def test_context_past_max_ctx_is_flagged():
    from cloverinfer_b200 import _lib
    out, ref, st = _case([300, 40], seed=8, max_ctx=200)
    assert st & _lib.DEV_CTX_RANGE
    assert_attn_close(out[1], ref[1], what="unaffected row")
