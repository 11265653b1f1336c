"""fp8 (e4m3) KV cache: paged decode, fused append and the drop-in backend
against the CPU oracle.

The cache holds 1-byte e4m3 values; the decode expands each landed stage to
fp16 (exact) for the tensor-core step.  As for the 16-bit caches, the oracle
is fed the very values the cache holds (the e4m3-rounded K/V, as fp32), so
the tolerance is the same: ``conftest.assert_attn_close``.  Appends are
compared byte for byte.
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import assert_attn_close, gpu
from oracle import attend, repeat_kv

pytestmark = gpu

F8 = torch.float8_e4m3fn


def _case(lens, n_new=None, *, hq=32, hkv=8, D=128, bs=16, q_dt=torch.float32, pt=0, seed=0,
          step=False):
    from cloverinfer_b200 import _lib
    dev = "cuda"
    g = torch.Generator().manual_seed(seed)
    B = len(lens)
    n_new = [1] * B if n_new is None else list(n_new)
    nblk = [max(1, -(-n // bs)) for n in lens]
    nb = sum(nblk) + 3
    kc = torch.randn(nb, bs, hkv, D, generator=g).to(F8)
    vc = torch.randn(nb, bs, hkv, D, generator=g).to(F8)
    perm = torch.randperm(nb, generator=g)
    tables = torch.full((B, max(nblk) + 1), -1, dtype=torch.int32)
    o = 0
    for i, k in enumerate(nblk):
        tables[i, :k] = perm[o:o + k].to(torch.int32)
        o += k
    T = sum(n_new)
    q = torch.randn(T, hq, D, generator=g).to(q_dt)
    kn = torch.randn(T, hkv, D, generator=g).to(F8)
    vn = torch.randn(T, hkv, D, generator=g).to(F8)
    qsl, ctx = [0], []
    for n, k in zip(lens, n_new):
        qsl.append(qsl[-1] + k)
        ctx += [max(0, n - k + 1 + j) for j in range(k)] if n > 0 else [0] * k
    out = torch.full((T, hq, D), float("nan"), dtype=q_dt, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    max_q = max(n_new)
    nbytes = _lib.decode_workspace_bytes(B, T, max_q, max(lens), hq, hkv, D, bs, F8, q_dt, pt)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    kcd, vcd = kc.to(dev), vc.to(dev)
    common = dict(max_queries_per_seq=max_q, max_ctx_len=max(lens), score_scale=1 / math.sqrt(D),
                  partition_tokens=pt, workspace=ws, status=status)
    qsl_d = torch.tensor(qsl, dtype=torch.int32, device=dev)
    ctx_d = torch.tensor(ctx, dtype=torch.int32, device=dev)
    if step:
        _lib.decode_step(out, q.to(dev), kcd, vcd, kn.to(dev), vn.to(dev), tables.to(dev), qsl_d,
                         ctx_d, **common)
    else:
        _lib.paged_decode(out, q.to(dev), kcd, vcd, tables.to(dev), qsl_d, ctx_d, **common)
    torch.cuda.synchronize()
    kref, vref = kc.view(torch.uint8).clone(), vc.view(torch.uint8).clone()
    if step:
        r = 0
        for b in range(B):
            for j in range(n_new[b]):
                pos = ctx[r] - 1
                blk = int(tables[b, pos // bs])
                kref[blk, pos % bs] = kn[r].view(torch.uint8)
                vref[blk, pos % bs] = vn[r].view(torch.uint8)
                r += 1
        assert torch.equal(kcd.cpu().view(torch.uint8), kref)
        assert torch.equal(vcd.cpu().view(torch.uint8), vref)
    kf, vf = kref.view(F8).float(), vref.view(F8).float()
    refs, r = [], 0
    for b, n in enumerate(lens):
        idx = tables[b, :nblk[b]].long()
        keys, vals = kf[idx].reshape(-1, hkv, D), vf[idx].reshape(-1, hkv, D)
        for j in range(n_new[b]):
            c = ctx[r]
            refs.append(torch.zeros(hq, D) if c == 0 else
                        attend(q[r].float(), repeat_kv(keys[:c], hq // hkv),
                               repeat_kv(vals[:c], hq // hkv), 1 / math.sqrt(D)))
            r += 1
    return out.cpu(), torch.stack(refs), int(status.item())


@pytest.mark.parametrize("D,bs,hq,hkv", [(128, 16, 32, 8), (128, 32, 28, 4), (256, 16, 8, 1)])
@pytest.mark.parametrize("pt", [0, 64])
def test_fp8_boundaries_and_shapes(D, bs, hq, hkv, pt):
    if pt % bs:
        pytest.skip("partition must be a multiple of the block size")
    lens = [0, 1, 15, 16, 17, 63, 64, 65, 511, 512, 513, 4097]
    out, ref, st = _case(lens, hq=hq, hkv=hkv, D=D, bs=bs, pt=pt, seed=D + bs + pt)
    assert st == 0
    assert torch.equal(out[0], torch.zeros_like(out[0]))
    assert_attn_close(out, ref, what=f"fp8 D{D} bs{bs} {hq}/{hkv} pt{pt}")


def test_fp8_half_queries_and_long_context():
    out, ref, st = _case([32768, 3, 2000], q_dt=torch.float16, seed=2)
    assert st == 0 and out.dtype == torch.float16
    assert_attn_close(out, ref, out_dtype=torch.float16, what="fp16 q")


@pytest.mark.parametrize("hq,hkv,bs", [(32, 8, 32), (16, 8, 16)])
def test_fp8_multitoken_step_with_fused_append(hq, hkv, bs):
    lens = [1, 2, 5, 17, 33, 64, 900, 2048]
    n_new = [1, 2, 4, 3, 4, 4, 2, 4]
    out, ref, st = _case(lens, n_new, hq=hq, hkv=hkv, bs=bs, step=True, seed=hq + bs)
    assert st == 0
    assert_attn_close(out, ref, what=f"fp8 step {hq}/{hkv} bs{bs}")


def test_fp8_kv_append_is_bitexact():
    from cloverinfer_b200 import _lib
    g = torch.Generator().manual_seed(4)
    nb, bs, h, d = 12, 16, 8, 128
    kc = torch.zeros(nb, bs, h, d, dtype=F8, device="cuda")
    vc = torch.zeros_like(kc)
    kn = torch.randn(20, h, d, generator=g).to(F8)
    vn = torch.randn(20, h, d, generator=g).to(F8)
    slots = torch.randperm(nb * bs, generator=g)[:20]
    status = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.kv_append(kc, vc, kn.cuda(), vn.cuda(), slots.cuda(), status)
    torch.cuda.synchronize()
    flat_k = kc.view(torch.uint8).reshape(nb * bs, h, d).cpu()
    flat_v = vc.view(torch.uint8).reshape(nb * bs, h, d).cpu()
    assert torch.equal(flat_k[slots], kn.view(torch.uint8))
    assert torch.equal(flat_v[slots], vn.view(torch.uint8))
    assert int(status.item()) == 0


def test_fp8_backend_drop_in():
    from cloverinfer_b200 import B200AttentionBackend
    hq, hkv, D = 32, 8, 128
    be = B200AttentionBackend(num_blocks=128, num_kv_heads=hkv, kv_dtype=F8, device="cuda",
                              max_seqs=4)
    g = torch.Generator().manual_seed(7)
    kv = {}
    for rid, n in [("a", 700), ("b", 40)]:
        k = torch.randn(n, hkv, D, generator=g).bfloat16()
        v = torch.randn(n, hkv, D, generator=g).bfloat16()
        be.init_request(rid, [{"key": k, "value": v}])
        kv[rid] = [k.to(F8).float(), v.to(F8).float()]
    for _ in range(3):  # eager, then the captured step
        items = [{"request_id": rid, "layer_idx": 0, "score_scale": 1 / math.sqrt(D),
                  "query": torch.randn(hq, D, generator=g),
                  "key": torch.randn(hkv, D, generator=g).bfloat16(),
                  "value": torch.randn(hkv, D, generator=g).bfloat16()} for rid in kv]
        res = be.decode_layer_batch(items)
        for it, o in zip(items, res):
            k, v = kv[it["request_id"]]
            k = torch.cat([k, it["key"].to(F8).float()[None]])
            v = torch.cat([v, it["value"].to(F8).float()[None]])
            kv[it["request_id"]] = [k, v]
            ref = attend(it["query"], repeat_kv(k, hq // hkv), repeat_kv(v, hq // hkv),
                         1 / math.sqrt(D))
            assert_attn_close(o[0], ref, what=f"backend fp8 {it['request_id']}")


def test_fp8_unsupported_shapes_raise():
    from cloverinfer_b200 import _lib
    with pytest.raises(Exception):
        _lib.decode_workspace_bytes(2, 2, 1, 100, 8, 2, 64, 16, F8, torch.float32, 0)
