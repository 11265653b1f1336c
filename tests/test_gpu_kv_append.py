"""KV append (reshape-and-cache) and slot mapping: bit-exact on the GPU."""

from __future__ import annotations

import pytest
import torch

from conftest import gpu

pytestmark = gpu


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("heads,dim,bs", [(8, 128, 16), (1, 128, 16), (12, 64, 16), (2, 32, 32), (3, 40, 8)])
def test_append_bit_exact(dtype, heads, dim, bs):
    from cloverinfer_b200 import _lib
    nb = 97
    dev = "cuda"
    g = torch.Generator().manual_seed(heads * 1000 + dim)
    kc = torch.randn(nb, bs, heads, dim, generator=g).to(dtype).to(dev)
    vc = torch.randn(nb, bs, heads, dim, generator=g).to(dtype).to(dev)
    n = 300
    slots = torch.randperm(nb * bs, generator=g)[:n].to(torch.int64)
    slots[::17] = -1  # padding tokens are skipped
    kn = torch.randn(n, heads, dim, generator=g).to(dtype)
    vn = torch.randn(n, heads, dim, generator=g).to(dtype)
    ref_k = kc.cpu().reshape(nb * bs, heads, dim).clone()
    ref_v = vc.cpu().reshape(nb * bs, heads, dim).clone()
    keep = slots >= 0
    ref_k[slots[keep]] = kn[keep]
    ref_v[slots[keep]] = vn[keep]
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.kv_append(kc, vc, kn.to(dev), vn.to(dev), slots.to(dev), status)
    assert int(status.item()) == 0
    assert torch.equal(kc.cpu().reshape(nb * bs, heads, dim), ref_k)
    assert torch.equal(vc.cpu().reshape(nb * bs, heads, dim), ref_v)


def test_append_strided_source_and_bad_slot():
    from cloverinfer_b200 import _lib
    dev = "cuda"
    nb, bs, h, d = 8, 16, 2, 64
    kc = torch.zeros(nb, bs, h, d, dtype=torch.bfloat16, device=dev)
    vc = torch.zeros_like(kc)
    # rows of a fused [n, 3, H, D] qkv-like buffer: token stride 3*H*D
    fused = torch.randn(5, 3, h, d, device=dev).to(torch.bfloat16)
    kn, vn = fused[:, 1], fused[:, 2]
    slots = torch.tensor([0, 17, nb * bs - 1, nb * bs, -1], dtype=torch.int64, device=dev)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    _lib.kv_append(kc, vc, kn, vn, slots, status)
    assert int(status.item()) & _lib.DEV_BAD_SLOT
    flat_k = kc.reshape(-1, h, d)
    assert torch.equal(flat_k[0], kn[0]) and torch.equal(flat_k[17], kn[1])
    assert torch.equal(flat_k[nb * bs - 1], kn[2])
    assert torch.equal(vc.reshape(-1, h, d)[17], vn[1])
    assert int((flat_k != 0).any(dim=(1, 2)).sum()) == 3


def test_compute_slots_matches_upstream_arithmetic():
    """slot = table[pos // bs] * bs + pos % bs (memory_manager.py:113-121)."""
    from cloverinfer_b200 import PagedKVPool
    from oracle import KVCacheOracle
    pool = PagedKVPool(200, 16, 1, 64, device="cuda", max_seqs=16, max_blocks_per_seq=32)
    pool.shuffle_free_stack(9)
    ref = KVCacheOracle(200, 16, 1, 64, with_storage=False)
    ref.free_blocks = pool.free_stack.cpu().tolist()
    lens = [5, 16, 17, 100, 255, 0, 31]
    rows = list(range(len(lens)))
    for r, n in zip(rows, lens):
        ref.allocate(f"s{r}", n)
    pool.reserve(rows, [n + 1 for n in lens])
    n_new = [1, 3, 2, 4, 1, 2, 1]
    for r, (n, k) in enumerate(zip(lens, n_new)):
        for _ in range(k):
            ref.append_slot(f"s{r}")
    pool.reserve(rows, [n + k for n, k in zip(lens, n_new)])
    offs = [0]
    for k in n_new:
        offs.append(offs[-1] + k)
    dev = pool.device
    slots = pool.slots(torch.tensor(rows, dtype=torch.int32, device=dev),
                       torch.tensor(lens, dtype=torch.int32, device=dev),
                       torch.tensor(offs, dtype=torch.int32, device=dev), offs[-1]).cpu().tolist()
    want = []
    for r, (n, k) in enumerate(zip(lens, n_new)):
        want += [ref.slot(f"s{r}", n + j) for j in range(k)]
    assert slots == want
    pool.check_status()


@pytest.mark.parametrize("dt,D,bs,n_new,hq,hkv", [(torch.bfloat16, 128, 16, [1, 1, 1, 1], 32, 8),
                                                  (torch.float16, 128, 32, [1, 3, 4, 2], 32, 8),
                                                  (torch.float32, 64, 16, [1, 1, 2], 12, 12),
                                                  (torch.bfloat16, 64, 16, [2, 1, 1], 8, 2)])
def test_decode_step_matches_append_then_decode(dt, D, bs, n_new, hq, hkv):
    """clover_b200_decode_step (fused append, or its separate-append fallback
    when a sequence's columns span several CTAs) == kv_append + paged_decode:
    same cache bytes, same outputs."""
    import math
    from cloverinfer_b200 import _lib
    from cloverinfer_b200.kv_cache import PagedKVPool
    lens = [700, 33, 1500, 16][:len(n_new)]
    outs, caches = [], []
    for fused in (True, False):
        g = torch.Generator().manual_seed(sum(n_new) + D)
        pool = PagedKVPool(400, bs, hkv, D, dtype=dt, device="cuda", max_seqs=8, max_blocks_per_seq=128)
        pool.shuffle_free_stack(5)
        rows = list(range(len(lens)))
        pool.reserve(rows, [n + k for n, k in zip(lens, n_new)])
        gg = torch.Generator(device="cuda").manual_seed(1)
        pool.k.normal_(generator=gg) if dt == torch.float32 else pool.k.copy_(torch.randn(pool.k.shape, generator=gg, device="cuda").to(dt))
        pool.v.copy_(torch.randn(pool.v.shape, generator=gg, device="cuda").to(dt))
        T = sum(n_new)
        q = torch.randn(T, hq, D, generator=g).to(dt).float().cuda()
        kn = torch.randn(T, hkv, D, generator=g).to(dt).cuda()
        vn = torch.randn(T, hkv, D, generator=g).to(dt).cuda()
        offs, ctx = [0], []
        for n, k in zip(lens, n_new):
            offs.append(offs[-1] + k)
            ctx += list(range(n + 1, n + k + 1))
        dev = "cuda"
        rows_d = torch.tensor(rows, dtype=torch.int32, device=dev)
        offs_d = torch.tensor(offs, dtype=torch.int32, device=dev)
        ctx_d = torch.tensor(ctx, dtype=torch.int32, device=dev)
        if fused:
            out = pool.decode_step(0, q, kn, vn, offs_d, ctx_d, rows_d, max(n_new), max(ctx), 1 / math.sqrt(D))
        else:
            slots = pool.slots(rows_d, torch.tensor(lens, dtype=torch.int32, device=dev), offs_d, T)
            pool.append(0, kn, vn, slots)
            out = pool.decode(0, q, offs_d, ctx_d, rows_d, max(n_new), max(ctx), 1 / math.sqrt(D))
        torch.cuda.synchronize()
        pool.check_status()
        outs.append(out.cpu())
        caches.append((pool.k.cpu(), pool.v.cpu()))
    assert torch.equal(caches[0][0], caches[1][0]) and torch.equal(caches[0][1], caches[1][1])
    assert torch.equal(outs[0], outs[1])


@pytest.mark.parametrize("src", ["host", "device"])
@pytest.mark.parametrize("expanded", [False, True])
def test_prefill_ingestion_every_layer_bit_exact(src, expanded):
    """init_request ingests every layer's prefill K/V (attention_backend.py:68-80)
    through one staging buffer and one multi-layer append on a side stream: the
    cache then holds, bit for bit, what KVCacheOracle.load_initial_kv
    (memory_manager.py:74-93) stores for each layer, with the same block
    tables; a decode issued right after it sees the ingested KV."""
    from cloverinfer_b200 import B200AttentionBackend
    from oracle import KVCacheOracle, repeat_kv
    L, hkv, grp, D, bs, nb = 4, 2, 4, 128, 16, 64
    dt = torch.bfloat16
    be = B200AttentionBackend(device="cuda", num_blocks=nb, block_size=bs, num_kv_heads=hkv,
                              kv_dtype=dt, max_seqs=4)
    orc = [KVCacheOracle(nb, bs, hkv, D, dtype=dt) for _ in range(L)]
    g = torch.Generator().manual_seed(21)
    for rid, T in [("a", 37), ("b", 100), ("c", 16)]:
        layers = [{"key": torch.randn(T, hkv, D, generator=g), "value": torch.randn(T, hkv, D, generator=g)}
                  for _ in range(L)]  # fp32 inputs: the cache rounds them to bf16
        feed = [{k: (repeat_kv(t, grp) if expanded else t) for k, t in l.items()} for l in layers]
        if src == "device":
            feed = [{k: t.cuda() for k, t in l.items()} for l in feed]
        assert be.init_request(rid, feed) == T
        for li in range(L):
            orc[li].load_initial_kv(rid, layers[li]["key"], layers[li]["value"])
        table = be.pool.row_table(be._reqs[rid].row)
        assert table == orc[0].block_tables[rid]
        slots = torch.tensor([table[t // bs] * bs + t % bs for t in range(T)])
        for li in range(L):
            kc = be.pool.k[li].reshape(-1, hkv, D)[slots.cuda()].cpu()
            vc = be.pool.v[li].reshape(-1, hkv, D)[slots.cuda()].cpu()
            ko = orc[li].k_cache.reshape(-1, hkv, D)[slots]
            vo = orc[li].v_cache.reshape(-1, hkv, D)[slots]
            assert torch.equal(kc.view(torch.int16), ko.view(torch.int16)), (rid, li)
            assert torch.equal(vc.view(torch.int16), vo.view(torch.int16)), (rid, li)
    be.pool.check_status()
    # a decode issued right after the ingestion sees it (stream ordering)
    q = torch.randn(hkv * grp, D, generator=g)
    kn = torch.randn(hkv, D, generator=g).to(dt)
    out = be.decode_layer("b", 0, q, kn, kn)
    keys = torch.cat([orc[0].k_cache.reshape(-1, hkv, D)[torch.tensor(
        [orc[0].block_tables["b"][t // bs] * bs + t % bs for t in range(100)])], kn[None]])
    vals = torch.cat([orc[0].v_cache.reshape(-1, hkv, D)[torch.tensor(
        [orc[0].block_tables["b"][t // bs] * bs + t % bs for t in range(100)])], kn[None]])
    from oracle import attend
    ref = attend(q, repeat_kv(keys, grp), repeat_kv(vals, grp), 1.0)
    assert float((out[0] - ref).abs().max()) < 2e-3
    for rid in ("a", "b", "c"):
        be.free_request(rid)
    assert be.pool.free_count == nb

