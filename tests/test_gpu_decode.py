"""Paged decode attention on the GPU vs the CPU oracle.

* golden scenarios recorded from the upstream CpuAttentionBackend, replayed
  through B200AttentionBackend (same interface, native GQA);
* the five reference configurations (seeded synthetic inputs; c3 at its full
  32k context, c4/c5 with reduced batch) against ``oracle.attend`` with
  repeat_kv-expanded K/V;
* edge cases: empty / block-boundary / partition-boundary contexts, split-K
  invariance, bf16 queries, expanded K/V, bad block ids, interface errors.
Tolerance: ``conftest.assert_attn_close``.
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import assert_attn_close, attn_errors, gpu, load_golden
from oracle import attend, repeat_kv

pytestmark = gpu


def _backend(**kw):
    from cloverinfer_b200 import B200AttentionBackend
    return B200AttentionBackend(device="cuda", **kw)


# ---------------------------------------------------------------- golden replay
@pytest.mark.parametrize("expanded", [False, True])
def test_golden_scenarios(expanded):
    g = load_golden("cpu_backend.pt")
    for sc in g["scenarios"]:
        rep = sc["hq"] // sc["hkv"]
        be = _backend(num_blocks=64, block_size=16, num_kv_heads=sc["hkv"], max_seqs=8)
        ex = (lambda t: repeat_kv(t, rep)) if expanded else (lambda t: t)
        for r in sc["requests"]:
            kv = [{"key": ex(l["key"]), "value": ex(l["value"])} for l in r["initial_kv"]]
            assert be.init_request(r["id"], kv) == r["init_ret"]
        kv_dtype = sc["requests"][0]["initial_kv"][0]["key"].dtype
        for call in sc["calls"]:
            items = [dict(it, key=ex(it["key"]), value=ex(it["value"])) for it in call["items"]]
            outs = be.decode_layer_batch(items)
            assert [be.get_context_len(r["id"]) for r in sc["requests"]] == call["ctx_after"]
            for o, ref, it in zip(outs, call["outputs"], items):
                assert o.shape == ref.shape and o.dtype == ref.dtype and o.device.type == "cpu"
                assert_attn_close(o, ref, kv_dtype=kv_dtype, out_dtype=ref.dtype,
                                  what=f"{sc['name']} s{call['step']} l{call['layer']}")
        for r in sc["requests"]:
            be.free_request(r["id"])
            be.free_request(r["id"])
        assert be.pool.free_count == be.pool.num_blocks


# ---------------------------------------------------------------- configurations
def _run_config(name, *, batch=None, seed=0, steps=1, churn_step=False, ctx_cap=None, check=None):
    """Drive B200AttentionBackend.decode_batch on a config; compare every
    query row (or the rows in ``check``) with the oracle."""
    from cloverinfer_b200.workloads import CONFIGS, context_lengths, new_tokens, randn
    cfg = CONFIGS[name]
    B = batch or cfg.batch
    lens = context_lengths(cfg, seed, B)
    if ctx_cap:
        lens = [min(x, ctx_cap) for x in lens]
    bs, hkv, hq, D, dt = cfg.block_size, cfg.num_kv_heads, cfg.num_q_heads, cfg.head_dim, cfg.dtype
    L = cfg.num_layers
    blocks = sum(-(-(n + 8 * steps) // bs) for n in lens) * 2 + 64
    be = _backend(num_blocks=blocks, block_size=bs, num_kv_heads=hkv, kv_dtype=dt,
                  max_seqs=2 * B + 4, shuffle_seed=seed + 11, partition_tokens=cfg.partition_tokens)
    kv_host = {}
    ids = [f"{name}-{seed}-{i}" for i in range(B)]
    for i, (rid, n) in enumerate(zip(ids, lens)):
        layers = []
        for l in range(L):
            k = randn((n, hkv, D), seed * 100003 + i * 7919 + l * 2 + 1, cfg.value_scale, dt)
            v = randn((n, hkv, D), seed * 100003 + i * 7919 + l * 2 + 2, cfg.value_scale, dt)
            layers.append({"key": k, "value": v})
        assert be.init_request(rid, layers) == n
        kv_host[rid] = layers
    worst = (0.0, 0.0)
    for step in range(steps):
        nn = new_tokens(cfg, seed + step, B)
        T = sum(nn)
        for l in range(L):
            q = randn((T, hq, D), 7 + step * 31 + l, cfg.value_scale, torch.float32)
            q = q.to(dt).float()  # values representable in the cache dtype
            k = randn((T, hkv, D), 8 + step * 31 + l, cfg.value_scale, dt)
            v = randn((T, hkv, D), 9 + step * 31 + l, cfg.value_scale, dt)
            out = be.decode_batch(ids, l, q.cuda(), k.cuda(), v.cuda(), cfg.score_scale, n_new=nn).cpu()
            off = 0
            for b, rid in enumerate(ids):
                layer = kv_host[rid][l]
                for j in range(nn[b]):
                    layer["key"] = torch.cat([layer["key"], k[off + j:off + j + 1]])
                    layer["value"] = torch.cat([layer["value"], v[off + j:off + j + 1]])
                    if check is None or b in check:
                        ref = attend(q[off + j], repeat_kv(layer["key"], cfg.group),
                                     repeat_kv(layer["value"], cfg.group), cfg.score_scale)
                        assert_attn_close(out[off + j], ref, kv_dtype=dt,
                                          what=f"{name} step {step} layer {l} seq {b} tok {j}")
                        e = attn_errors(out[off + j], ref)
                        worst = (max(worst[0], e[0]), max(worst[1], e[1]))
                off += nn[b]
        if churn_step:
            # free ~30 % of the sequences and admit new ones (allocator churn)
            g = torch.Generator().manual_seed(seed + 99 + step)
            drop = [i for i in range(B) if float(torch.rand(1, generator=g)) < cfg.churn or i == 0]
            for i in drop:
                be.free_request(ids[i])
                del kv_host[ids[i]]
                ids[i] = f"{ids[i]}-r{step}"
                n = int(torch.randint(16, 2048, (1,), generator=g))
                layers = [{"key": randn((n, hkv, D), 5000 + i * 3 + step, 1.0, dt),
                           "value": randn((n, hkv, D), 6000 + i * 3 + step, 1.0, dt)}
                          for _ in range(L)]
                be.init_request(ids[i], layers)
                kv_host[ids[i]] = layers
    be.pool.check_status()
    return worst


def test_c1_opt125m_fp32_full():
    abs_e, rel_e = _run_config("c1", steps=2)
    assert abs_e < 1e-4


def test_c2_qwen_gqa7_bf16_full():
    _run_config("c2")


def test_c3_llama8b_32k_full_context():
    # full 32k contexts for all 8 sequences; the oracle checks three of them
    _run_config("c3", check={0, 3, 7})


def test_c4_mixed_multitoken_fp16_churn():
    _run_config("c4", batch=48, steps=3, churn_step=True, check=set(range(0, 48, 3)))


def test_c5_llama70b_gqa8_bf16():
    _run_config("c5", batch=4, ctx_cap=20000)


# ---------------------------------------------------------------- raw-API edge cases
def _raw_case(lens, *, hq=8, hkv=2, D=128, bs=16, dt=torch.bfloat16, q_dt=torch.float32,
              pt=0, seed=0, table_width=None, bad_block=False):
    from cloverinfer_b200 import _lib
    dev = "cuda"
    g = torch.Generator().manual_seed(seed)
    nblk = [max(1, -(-n // bs)) for n in lens]
    nb = sum(nblk) + 3
    kc = torch.randn(nb, bs, hkv, D, generator=g).to(dt)
    vc = torch.randn(nb, bs, hkv, D, generator=g).to(dt)
    perm = torch.randperm(nb, generator=g)
    width = table_width or max(nblk)
    tables = torch.full((len(lens), width), -1, dtype=torch.int32)
    o = 0
    for i, k in enumerate(nblk):
        tables[i, :k] = perm[o:o + k].to(torch.int32)
        o += k
    if bad_block:
        tables[0, 0] = nb + 5
    q = torch.randn(len(lens), hq, D, generator=g).to(dt).to(q_dt)
    out = torch.full_like(q, float("nan")).to(dev)
    qsl = torch.arange(len(lens) + 1, dtype=torch.int32)
    ctx = torch.tensor(lens, dtype=torch.int32)
    status = torch.zeros(1, dtype=torch.int32, device=dev)
    nbytes = _lib.decode_workspace_bytes(len(lens), len(lens), 1, max(lens), hq, hkv, D, bs, dt, q_dt, pt)
    ws = torch.empty(max(nbytes, 1), dtype=torch.uint8, device=dev)
    _lib.paged_decode(out, q.to(dev), kc.to(dev), vc.to(dev), tables.to(dev), qsl.to(dev), ctx.to(dev),
                      max_queries_per_seq=1, max_ctx_len=max(lens), score_scale=1 / math.sqrt(D),
                      partition_tokens=pt, workspace=ws, status=status)
    refs = []
    for i, n in enumerate(lens):
        if n == 0 or (bad_block and i == 0):
            refs.append(torch.zeros(hq, D))  # row 0 of a bad-block case is flagged, not checked
            continue
        idx = tables[i, :nblk[i]].long()
        keys = kc[idx].reshape(-1, hkv, D)[:n]
        vals = vc[idx].reshape(-1, hkv, D)[:n]
        refs.append(attend(q[i].float(), repeat_kv(keys, hq // hkv), repeat_kv(vals, hq // hkv),
                           1 / math.sqrt(D)))
    return out.cpu(), torch.stack(refs), int(status.item())


@pytest.mark.parametrize("dt,D,bs", [(torch.bfloat16, 128, 16), (torch.float16, 128, 32),
                                     (torch.bfloat16, 64, 16), (torch.bfloat16, 256, 16),
                                     (torch.float32, 64, 16), (torch.float16, 96, 8)])
@pytest.mark.parametrize("pt", [0, 64, 512])
def test_boundary_contexts(dt, D, bs, pt):
    lens = [0, 1, 15, 16, 17, 63, 64, 65, 511, 512, 513, 1500]
    if pt and pt % bs:
        pytest.skip("partition must be a multiple of the block size")
    out, ref, st = _raw_case(lens, D=D, bs=bs, dt=dt, pt=pt)
    assert st == 0
    assert torch.equal(out[0], torch.zeros_like(out[0]))  # empty context -> zeros
    assert_attn_close(out, ref, kv_dtype=dt, what=f"{dt} D{D} bs{bs} pt{pt}")


def test_split_k_invariance():
    lens = [4096, 3000, 777]
    outs = [_raw_case(lens, pt=pt, seed=3)[0] for pt in (64, 128, 512, 1024)]
    for o in outs[1:]:
        assert float((o - outs[0]).abs().max()) < 2e-5


@pytest.mark.parametrize("q_dt", [torch.bfloat16, torch.float32])
def test_query_dtype_and_output_dtype(q_dt):
    out, ref, st = _raw_case([100, 2000], q_dt=q_dt, seed=4)
    assert out.dtype == q_dt and st == 0
    assert_attn_close(out, ref, kv_dtype=torch.bfloat16, out_dtype=q_dt, what=str(q_dt))


def test_gqa_groups_and_mha():
    for hq, hkv in [(32, 8), (28, 4), (64, 8), (8, 8), (16, 1)]:
        out, ref, st = _raw_case([300, 1025], hq=hq, hkv=hkv, seed=hq)
        assert st == 0
        assert_attn_close(out, ref, what=f"hq{hq} hkv{hkv}")


def test_bad_block_id_is_flagged_not_fatal():
    from cloverinfer_b200 import _lib
    out, ref, st = _raw_case([40, 40], bad_block=True, seed=6)
    assert st & _lib.DEV_BAD_BLOCK
    assert_attn_close(out[1], ref[1], what="unaffected row")


# ---------------------------------------------------------------- interface semantics
def test_backend_interface_semantics():
    be = _backend(num_blocks=64, num_kv_heads=2, max_seqs=4)
    kv = [{"key": torch.randn(5, 2, 64).bfloat16(), "value": torch.randn(5, 2, 64).bfloat16()}
          for _ in range(3)]
    assert be.init_request("r", kv) == 5
    with pytest.raises(ValueError):
        be.init_request("r", kv)
    with pytest.raises(ValueError):
        be.init_request("e", [])
    with pytest.raises(KeyError):
        be.decode_layer("nope", 0, torch.zeros(8, 64), torch.zeros(2, 64), torch.zeros(2, 64))
    for layer in range(3):
        out = be.decode_layer("r", layer, torch.randn(1, 8, 64), torch.randn(1, 2, 64).bfloat16(),
                              torch.randn(1, 2, 64).bfloat16(), 0.125)
        assert out.shape == (1, 8, 64) and out.dtype == torch.float32
        assert be.get_context_len("r") == (5 if layer < 2 else 6)
    info = be.get_debug_info()
    assert info["live_requests"] == 1 and info["num_layers"] == 3
    be.free_request("r")
    be.free_request("r")
    with pytest.raises(KeyError):
        be.get_context_len("r")
    assert be.pool.free_count == 64


# ---------------------------------------------------------------- host inputs
@pytest.mark.parametrize("form", ["pinned", "pageable", "expanded-kv"])
def test_decode_batch_host_inputs_match_device_inputs(form):
    """decode_batch with host tensors (copied asynchronously, through a
    pinned staging copy where the heads it keeps are not contiguous) gives
    exactly what the same call with device tensors gives."""
    hkv, grp, D, bs = 2, 4, 128, 16
    hq = hkv * grp
    lens, n_new = [300, 17, 1000], [2, 1, 3]
    g = torch.Generator().manual_seed(21)
    bes = [_backend(num_blocks=256, block_size=bs, num_kv_heads=hkv, max_seqs=4, shuffle_seed=3)
           for _ in range(2)]
    ids = [f"h{i}" for i in range(len(lens))]
    for rid, n in zip(ids, lens):
        kv = [{"key": torch.randn(n, hkv, D, generator=g).bfloat16(),
               "value": torch.randn(n, hkv, D, generator=g).bfloat16()}]
        for be in bes:
            be.init_request(rid, kv)
    T = sum(n_new)
    for step in range(2):
        q = torch.randn(T, hq, D, generator=g).bfloat16().float()
        k = torch.randn(T, hkv, D, generator=g).bfloat16()
        v = torch.randn(T, hkv, D, generator=g).bfloat16()
        ref = bes[0].decode_batch(ids, 0, q.cuda(), k.cuda(), v.cuda(), 1 / math.sqrt(D),
                                  n_new=n_new).cpu()
        if form == "expanded-kv":
            k, v = repeat_kv(k, grp), repeat_kv(v, grp)
        if form != "pageable":
            q, k, v = q.pin_memory(), k.pin_memory(), v.pin_memory()
        out = bes[1].decode_batch(ids, 0, q, k, v, 1 / math.sqrt(D), n_new=n_new)
        assert out.is_cuda and out.shape == (T, hq, D)
        assert torch.equal(out.cpu(), ref), f"{form}, step {step}"
        assert [bes[1].get_context_len(r) for r in ids] == [bes[0].get_context_len(r) for r in ids]
