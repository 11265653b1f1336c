"""Pin the CPU oracle to golden vectors recorded from the upstream code itself
(tests/golden/make_golden.py imports CloverInfer's CpuAttentionBackend and
KVCacheManager).  Bit-exact: the oracle must reproduce every recorded output,
context length, slot, free stack and block table."""

from __future__ import annotations

import math

import pytest
import torch

from conftest import load_golden
from oracle import CpuAttentionOracle, KVCacheOracle, repeat_kv


@pytest.fixture(scope="module")
def cpu_golden():
    return load_golden("cpu_backend.pt")


@pytest.fixture(scope="module")
def kv_golden():
    return load_golden("kv_manager.pt")


def _replay_backend(sc):
    rep = sc["hq"] // sc["hkv"]
    be = CpuAttentionOracle()
    for r in sc["requests"]:
        layers = [{"key": repeat_kv(l["key"], rep), "value": repeat_kv(l["value"], rep)}
                  for l in r["initial_kv"]]
        assert be.init_request(r["id"], layers) == r["init_ret"]
    for call in sc["calls"]:
        items = [dict(it, key=repeat_kv(it["key"], rep), value=repeat_kv(it["value"], rep))
                 for it in call["items"]]
        outs = be.decode_layer_batch(items)
        yield call, outs, [be.get_context_len(r["id"]) for r in sc["requests"]]


def test_cpu_oracle_bit_exact(cpu_golden):
    n = 0
    for sc in cpu_golden["scenarios"]:
        for call, outs, ctx in _replay_backend(sc):
            assert ctx == call["ctx_after"], sc["name"]
            for o, g in zip(outs, call["outputs"]):
                assert o.dtype == g.dtype and o.shape == g.shape
                assert torch.equal(o, g), f"{sc['name']} step {call['step']} layer {call['layer']}"
                n += 1
    assert n >= 26


def test_cpu_oracle_errors():
    be = CpuAttentionOracle()
    kv = [{"key": torch.zeros(3, 2, 4), "value": torch.zeros(3, 2, 4)}]
    assert be.init_request("a", kv) == 3
    with pytest.raises(ValueError):
        be.init_request("a", kv)
    with pytest.raises(ValueError):
        be.init_request("b", [])
    with pytest.raises(KeyError):
        be.decode_layer("zz", 0, torch.zeros(2, 4), torch.zeros(2, 4), torch.zeros(2, 4))
    be.free_request("a")
    be.free_request("a")  # idempotent


def test_kv_oracle_op_stream(kv_golden):
    g = kv_golden
    m = KVCacheOracle(g["num_blocks"], g["block_size"], 2, 8, with_storage=False)
    for op in g["ops"]:
        try:
            if op["op"] == "allocate":
                m.allocate(op["id"], seq_len=op["seq_len"])
            elif op["op"] == "append_slot":
                assert list(m.append_slot(op["id"])) == op["ret"]
            else:
                m.free(op["id"])
            assert "error" not in op, op
        except RuntimeError as e:
            assert op.get("error") == str(e)
        assert m.free_blocks == op["free_blocks"]
        assert m.block_tables == op["tables"]
        assert m.context_lens == op["ctx"]
    assert any("error" in op for op in g["ops"]), "fixture should exercise OOM"


def test_kv_oracle_pins(kv_golden):
    g = kv_golden
    # tests/test_kernels.py:8-34 — 5 appends at block size 4 -> len 5, 2 blocks
    pin = KVCacheOracle(16, 4, 2, 8)
    pin.allocate("req_1", seq_len=0)
    for _ in range(5):
        pin.append_slot("req_1")
    assert pin.context_lens["req_1"] == g["pin_ctx"] == 5
    assert pin.block_tables["req_1"] == g["pin_tables"]
    assert len(pin.block_tables["req_1"]) == 2
    # tests/verify_attention.py:88-136 reference path (fp32 here)
    ref = KVCacheOracle(100, 16, 4, 32)
    ref.allocate("r", seq_len=0)
    for _ in range(50):
        ref.write_new_kv("r", g["pin_ref"]["k"], g["pin_ref"]["v"])
    out = ref.paged_attention_ref(g["pin_ref"]["q"], ["r"])
    assert torch.equal(out, g["pin_ref"]["out"])
    # ragged multi-request gather reference
    rg = g["ragged"]
    m = KVCacheOracle(10, 16, 2, 32)
    for rid, n in zip(rg["ids"], [5, 37, 70]):
        m.allocate(rid, n)
    m.k_cache.copy_(rg["k_cache"])
    m.v_cache.copy_(rg["v_cache"])
    for rid, n in zip(rg["ids"], [5, 37, 70]):
        m.context_lens[rid] = n
    t, l, mx = m.get_kernel_inputs(rg["ids"])
    assert torch.equal(t, rg["tables"]) and torch.equal(l, rg["lens"]) and mx == rg["max"]
    assert torch.equal(m.paged_attention_ref(rg["q"], rg["ids"]), rg["out"])


def test_kernel_inputs_padding(kv_golden):
    g = kv_golden
    m = KVCacheOracle(g["num_blocks"], g["block_size"], 2, 8, with_storage=False)
    for op in g["ops"]:
        try:
            if op["op"] == "allocate":
                m.allocate(op["id"], seq_len=op["seq_len"])
            elif op["op"] == "append_slot":
                m.append_slot(op["id"])
            else:
                m.free(op["id"])
        except RuntimeError:
            pass
    t, l, mx = m.get_kernel_inputs(g["final_ids"])
    assert torch.equal(t, g["kernel_tables"]) and torch.equal(l, g["kernel_lens"])
    assert mx == g["kernel_max"]
    assert (t == -1).any() or t.shape[1] == max(len(v) for v in m.block_tables.values())


def test_paged_ref_matches_contiguous_attend():
    """The paged gather reference (fixed 1/sqrt(D)) equals the contiguous
    backend math at score_scale = 1/sqrt(D): both upstream paths agree."""
    from oracle import attend
    g = torch.Generator().manual_seed(5)
    m = KVCacheOracle(12, 16, 3, 32)
    k = torch.randn(41, 3, 32, generator=g)
    v = torch.randn(41, 3, 32, generator=g)
    m.load_initial_kv("x", k, v)
    q = torch.randn(1, 3, 32, generator=g)
    a = m.paged_attention_ref(q, ["x"])[0]
    b = attend(q[0], k, v, 1.0 / math.sqrt(32))
    assert torch.allclose(a, b, atol=1e-6, rtol=1e-5)
