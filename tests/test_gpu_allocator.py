"""GPU block allocator / tables vs the upstream KVCacheManager, bit-exact.

Replays the op stream recorded from src/core/memory_manager.py
(tests/golden/kv_manager.pt) on the device-resident allocator behind
``cloverinfer_b200.KVCacheManager``: every append_slot (block, offset), the
free stack, every block table, context lengths and the OOM errors must match.
"""

from __future__ import annotations

import math

import pytest
import torch

from conftest import assert_attn_close, gpu, load_golden

pytestmark = gpu


@pytest.fixture(scope="module")
def kv_golden():
    return load_golden("kv_manager.pt")


def test_op_stream_bit_exact(kv_golden):
    from cloverinfer_b200 import KVCacheManager
    g = kv_golden
    m = KVCacheManager(g["num_blocks"], g["block_size"], 2, 8, dtype=torch.float32, device="cuda")
    for i, op in enumerate(g["ops"]):
        try:
            if op["op"] == "allocate":
                m.allocate(op["id"], seq_len=op["seq_len"])
            elif op["op"] == "append_slot":
                assert list(m.append_slot(op["id"])) == op["ret"], (i, op)
            else:
                m.free(op["id"])
            assert "error" not in op, (i, op)
        except RuntimeError as e:
            assert op.get("error") == str(e), (i, op, str(e))
        assert m.free_blocks == op["free_blocks"], i
        assert m.block_tables == op["tables"], i
        assert m.context_lens == op["ctx"], i
    m.pool.check_status()
    t, l, mx = m.get_kernel_inputs(g["final_ids"])
    assert torch.equal(t.cpu(), g["kernel_tables"]) and torch.equal(l.cpu(), g["kernel_lens"])
    assert mx == g["kernel_max"]


def test_upstream_pin_append_and_shape():
    """tests/test_kernels.py:8-63: 5 appends at block 4 -> length 5 on 2 blocks;
    attention returns q's shape."""
    from cloverinfer_b200 import KVCacheManager
    m = KVCacheManager(16, 4, 2, 8, device="cuda")
    m.allocate("req_1", seq_len=0)
    for _ in range(5):
        m.append_slot("req_1")
    assert m.context_lens["req_1"] == 5
    assert len(m.block_tables["req_1"]) == 2
    blocks = m.block_tables["req_1"]
    for i in range(4):
        m.k_cache[blocks[0], i] = i
        m.v_cache[blocks[0], i] = i
    m.k_cache[blocks[1], 0] = 4
    m.v_cache[blocks[1], 0] = 4
    q = torch.ones((1, 2, 8), device="cuda")
    out = m.attention(q, ["req_1"])
    assert out.shape == q.shape
    # all keys equal per token -> weights softmax(8*t/sqrt(8)); output = E[t]
    w = torch.softmax(torch.arange(5.0) * 8 / math.sqrt(8), 0)
    assert torch.allclose(out.cpu(), torch.full((1, 2, 8), float((w * torch.arange(5.0)).sum())), atol=1e-4)


def test_upstream_pin_kernel_vs_reference(kv_golden):
    """tests/verify_attention.py:88-136: fp16, block 16, 4 heads, D=32, 50
    identical tokens; upstream compared allclose(1e-2, 1e-2) with the slow ref."""
    from cloverinfer_b200 import KVCacheManager
    p = kv_golden["pin_ref"]
    m = KVCacheManager(100, 16, 4, 32, dtype=torch.float16, device="cuda")
    m.allocate("req_test_kernel", seq_len=0)
    for _ in range(50):
        m.write_new_kv("req_test_kernel", p["k"].half().cuda(), p["v"].half().cuda())
    q = p["q"].cuda()
    out = m.attention(q, ["req_test_kernel"])
    assert out.dtype == torch.float32 and out.shape == (1, 4, 32)
    ref16 = p["out"]  # fp32 reference on the fp32 tokens
    assert torch.allclose(out.cpu(), ref16, atol=1e-2, rtol=1e-2)
    # and against the exact answer on the fp16-rounded tokens
    from oracle import attend
    exact = attend(p["q"][0], p["k"].half().float().expand(50, 4, 32), p["v"].half().float().expand(50, 4, 32),
                   1.0 / math.sqrt(32))
    assert_attn_close(out[0], exact, kv_dtype=torch.float16, what="verify_attention pin")
    assert m.context_lens["req_test_kernel"] == 50


def test_oom_leaves_state_unchanged():
    from cloverinfer_b200 import KVCacheManager
    m = KVCacheManager(4, 4, 1, 8, device="cuda")
    m.allocate("a", seq_len=7)   # 2 blocks
    m.allocate("b", seq_len=3)   # 1 block
    before = (m.free_blocks, m.block_tables)
    with pytest.raises(RuntimeError, match="OOM: Not enough blocks"):
        m.allocate("c", seq_len=4)  # needs 2, 1 free
    assert (m.free_blocks, m.block_tables) == before
    assert "c" not in m.context_lens
    m.append_slot("b"); m.append_slot("b"); m.append_slot("b")  # fills block of b (len 6 -> 2 blocks)
    with pytest.raises(RuntimeError, match="OOM during append"):
        for _ in range(8):
            m.append_slot("a")
    m.free("a")
    m.free("a")  # idempotent
    m.pool.check_status()


def test_batched_reserve_matches_sequential_pops():
    """One reserve launch for many rows hands out the blocks the upstream
    manager pops for the same calls issued one by one."""
    from cloverinfer_b200 import PagedKVPool
    from oracle import KVCacheOracle
    pool = PagedKVPool(512, 16, 1, 64, device="cuda", max_seqs=64, max_blocks_per_seq=64)
    ref = KVCacheOracle(512, 16, 1, 64, with_storage=False)
    g = torch.Generator().manual_seed(3)
    rows = list(range(40))
    lens = torch.randint(0, 300, (40,), generator=g).tolist()
    for r, n in zip(rows, lens):
        ref.allocate(f"s{r}", n)
    pool.reserve(rows, [n + 1 for n in lens])
    for r in rows:
        assert pool.row_table(r) == ref.block_tables[f"s{r}"]
    # grow a subset by several tokens each, batched vs sequential append_slot
    grow = [(r, int(x)) for r, x in zip(rows[::3], torch.randint(1, 40, (len(rows[::3]),), generator=g))]
    for r, k in grow:
        for _ in range(k):
            ref.append_slot(f"s{r}")
    pool.reserve([r for r, _ in grow], [lens[r] + k for r, k in grow])
    for r in rows:
        assert pool.row_table(r) == ref.block_tables[f"s{r}"], r
    pool.release(rows[5:25])
    for r in rows[5:25]:
        ref.free(f"s{r}")
    assert pool.free_list() == ref.free_blocks
    pool.check_status()
