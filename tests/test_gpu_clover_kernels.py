"""``cloverinfer_b200.clover_kernels.paged_attention`` — the drop-in for the
reference's ``clover_kernels`` extension — driven exactly as the reference's
``KVCacheManager.attention`` drives it (src/core/memory_manager.py:175-190:
``get_kernel_inputs`` -> ``out = empty_like(q)`` -> ``paged_attention(out, q,
k_cache, v_cache, block_tables, ctx_lens, block_size, max_len)``), against the
oracle's restatement of ``_paged_attention_ref`` (:192-239) on the same
manager state.  Cases: the reference's own kernel check
(tests/verify_attention.py:88-136: fp16, block 16, 4 heads, head_dim 32, 50
tokens written one by one), a bf16 tensor-core case with split-K contexts, an
fp32 case, and native GQA (caches with fewer heads than q)."""

from __future__ import annotations

import pytest
import torch

from conftest import assert_attn_close, gpu
from oracle import KVCacheOracle, repeat_kv

pytestmark = gpu


def _manager(dtype, nb, bs, h, d, lens, seed):
    """An oracle manager holding `lens` tokens per request, filled in the
    reference's own way (load_initial_kv, then write_new_kv one token at a time)."""
    g = torch.Generator().manual_seed(seed)
    m = KVCacheOracle(nb, bs, h, d, dtype=dtype)
    perm = torch.randperm(nb, generator=g).tolist()
    m.free_blocks = perm  # non-contiguous tables
    ids = []
    for i, n in enumerate(lens):
        rid = f"r{i}"
        n0 = n // 2
        m.load_initial_kv(rid, torch.randn(n0, h, d, generator=g).to(dtype),
                          torch.randn(n0, h, d, generator=g).to(dtype))
        for _ in range(n - n0):
            m.write_new_kv(rid, torch.randn(h, d, generator=g).to(dtype),
                           torch.randn(h, d, generator=g).to(dtype))
        ids.append(rid)
    return m, ids


def _ref(m, q, ids):
    """The oracle's _paged_attention_ref in fp32: the same manager state with
    the caches widened (the upstream reference computes in the cache dtype)."""
    mf = KVCacheOracle(m.num_blocks, m.block_size, m.num_heads, m.head_dim, dtype=torch.float32,
                       with_storage=False)
    mf.k_cache, mf.v_cache = m.k_cache.float(), m.v_cache.float()
    mf.block_tables, mf.context_lens = m.block_tables, m.context_lens
    return mf.paged_attention_ref(q.float(), ids)


def _run(m, ids, q, kv_heads=None):
    from cloverinfer_b200 import clover_kernels
    dev = torch.device("cuda")
    kc, vc = m.k_cache, m.v_cache
    if kv_heads is not None:  # keep one head per group: the cache GQA models would store
        step = kc.shape[2] // kv_heads
        kc, vc = kc[:, :, ::step].contiguous(), vc[:, :, ::step].contiguous()
    block_tables, ctx_lens, max_len = m.get_kernel_inputs(ids)
    qd = q.to(dev)
    out = torch.empty_like(qd)
    clover_kernels.paged_attention(out, qd, kc.to(dev), vc.to(dev), block_tables.to(dev),
                                   ctx_lens.to(dev), m.block_size, max_len)
    assert clover_kernels.device_status(dev) == 0
    return out.cpu()


def test_reference_kernel_check_case():
    """tests/verify_attention.py:88-136 with allclose(1e-2, 1e-2) tightened to
    the north-star bound."""
    m, ids = _manager(torch.float16, 100, 16, 4, 32, [50], seed=1)
    q = torch.randn(1, 4, 32, generator=torch.Generator().manual_seed(2)).half()
    out = _run(m, ids, q)
    ref = _ref(m, q, ids)
    assert out.dtype == torch.float16
    assert_attn_close(out, ref, kv_dtype=torch.float16, out_dtype=torch.float16,
                      what="verify_attention case")


@pytest.mark.parametrize("dtype,d,lens", [
    (torch.bfloat16, 128, [1, 15, 16, 17, 700, 4096, 9000]),
    (torch.float32, 64, [5, 300, 1500]),
    (torch.float16, 128, [64, 2049]),
])
def test_manager_attention_matches_reference(dtype, d, lens):
    bs, h = 16, 8
    nb = sum(-(-(n + 1) // bs) for n in lens) + 8
    m, ids = _manager(dtype, nb, bs, h, d, lens, seed=3)
    q = torch.randn(len(lens), h, d, generator=torch.Generator().manual_seed(4)).to(dtype).float()
    out = _run(m, ids, q)
    ref = _ref(m, q, ids)
    assert_attn_close(out, ref, kv_dtype=dtype, what=f"paged_attention {dtype} D{d}")


def test_native_gqa_caches():
    bs, hq, hkv, d = 16, 16, 4, 128
    lens = [33, 1000, 5000]
    nb = sum(-(-(n + 1) // bs) for n in lens) + 4
    m, ids = _manager(torch.bfloat16, nb, bs, hkv, d, lens, seed=5)
    # the oracle's manager holds the repeat_kv expansion (one cache head per query head)
    mx = KVCacheOracle(nb, bs, hq, d, dtype=torch.bfloat16)
    mx.k_cache, mx.v_cache = repeat_kv(m.k_cache, hq // hkv), repeat_kv(m.v_cache, hq // hkv)
    mx.block_tables, mx.context_lens = m.block_tables, m.context_lens
    q = torch.randn(len(lens), hq, d, generator=torch.Generator().manual_seed(6)).bfloat16().float()
    out = _run(mx, ids, q, kv_heads=hkv)
    assert_attn_close(out, _ref(mx, q, ids), kv_dtype=torch.bfloat16, what="GQA caches")
