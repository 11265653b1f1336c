"""The allocation-free decode entry point, called through the C ABI.

``clover_b200_paged_decode_noalloc`` is for callers that cannot call
cudaMalloc — an engine whose memory pool owns all of HBM, or a host behind a
foreign-function binding with no CUDA allocator — so it takes its split-K
scratch from a static device array instead of a caller workspace.  Its output
must match the regular entry point (with a caller workspace) on the same
inputs, on two calls in a row (the second call reuses the array the first one
left filled), and it must refuse work that needs more scratch than the array.
This file is collected last so a failure here never hides another test.
"""

from __future__ import annotations

import ctypes
import math

import pytest
import torch

from conftest import assert_attn_close, gpu

pytestmark = gpu


def _case(seed, lens, hq=32, hkv=8, D=128, bs=16, dt=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    nblk = [-(-n // bs) for n in lens]
    nb = sum(nblk) + 5
    dev = "cuda"
    kc = torch.randn(nb, bs, hkv, D, generator=g).to(dt).to(dev)
    vc = torch.randn(nb, bs, hkv, D, generator=g).to(dt).to(dev)
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    tables = torch.full((len(lens), max(nblk)), -1, dtype=torch.int32)
    o = 0
    for i, k in enumerate(nblk):
        tables[i, :k] = perm[o:o + k]
        o += k
    q = torch.randn(len(lens), hq, D, generator=g).to(dt).float().to(dev)
    return dict(kc=kc, vc=vc, tables=tables.to(dev), q=q,
                qsl=torch.arange(len(lens) + 1, dtype=torch.int32, device=dev),
                ctx=torch.tensor(lens, dtype=torch.int32, device=dev),
                lens=lens, hq=hq, hkv=hkv, D=D, bs=bs, dt=dt, nb=nb)


def _with_workspace(c, pt):
    """The regular entry point with a fresh workspace filled with NaN bytes, so
    a partial that a call forgets to write cannot pass for a correct one."""
    from cloverinfer_b200 import _lib
    out = torch.empty_like(c["q"])
    need = _lib.decode_workspace_bytes(len(c["lens"]), len(c["lens"]), 1, max(c["lens"]), c["hq"],
                                       c["hkv"], c["D"], c["bs"], c["dt"], c["q"].dtype, pt)
    ws = torch.full((max(need, 1),), 255, dtype=torch.uint8, device="cuda")
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.paged_decode(out, c["q"], c["kc"], c["vc"], c["tables"], c["qsl"], c["ctx"],
                      max_queries_per_seq=1, max_ctx_len=max(c["lens"]),
                      score_scale=1 / math.sqrt(c["D"]), partition_tokens=pt, workspace=ws, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0 and need > 0  # the case must exercise split-K scratch
    return out


def _no_alloc(c, pt, out=None):
    from cloverinfer_b200 import _lib
    lib = _lib.lib()
    out = torch.full_like(c["q"], float("nan")) if out is None else out
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    rc = lib.clover_b200_paged_decode_noalloc(
        out.data_ptr(), out.stride(0), c["q"].data_ptr(), c["q"].stride(0), _lib.F32,
        c["kc"].data_ptr(), c["vc"].data_ptr(), _lib.BF16, c["nb"], c["bs"],
        c["tables"].data_ptr(), c["tables"].stride(0), None, c["qsl"].data_ptr(), c["ctx"].data_ptr(),
        len(c["lens"]), len(c["lens"]), 1, max(c["lens"]), c["hq"], c["hkv"], c["D"],
        1 / math.sqrt(c["D"]), pt, st.data_ptr(), torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    return rc, out, int(st.item())


def test_no_alloc_matches_workspace_entry_point_twice():
    from cloverinfer_b200 import _lib
    first = _case(1, [4096, 1500, 700, 33, 2600, 9000, 64, 512])
    second = _case(2, [300, 5000, 129, 12000])
    for c, pt in [(first, 512), (second, 256)]:
        ref = _with_workspace(c, pt)
        rc, out, st = _no_alloc(c, pt)
        assert rc == _lib.OK, _lib.lib().clover_b200_last_error()
        assert st == 0
        assert_attn_close(out, ref, kv_dtype=torch.bfloat16, what=f"no-alloc vs workspace pt={pt}")


def test_no_alloc_balanced_split_twice():
    """The balanced split keeps per-(row, head) part counts in the shared array
    too: a second, more ragged call with fewer rows and an empty context must
    not read the first call's counts or partials."""
    from cloverinfer_b200 import _lib
    # sized to fit the static scratch: the balanced plan bounds the parts of a
    # (row, head) by the resident warps per KV head, not by the batch's work
    first = _case(3, [4096, 1500, 9000, 33])
    second = _case(4, [0, 40, 3000])
    for c in (first, second):
        ref = _with_workspace(c, _lib.PARTITION_BALANCED)
        rc, out, st = _no_alloc(c, _lib.PARTITION_BALANCED)
        assert rc == _lib.OK, _lib.lib().clover_b200_last_error()
        assert st == 0
        if c is second:
            assert bool((out[0] == 0).all())  # the empty context reads 0
        assert_attn_close(out, ref, kv_dtype=torch.bfloat16, what="no-alloc vs workspace, balanced")


def test_no_alloc_rejects_oversized_scratch():
    from cloverinfer_b200 import _lib
    lens = [65536] * 64  # 64 rows x 32 heads x 1024 partitions x 129 floats >> 16 MiB
    c = dict(q=torch.zeros(64, 32, 128, device="cuda"), kc=torch.zeros(1, 16, 8, 128, dtype=torch.bfloat16, device="cuda"),
             lens=lens, hq=32, hkv=8, D=128, bs=16, nb=1,
             tables=torch.zeros(64, 1, dtype=torch.int32, device="cuda"),
             qsl=torch.arange(65, dtype=torch.int32, device="cuda"),
             ctx=torch.full((64,), 65536, dtype=torch.int32, device="cuda"))
    c["vc"] = c["kc"]
    out = torch.zeros_like(c["q"])
    rc, out, st = _no_alloc(c, 64, out=out)
    assert rc == _lib.ERR_WORKSPACE
    assert b"exceeds the static maximum" in _lib.lib().clover_b200_last_error()
    assert st == 0 and bool((out == 0).all())  # nothing ran
