"""The C-ABI library builds for sm_100a, loads, and exports every symbol the
public header declares; argument validation answers with error codes (no
GPU work is issued by these checks)."""

from __future__ import annotations

import ctypes
import os
import re

from conftest import ROOT

from cloverinfer_b200 import _lib


def _declared_symbols():
    with open(os.path.join(ROOT, "include", "clover_b200.h")) as f:
        text = f.read()
    return sorted(set(re.findall(r"\b(clover_b200_[a-z0-9_]+)\s*\(", text)))


def test_header_and_binding_agree():
    assert _declared_symbols() == sorted(_lib.SIGNATURES)


def test_library_exports_every_symbol():
    lib = _lib.lib()
    for name in _declared_symbols():
        assert hasattr(lib, name), name
        assert ctypes.cast(getattr(lib, name), ctypes.c_void_p).value


def test_version_and_errors():
    lib = _lib.lib()
    assert lib.clover_b200_version() >= 100
    rc = lib.clover_b200_block_reserve(None, None, 16, None, -1, None, None, None, 1, 16, None, None)
    assert rc == _lib.ERR_INVALID_ARG
    assert b"bad sizes" in lib.clover_b200_last_error()
    rc = lib.clover_b200_kv_append(None, None, None, None, 0, None, 1, 1, 64, 16, 4, 7, None, None)
    assert rc == _lib.ERR_INVALID_ARG  # null pointers are rejected before the dtype
    rc = lib.clover_b200_paged_decode(
        None, 0, None, 0, 0, None, None, 2, 1, 16, None, 1, None, None, None,
        1, 1, 1, 16, 6, 4, 64, 1.0, 0, None, 0, None, None)
    assert rc == _lib.ERR_INVALID_ARG
    # zero-sized batches are valid no-ops
    assert lib.clover_b200_kv_append(None, None, None, None, 0, None, 0, 1, 64, 16, 4, 2, None, None) == 0


def test_workspace_bytes():
    lib = _lib.lib()
    BF16, F32 = _lib.BF16, _lib.F32
    # contexts within one partition need no workspace
    assert lib.clover_b200_decode_workspace_bytes(8, 8, 1, 512, 32, 8, 128, 16, BF16, F32, 512) == 0
    nb = lib.clover_b200_decode_workspace_bytes(8, 8, 1, 32768, 32, 8, 128, 16, BF16, F32, 512)
    assert nb >= 8 * 32 * 64 * 129 * 4
    assert lib.clover_b200_decode_workspace_bytes(-1, 8, 1, 1, 32, 8, 128, 16, BF16, F32, 0) < 0
    assert lib.clover_b200_decode_workspace_bytes(8, 8, 1, 1, 30, 8, 128, 16, BF16, F32, 0) < 0


def test_sources_target_sm100a_only():
    from cloverinfer_b200 import build
    assert build.ARCH_FLAGS == ["-gencode", "arch=compute_100a,code=sm_100a"]
    files = [os.path.join(build.CSRC, f) for f in os.listdir(build.CSRC)
             if f.endswith((".cu", ".cuh"))]
    srcs = "".join(open(p).read() for p in files)
    assert "cp.async.bulk.tensor" in srcs and "mma.sync" in srcs


def test_no_alloc_reports_the_plan_error():
    """The allocation-free decode returns the code the regular entry point
    returns for the same unsupported request (an fp8 cache at head_dim 64),
    not a generic invalid-argument code.  No GPU work is issued."""
    lib = _lib.lib()
    args = (None, 0, None, 0, _lib.F32, None, None, _lib.FP8_E4M3, 1, 16, None, 1, None, None, None,
            1, 1, 1, 4096, 8, 2, 64, 1.0, 0)
    rc = lib.clover_b200_paged_decode(*args, None, 0, None, None)
    assert rc == _lib.ERR_UNSUPPORTED
    rc2 = lib.clover_b200_paged_decode_noalloc(*args, None, None)
    assert rc2 == rc
    assert b"fp8" in lib.clover_b200_last_error()


def test_wait_limit_setter_round_trips():
    lib = _lib.lib()
    prev = _lib.set_wait_limit_ns(5_000_000)
    try:
        assert _lib.set_wait_limit_ns(1) == 5_000_000      # clamped up to 1 ms next
        assert _lib.set_wait_limit_ns(0) == 1_000_000      # 0 restores the default
        assert _lib.set_wait_limit_ns(10 ** 15) == 1_000_000_000
        assert lib.clover_b200_set_wait_limit_ns(prev) == 60 * 10 ** 9
    finally:
        _lib.set_wait_limit_ns(prev)


def test_clover_kernels_shim_rejects_bad_shapes_on_cpu():
    """The clover_kernels stand-in validates arguments before any GPU work."""
    import pytest
    import torch
    from cloverinfer_b200 import clover_kernels
    q = torch.zeros(2, 4, 32)
    kc = torch.zeros(8, 16, 4, 32)
    with pytest.raises(ValueError):
        clover_kernels.paged_attention(torch.zeros(3, 4, 32), q, kc, kc, torch.zeros(2, 1, dtype=torch.int32),
                                       torch.ones(2, dtype=torch.int32), 16, 1)
    with pytest.raises(ValueError):
        clover_kernels.paged_attention(torch.zeros_like(q), q, kc, kc, torch.zeros(2, 1, dtype=torch.int32),
                                       torch.ones(2, dtype=torch.int32), 8, 1)


def test_append_layers_strides_checked():
    """Overlapping layer strides are rejected before any launch (no GPU work)."""
    lib = _lib.lib()
    rc = lib.clover_b200_kv_append_layers(1 << 12, 1 << 13, 16, 1 << 14, 1 << 15, 8, 128, 1 << 16, 4, 2,
                                          1, 128, 16, 8, _lib.BF16, None, None)
    assert rc == _lib.ERR_INVALID_ARG
    assert b"overlap" in lib.clover_b200_last_error()
