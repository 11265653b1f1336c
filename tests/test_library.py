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
