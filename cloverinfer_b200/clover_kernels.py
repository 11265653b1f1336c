"""``clover_kernels``-compatible module over the B200 library.

CloverInfer's ``KVCacheManager.attention`` imports an extension module named
``clover_kernels`` and, when it is present and the manager lives on a GPU,
calls (src/core/memory_manager.py:6-11, :175-190)::

    clover_kernels.paged_attention(out, q, k_cache, v_cache, block_tables,
                                   context_lens, block_size, max_context_len)

with the signature bound in src/kernels/csrc/manager.cpp:19-42: ``out`` and
``q`` ``[num_seqs, num_heads, head_dim]``, caches
``[num_blocks, block_size, num_heads, head_dim]``, ``block_tables``
``[num_seqs, max_blocks]`` int32 padded with -1, ``context_lens [num_seqs]``
int32, the scale fixed at ``1/sqrt(head_dim)`` (attention.cu:60).  This module
provides that function on the sm_100a decode (``clover_b200_paged_decode``), so
the reference's own manager runs on it unchanged once the module is importable
under that name::

    import sys, cloverinfer_b200.clover_kernels as ck
    sys.modules["clover_kernels"] = ck          # before importing core.memory_manager

Same argument meaning and in-place output; differences: fp32 accumulation of
the output (upstream accumulates it in the storage type, attention.cu:101-106),
bf16 accepted, native GQA when the caches hold fewer heads than ``q`` (a
multiple), and malformed arguments raise ``ValueError``.  Like the upstream
call it does not synchronise: a table entry outside the cache is skipped on
the device and recorded in a per-device status word that
``device_status(device)`` reads (and clears).  The split-K workspace is
allocated here per device and reused.
"""

from __future__ import annotations

import math
from typing import Dict

import torch

from . import _lib

_workspaces: Dict[int, torch.Tensor] = {}
_status: Dict[int, torch.Tensor] = {}


def _index(device: torch.device) -> int:
    return device.index if device.index is not None else torch.cuda.current_device()


def _status_word(device: torch.device) -> torch.Tensor:
    idx = _index(device)
    st = _status.get(idx)
    if st is None:
        st = torch.zeros(1, dtype=torch.int32, device=device)
        _status[idx] = st
    return st


def device_status(device=None) -> int:
    """CLOVER_B200_DEV_* bits raised by paged_attention calls on ``device``
    since the last read (synchronises; clears the word)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    st = _status_word(dev)
    code = int(st.item())
    st.zero_()
    return code


def _workspace(device: torch.device, nbytes: int):
    if nbytes <= 0:
        return None
    idx = _index(device)
    ws = _workspaces.get(idx)
    if ws is None or ws.numel() < nbytes:
        ws = torch.empty(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _workspaces[idx] = ws
    return ws


def paged_attention(out: torch.Tensor, q: torch.Tensor, k_cache: torch.Tensor,
                    v_cache: torch.Tensor, block_tables: torch.Tensor, context_lens: torch.Tensor,
                    block_size: int, max_context_len: int) -> None:
    """Paged decode attention into ``out`` (manager.cpp:19-38 semantics)."""
    if q.dim() != 3 or out.shape != q.shape:
        raise ValueError(f"paged_attention: q/out must be [num_seqs, num_heads, head_dim], "
                         f"got {tuple(q.shape)} / {tuple(out.shape)}")
    if k_cache.dim() != 4 or v_cache.shape != k_cache.shape:
        raise ValueError("paged_attention: caches must be [num_blocks, block_size, heads, head_dim]")
    if int(k_cache.shape[1]) != int(block_size):
        raise ValueError(f"paged_attention: block_size {block_size} != cache block dim {k_cache.shape[1]}")
    n, h, d = (int(x) for x in q.shape)
    if n == 0:
        return
    if block_tables.dim() != 2 or block_tables.shape[0] != n or context_lens.numel() != n:
        raise ValueError("paged_attention: block_tables / context_lens do not match num_seqs")
    dev = q.device
    tables = block_tables if block_tables.dtype == torch.int32 else block_tables.to(torch.int32)
    lens = context_lens if context_lens.dtype == torch.int32 else context_lens.to(torch.int32)
    tables, lens = tables.contiguous(), lens.contiguous()
    qc = q if q.stride(2) == 1 and q.stride(1) == d else q.contiguous()
    dst = out if out.stride(2) == 1 and out.stride(1) == d else torch.empty_like(qc)
    qsl = torch.arange(n + 1, dtype=torch.int32, device=dev)
    max_len = int(max_context_len)
    nbytes = _lib.decode_workspace_bytes(n, n, 1, max_len, h, int(k_cache.shape[2]), d, int(block_size),
                                         k_cache.dtype, qc.dtype)
    _lib.paged_decode(dst, qc, k_cache, v_cache, tables, qsl, lens, max_queries_per_seq=1,
                      max_ctx_len=max_len, score_scale=1.0 / math.sqrt(d),
                      workspace=_workspace(dev, nbytes), status=_status_word(dev))
    if dst is not out:
        out.copy_(dst)
