"""ctypes binding of libclover_b200.so and thin tensor-level wrappers.

The library is the C ABI declared in ``include/clover_b200.h``.  Loading it
builds it in-tree first when the sources changed (nvcc, sm_100a).  There is no
fallback: if the library cannot be built or loaded, every op raises.
"""

from __future__ import annotations

import ctypes
import fcntl
import os
import threading
from typing import Optional

import torch

from . import build as _build

OK = 0
ERR_INVALID_ARG = -1
ERR_UNSUPPORTED = -2
ERR_CUDA = -3
ERR_WORKSPACE = -4

DEV_BAD_SLOT = 0x1
DEV_BAD_BLOCK = 0x2
DEV_TABLE_FULL = 0x4
DEV_OOM = 0x8
DEV_TIMEOUT = 0x10
DEV_CTX_RANGE = 0x20

PARTITION_BALANCED = -1  # CLOVER_B200_PARTITION_BALANCED: the balanced split

F32, F16, BF16, FP8_E4M3 = 0, 1, 2, 3
_DTYPE = {torch.float32: F32, torch.float16: F16, torch.bfloat16: BF16,
          torch.float8_e4m3fn: FP8_E4M3}  # fp8: KV caches only

# Every symbol include/clover_b200.h declares: name -> (restype, argtypes)
_P = ctypes.c_void_p
_I32 = ctypes.c_int32
_I64 = ctypes.c_int64
_F = ctypes.c_float
SIGNATURES = {
    "clover_b200_version": (ctypes.c_int, []),
    "clover_b200_last_error": (ctypes.c_char_p, []),
    "clover_b200_set_wait_limit_ns": (ctypes.c_int64, [_I64]),
    "clover_b200_host_gather": (ctypes.c_int, [_P, _P, _I32, _P]),
    "clover_b200_block_reserve": (ctypes.c_int, [_P, _P, _I32, _P, _I32, _P, _P, _P, _I32, _I32, _P, _P]),
    "clover_b200_block_free": (ctypes.c_int, [_P, _P, _I32, _P, _I32, _P, _P, _I32, _P, _P]),
    "clover_b200_compute_slots": (ctypes.c_int, [_P, _I32, _P, _P, _P, _I32, _I32, _I64, _P, _P, _P]),
    "clover_b200_kv_append": (ctypes.c_int, [_P, _P, _P, _P, _I64, _P, _I64, _I32, _I32, _I32, _I64, _I32, _P, _P]),
    "clover_b200_kv_append_layers": (ctypes.c_int, [_P, _P, _I64, _P, _P, _I64, _I64, _P, _I64, _I32,
                                                    _I32, _I32, _I32, _I64, _I32, _P, _P]),
    "clover_b200_decode_workspace_bytes": (ctypes.c_int64, [_I32] * 11),
    "clover_b200_decode_partition_tokens": (ctypes.c_int, [_I32] * 11),
    "clover_b200_paged_decode": (ctypes.c_int, [
        _P, _I64, _P, _I64, _I32, _P, _P, _I32, _I64, _I32, _P, _I32, _P, _P, _P,
        _I32, _I32, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _I64, _P, _P]),
    "clover_b200_decode_step": (ctypes.c_int, [
        _P, _I64, _P, _I64, _I32, _P, _P, _I32, _I64, _I32, _P, _P, _I64, _P, _I32, _P, _P, _P,
        _I32, _I32, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _I64, _P, _P]),
    "clover_b200_ipc_alloc": (ctypes.c_int, [_I64, _P, _P]),
    "clover_b200_ipc_open": (ctypes.c_int, [_P, _P]),
    "clover_b200_ipc_close": (ctypes.c_int, [_P]),
    "clover_b200_ipc_free": (ctypes.c_int, [_P]),
    "clover_b200_gather_sync_bytes": (ctypes.c_int64, []),
    "clover_b200_decode_gather_workspace_bytes": (ctypes.c_int64, [_I32] * 11),
    "clover_b200_decode_step_gather": (ctypes.c_int, [
        _P, _I64, _P, _I64, _I32, _P, _P, _I32, _I64, _I32, _P, _P, _I64, _P, _I32, _P, _P, _P,
        _I32, _I32, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _P, _I32, _I32, _I64, _P, _I64,
        _P, _P]),
    "clover_b200_decode_step_gather_into": (ctypes.c_int, [
        _P, _I64, _I32, _P, _I64, _I32, _P, _P, _I32, _I64, _I32, _P, _P, _I64, _P, _I32, _P, _P, _P,
        _I32, _I32, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _P, _I32, _I32, _I64, _P, _I64,
        _P, _P]),
    "clover_b200_paged_decode_noalloc": (ctypes.c_int, [
        _P, _I64, _P, _I64, _I32, _P, _P, _I32, _I64, _I32, _P, _I32, _P, _P, _P,
        _I32, _I32, _I32, _I32, _I32, _I32, _I32, _F, _I32, _P, _P]),
}
NOALLOC_SCRATCH_BYTES = 16 << 20  # CLOVER_B200_NOALLOC_SCRATCH_BYTES


class CloverB200Error(RuntimeError):
    """A libclover_b200 entry point returned an error code."""


_lib: Optional[ctypes.CDLL] = None
_lock = threading.Lock()


def _build_locked() -> str:
    os.makedirs(_build.OUT_DIR, exist_ok=True)
    with open(os.path.join(_build.OUT_DIR, ".build.lock"), "w") as lk:
        fcntl.flock(lk, fcntl.LOCK_EX)
        try:
            return _build.build()
        finally:
            fcntl.flock(lk, fcntl.LOCK_UN)


def lib() -> ctypes.CDLL:
    """Load (building if needed) the CUDA library; raises if impossible."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = _build.LIB_PATH
            if not _build.up_to_date():
                path = _build_locked()
            handle = ctypes.CDLL(path)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def lib_path() -> str:
    return _build.LIB_PATH


def _check(rc: int, what: str) -> None:
    if rc != OK:
        msg = lib().clover_b200_last_error().decode(errors="replace")
        raise CloverB200Error(f"{what} failed ({rc}): {msg}")


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DTYPE[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require_cuda(*ts: Optional[torch.Tensor]) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("libclover_b200 ops take CUDA tensors")


# ---------------------------------------------------------------- allocator
def block_reserve(free_stack, free_top, tables, table_len, rows, target_tokens, block_size, status):
    _require_cuda(free_stack, free_top, tables, table_len, rows, target_tokens, status)
    rc = lib().clover_b200_block_reserve(
        _ptr(free_stack), _ptr(free_top), free_stack.numel(), _ptr(tables), tables.shape[1],
        _ptr(table_len), _ptr(rows), _ptr(target_tokens), rows.numel(), block_size,
        _ptr(status), _stream(free_stack.device))
    _check(rc, "clover_b200_block_reserve")


def block_free(free_stack, free_top, tables, table_len, rows, status):
    _require_cuda(free_stack, free_top, tables, table_len, rows, status)
    rc = lib().clover_b200_block_free(
        _ptr(free_stack), _ptr(free_top), free_stack.numel(), _ptr(tables), tables.shape[1],
        _ptr(table_len), _ptr(rows), rows.numel(), _ptr(status), _stream(free_stack.device))
    _check(rc, "clover_b200_block_free")


def compute_slots(tables, rows, positions, token_offsets, block_size, num_blocks, slot_mapping, status):
    _require_cuda(tables, rows, positions, token_offsets, slot_mapping, status)
    rc = lib().clover_b200_compute_slots(
        _ptr(tables), tables.shape[1], _ptr(rows), _ptr(positions), _ptr(token_offsets),
        rows.numel(), block_size, num_blocks, _ptr(slot_mapping), _ptr(status),
        _stream(tables.device))
    _check(rc, "clover_b200_compute_slots")


# ---------------------------------------------------------------- KV append
def kv_append(k_cache, v_cache, k_new, v_new, slot_mapping, status):
    """k_cache/v_cache [num_blocks, bs, H, D]; k_new/v_new [n, H, D] (token stride free)."""
    _require_cuda(k_cache, v_cache, k_new, v_new, slot_mapping, status)
    nb, bs, h, d = k_cache.shape
    if k_new.dtype != k_cache.dtype or v_new.dtype != v_cache.dtype:
        raise TypeError("kv_append: new K/V dtype must match the cache dtype")
    if k_new.shape[1:] != (h, d) or v_new.shape != k_new.shape:
        raise ValueError(f"kv_append: new K/V shape {tuple(k_new.shape)} != [n, {h}, {d}]")
    if k_new.stride(2) != 1 or k_new.stride(1) != d or v_new.stride() != k_new.stride():
        raise ValueError("kv_append: each token's [H, D] row must be contiguous")
    rc = lib().clover_b200_kv_append(
        _ptr(k_cache), _ptr(v_cache), _ptr(k_new), _ptr(v_new), k_new.stride(0),
        _ptr(slot_mapping), k_new.shape[0], h, d, bs, nb, dtype_code(k_cache.dtype),
        _ptr(status), _stream(k_cache.device))
    _check(rc, "clover_b200_kv_append")


def kv_append_layers(k_layers, v_layers, k_new, v_new, slot_mapping, status):
    """Every layer at once: caches [L, num_blocks, bs, H, D]; k_new/v_new
    [L, n, H, D] views (layer and token strides free, each token's [H, D]
    contiguous), one launch."""
    _require_cuda(k_layers, v_layers, k_new, v_new, slot_mapping, status)
    L, nb, bs, h, d = k_layers.shape
    if k_new.dim() != 4 or k_new.shape[0] != L or k_new.shape[2:] != (h, d) or v_new.shape != k_new.shape:
        raise ValueError(f"kv_append_layers: new K/V {tuple(k_new.shape)} != [{L}, n, {h}, {d}]")
    if k_new.dtype != k_layers.dtype or v_new.dtype != k_layers.dtype:
        raise TypeError("kv_append_layers: new K/V dtype must match the cache dtype")
    if (k_new.stride(3) != 1 or k_new.stride(2) != d or v_new.stride() != k_new.stride()
            or not k_layers.is_contiguous() or not v_layers.is_contiguous()):
        raise ValueError("kv_append_layers: token rows and caches must be contiguous")
    rc = lib().clover_b200_kv_append_layers(
        _ptr(k_layers), _ptr(v_layers), k_layers.stride(0), _ptr(k_new), _ptr(v_new), k_new.stride(0),
        k_new.stride(1), _ptr(slot_mapping), k_new.shape[1], L, h, d, bs, nb,
        dtype_code(k_layers.dtype), _ptr(status), _stream(k_layers.device))
    _check(rc, "clover_b200_kv_append_layers")


# ---------------------------------------------------------------- decode
def decode_workspace_bytes(n_seqs, n_rows, max_queries_per_seq, max_ctx_len, num_q_heads,
                           num_kv_heads, head_dim, block_size, kv_dtype, q_dtype,
                           partition_tokens=0) -> int:
    nb = int(lib().clover_b200_decode_workspace_bytes(
        n_seqs, n_rows, max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads, head_dim,
        block_size, dtype_code(kv_dtype), dtype_code(q_dtype), partition_tokens))
    if nb < 0:
        raise CloverB200Error(lib().clover_b200_last_error().decode(errors="replace"))
    return nb


def decode_partition_tokens(n_seqs, n_rows, max_queries_per_seq, max_ctx_len, num_q_heads,
                            num_kv_heads, head_dim, block_size, kv_dtype, q_dtype,
                            partition_tokens=0) -> int:
    """Partition length the call would use; 0 for the balanced split."""
    pt = int(lib().clover_b200_decode_partition_tokens(
        n_seqs, n_rows, max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads, head_dim,
        block_size, dtype_code(kv_dtype), dtype_code(q_dtype), partition_tokens))
    _check(OK if pt > 0 else pt, "clover_b200_decode_partition_tokens")
    return pt


def paged_decode(out, q, k_cache, v_cache, block_tables, query_start_loc, ctx_lens, *,
                 max_queries_per_seq, max_ctx_len, score_scale, seq_rows=None,
                 partition_tokens=0, workspace=None, status=None):
    """q/out [rows, Hq, D] (row stride free); caches [num_blocks, bs, Hkv, D]."""
    _require_cuda(out, q, k_cache, v_cache, block_tables, query_start_loc, ctx_lens, seq_rows,
                  workspace, status)
    nb, bs, hkv, d = k_cache.shape
    rows, hq, dq = q.shape
    if dq != d or out.shape != q.shape:
        raise ValueError("paged_decode: q/out shape mismatch")
    if q.stride(2) != 1 or q.stride(1) != d or out.stride(2) != 1 or out.stride(1) != d:
        raise ValueError("paged_decode: each row's [Hq, D] must be contiguous")
    if out.dtype != q.dtype:
        raise TypeError("paged_decode: out dtype must equal q dtype")
    for t in (block_tables, query_start_loc, ctx_lens) + ((seq_rows,) if seq_rows is not None else ()):
        if t.dtype != torch.int32 or not t.is_contiguous():
            raise TypeError("paged_decode: index tensors must be contiguous int32")
    n_seqs = query_start_loc.numel() - 1
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = lib().clover_b200_paged_decode(
        _ptr(out), out.stride(0), _ptr(q), q.stride(0), dtype_code(q.dtype),
        _ptr(k_cache), _ptr(v_cache), dtype_code(k_cache.dtype), nb, bs,
        _ptr(block_tables), block_tables.stride(0), _ptr(seq_rows), _ptr(query_start_loc),
        _ptr(ctx_lens), n_seqs, rows, max_queries_per_seq, max_ctx_len, hq, hkv, d,
        float(score_scale), partition_tokens, _ptr(workspace), ws_bytes, _ptr(status),
        _stream(q.device))
    _check(rc, "clover_b200_paged_decode")


def decode_step(out, q, k_cache, v_cache, k_new, v_new, block_tables, query_start_loc, ctx_lens, *,
                max_queries_per_seq, max_ctx_len, score_scale, seq_rows=None,
                partition_tokens=0, workspace=None, status=None, check=True):
    """Append row r's new token (k_new/v_new[r], [n_rows, Hkv, D]) at ctx_lens[r]-1, then
    paged decode as :func:`paged_decode` — one launch when the append can be fused.
    ``check=False`` skips the Python-side shape checks (callers that built the
    tensors themselves); the library still validates sizes and pointers."""
    nb, bs, hkv, d = k_cache.shape
    rows, hq, dq = q.shape
    if not check:
        ws_bytes = 0 if workspace is None else workspace.numel()
        rc = lib().clover_b200_decode_step(
            out.data_ptr(), out.stride(0), q.data_ptr(), q.stride(0), _DTYPE[q.dtype],
            k_cache.data_ptr(), v_cache.data_ptr(), _DTYPE[k_cache.dtype], nb, bs,
            k_new.data_ptr(), v_new.data_ptr(), k_new.stride(0), block_tables.data_ptr(),
            block_tables.stride(0), _ptr(seq_rows), query_start_loc.data_ptr(), ctx_lens.data_ptr(),
            query_start_loc.numel() - 1, rows, max_queries_per_seq, max_ctx_len, hq, hkv, d,
            float(score_scale), partition_tokens, _ptr(workspace), ws_bytes, _ptr(status),
            torch.cuda.current_stream(q.device).cuda_stream)
        if rc != OK:
            _check(rc, "clover_b200_decode_step")
        return
    _require_cuda(out, q, k_cache, v_cache, k_new, v_new, block_tables, query_start_loc,
                  ctx_lens, seq_rows, workspace, status)
    if dq != d or out.shape != q.shape or out.dtype != q.dtype:
        raise ValueError("decode_step: q/out mismatch")
    if k_new.shape != (rows, hkv, d) or v_new.shape != k_new.shape:
        raise ValueError(f"decode_step: new K/V must be [{rows}, {hkv}, {d}]")
    if k_new.dtype != k_cache.dtype or v_new.dtype != k_cache.dtype:
        raise TypeError("decode_step: new K/V dtype must match the cache")
    if k_new.stride(2) != 1 or k_new.stride(1) != d or v_new.stride() != k_new.stride():
        raise ValueError("decode_step: each token's [Hkv, D] row must be contiguous")
    if q.stride(2) != 1 or q.stride(1) != d or out.stride(2) != 1 or out.stride(1) != d:
        raise ValueError("decode_step: each row's [Hq, D] must be contiguous")
    n_seqs = query_start_loc.numel() - 1
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    rc = lib().clover_b200_decode_step(
        _ptr(out), out.stride(0), _ptr(q), q.stride(0), dtype_code(q.dtype),
        _ptr(k_cache), _ptr(v_cache), dtype_code(k_cache.dtype), nb, bs,
        _ptr(k_new), _ptr(v_new), k_new.stride(0),
        _ptr(block_tables), block_tables.stride(0), _ptr(seq_rows), _ptr(query_start_loc),
        _ptr(ctx_lens), n_seqs, rows, max_queries_per_seq, max_ctx_len, hq, hkv, d,
        float(score_scale), partition_tokens, _ptr(workspace), ws_bytes, _ptr(status),
        _stream(q.device))
    _check(rc, "clover_b200_decode_step")


# ---------------------------------------------------------------- peer memory / fused gather
IPC_HANDLE_BYTES = 64


def ipc_alloc(nbytes: int):
    """(device pointer, 64-byte IPC handle) of a zeroed cudaMalloc buffer."""
    ptr = ctypes.c_void_p()
    h = ctypes.create_string_buffer(IPC_HANDLE_BYTES)
    _check(lib().clover_b200_ipc_alloc(nbytes, ctypes.byref(ptr), h), "clover_b200_ipc_alloc")
    return int(ptr.value), bytes(h.raw)


def ipc_open(handle: bytes) -> int:
    ptr = ctypes.c_void_p()
    h = ctypes.create_string_buffer(handle, IPC_HANDLE_BYTES)
    _check(lib().clover_b200_ipc_open(h, ctypes.byref(ptr)), "clover_b200_ipc_open")
    return int(ptr.value)


def ipc_close(ptr: int) -> None:
    _check(lib().clover_b200_ipc_close(ptr), "clover_b200_ipc_close")


def ipc_free(ptr: int) -> None:
    _check(lib().clover_b200_ipc_free(ptr), "clover_b200_ipc_free")


def gather_sync_bytes() -> int:
    return int(lib().clover_b200_gather_sync_bytes())


def decode_gather_workspace_bytes(n_seqs, n_rows, max_queries_per_seq, max_ctx_len, num_q_heads,
                                  num_kv_heads, head_dim, block_size, kv_dtype, q_dtype,
                                  partition_tokens=0) -> int:
    nb = int(lib().clover_b200_decode_gather_workspace_bytes(
        n_seqs, n_rows, max_queries_per_seq, max_ctx_len, num_q_heads, num_kv_heads, head_dim,
        block_size, dtype_code(kv_dtype), dtype_code(q_dtype), partition_tokens))
    if nb < 0:
        raise CloverB200Error(lib().clover_b200_last_error().decode(errors="replace"))
    return nb


def decode_step_gather(q, k_cache, v_cache, k_new, v_new, block_tables, query_start_loc, ctx_lens,
                       gather, *, max_queries_per_seq, max_ctx_len, score_scale, seq_rows=None,
                       partition_tokens=0, workspace=None, status=None, out=None):
    """decode_step whose output, all-gathered over every rank of ``gather`` (a
    PeerGather), lands in ``out`` ([rows, Hq_total, D] in f32/f16/bf16, any
    row stride, each row's heads contiguous: e.g. a view of the consumer's
    [rows, Hq_total * D] input in the model's dtype), by default
    ``gather.out[:rows]``."""
    out = gather.out if out is None else out
    _require_cuda(q, k_cache, v_cache, k_new, v_new, block_tables, query_start_loc, ctx_lens,
                  seq_rows, workspace, status, out)
    nb, bs, hkv, d = k_cache.shape
    rows, hq, dq = q.shape
    if dq != d or q.stride(2) != 1 or q.stride(1) != d:
        raise ValueError("decode_step_gather: q must be [rows, Hq_local, D] with contiguous rows")
    if (out.dtype not in (torch.float32, torch.float16, torch.bfloat16) or out.dim() != 3
            or rows > out.shape[0] or hq * gather.world != out.shape[1] or out.shape[2] != d
            or out.stride(2) != 1 or out.stride(1) != d):
        raise ValueError("decode_step_gather: out must be [>= rows, Hq_local * world, D] "
                         "(f32/f16/bf16) with each row's heads contiguous")
    if rows * hq * gather.world * d > gather.half_words:
        raise ValueError("decode_step_gather: more rows than the gather buffers hold")
    if k_new is not None and (k_new.shape != (rows, hkv, d) or v_new.shape != k_new.shape
                              or k_new.dtype != k_cache.dtype):
        raise ValueError("decode_step_gather: new K/V must be [rows, Hkv_local, D] in the cache dtype")
    n_seqs = query_start_loc.numel() - 1
    ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
    if out.dtype != q.dtype:
        rc = lib().clover_b200_decode_step_gather_into(
            _ptr(out), out.stride(0), dtype_code(out.dtype), _ptr(q), q.stride(0), dtype_code(q.dtype),
            _ptr(k_cache), _ptr(v_cache), dtype_code(k_cache.dtype), nb, bs, _ptr(k_new), _ptr(v_new),
            0 if k_new is None else k_new.stride(0), _ptr(block_tables), block_tables.stride(0),
            _ptr(seq_rows), _ptr(query_start_loc), _ptr(ctx_lens), n_seqs, rows,
            max_queries_per_seq, max_ctx_len, hq, hkv, d, float(score_scale), partition_tokens,
            gather.peer_recv_d.data_ptr(), gather.sync.data_ptr(), gather.world, gather.rank,
            gather.half_words, _ptr(workspace), ws_bytes, _ptr(status), _stream(q.device))
        _check(rc, "clover_b200_decode_step_gather_into")
        return
    rc = lib().clover_b200_decode_step_gather(
        _ptr(out), out.stride(0), _ptr(q), q.stride(0), dtype_code(q.dtype), _ptr(k_cache),
        _ptr(v_cache), dtype_code(k_cache.dtype), nb, bs, _ptr(k_new), _ptr(v_new),
        0 if k_new is None else k_new.stride(0), _ptr(block_tables), block_tables.stride(0),
        _ptr(seq_rows), _ptr(query_start_loc), _ptr(ctx_lens), n_seqs, rows,
        max_queries_per_seq, max_ctx_len, hq, hkv, d, float(score_scale), partition_tokens,
        gather.peer_recv_d.data_ptr(), gather.sync.data_ptr(), gather.world, gather.rank,
        gather.half_words, _ptr(workspace), ws_bytes, _ptr(status), _stream(q.device))
    _check(rc, "clover_b200_decode_step_gather")


def set_wait_limit_ns(ns: int) -> int:
    """Limit of the kernels' bounded waits for later launches (<= 0: the 1 s
    default); returns the previous limit."""
    return int(lib().clover_b200_set_wait_limit_ns(int(ns)))


def host_gather(srcs, sizes, n: int, dst_ptr: int) -> None:
    """Copy n host buffers (ctypes arrays of pointers / byte counts) back to back into dst."""
    rc = lib().clover_b200_host_gather(srcs, sizes, n, dst_ptr)
    if rc != OK:
        _check(rc, "clover_b200_host_gather")

