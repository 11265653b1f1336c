"""B200 attention backend: drop-in for CloverInfer's AttentionNode backends.

``B200AttentionBackend`` exposes the interface ``AttentionNode`` calls
(src/core/nodes.py:88-223) — the one ``CpuAttentionBackend`` implements
(src/core/attention_backend.py:56-144):

    init_request(request_id, initial_kv, decode_reserve_tokens=0) -> int
    decode_layer(request_id, layer_idx, query, key, value, score_scale=1.0) -> [1, Hq, D]
    decode_layer_batch(items) -> list of [1, Hq, D]
    get_context_len(request_id) -> int
    free_request(request_id) -> None            (idempotent)
    get_debug_info() -> dict

with the same semantics: every call appends the new token's K/V to that
layer's cache before attending (the token attends to itself); ``score_scale``
is applied by the backend; ``context_len`` advances after the LAST layer
(:120-121); unknown ids raise ``KeyError``, duplicate ids and empty
``initial_kv`` raise ``ValueError``; outputs come back in the query's dtype
and on the query's device.

Differences that are the point of the rewrite: the KV cache is paged in HBM
(``PagedKVPool``) with native GQA (``Hkv`` heads stored, ``repeat_kv``-expanded
K/V accepted and collapsed); the attention is the sm_100a kernel; a batch is
one launch sequence (block reserve when a sequence crosses a block boundary,
then one fused append + decode kernel, then the split-K reduce) instead of a
Python loop; KV heads can be sharded over GPUs (``HeadShardGroup``) with one
all-gather of the outputs.

``decode_batch`` is the tensor API for a step-batched engine
(src/core/scheduler.py:980-1093): ``query [T, Hq, D]``, ``key/value [T, Hkv, D]``
for ``T = sum(n_new)`` new tokens (causal among a sequence's new tokens),
returning ``[T, Hq, D]`` on the GPU without a host sync.
"""

from __future__ import annotations

import math
import os
import warnings
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Dict, List, Optional, Sequence

import torch

from . import _lib
from .head_groups import local_inputs, select_kv_heads
from .kv_cache import PagedKVPool, auto_partition, to_device_i32


_HOST_Q_DTYPES = (torch.float32, torch.float16, torch.bfloat16)
_ONE = (1,)  # n_new of a single-token batch, as _split reads it (its max)


@dataclass
class _Request:
    row: int
    layer_len: List[int]
    ctx: int


@dataclass
class _Stats:
    batches: int = 0
    items: int = 0
    tokens: int = 0
    kv_bytes_read: int = 0


class _FastPlan:
    """Cached buffers of the host-tensor fast path for one batch shape: a
    pinned staging buffer and its device twin laid out as
    [queries | keys | values | int32 metadata], the ctypes source/size arrays
    the native gather fills it from, and the pinned output."""

    def __init__(self, device, B, q_shape, q_dtype, k_shape, k_dtype, n_meta, out_dtype, hq_total):
        import ctypes
        esz = lambda dt: torch.empty((), dtype=dt).element_size()  # noqa: E731
        self.qb = int(torch.Size(q_shape).numel()) * esz(q_dtype)
        self.kb = int(torch.Size(k_shape).numel()) * esz(k_dtype)
        self.n = 3 * B + 1
        self.k_off = B * self.qb
        self.v_off = self.k_off + B * self.kb
        self.m_off = self.v_off + B * self.kb
        total = self.m_off + 4 * n_meta
        self.host = torch.empty(total, dtype=torch.uint8, pin_memory=True)
        self.dev = torch.empty(total, dtype=torch.uint8, device=device)
        self.q = self.dev[:self.k_off].view(q_dtype).view(B, *q_shape)
        self.k = self.dev[self.k_off:self.v_off].view(k_dtype).view(B, *k_shape)
        self.v = self.dev[self.v_off:self.m_off].view(k_dtype).view(B, *k_shape)
        meta = self.dev[self.m_off:].view(torch.int32)
        self.rows, self.offs_d, self.ctx = meta[0:B], meta[B:2 * B + 1], meta[2 * B + 1:]
        self.meta = (ctypes.c_int32 * n_meta)()
        self.srcs = (ctypes.c_void_p * self.n)()
        self.sizes = (ctypes.c_int64 * self.n)(*([self.qb] * B + [self.kb] * (2 * B) + [4 * n_meta]))
        self.srcs[self.n - 1] = ctypes.addressof(self.meta)
        self.offs_list = list(range(B + 1))  # one new token per item
        self.out = torch.empty((B, hq_total, q_shape[-1]), dtype=out_dtype, pin_memory=True)
        self.warm = False  # one eager call ran with this shape (one-time set-up done)
        self.graphs: Dict[tuple, "_StepGraph"] = {}
        # The captured steps' result buffer, shared by this shape's graphs (they
        # replay one after another on one stream): the output [B, Hq, D] and,
        # after it, the status word those steps' kernels raise bits in, so one
        # D2H copy brings both back.
        self.out_bytes = B * hq_total * q_shape[-1] * esz(out_dtype)
        self.res_dev = torch.zeros(self.out_bytes + 16, dtype=torch.uint8, device=device)
        self.out_dev = self.res_dev[:self.out_bytes].view(out_dtype).view(B, hq_total, q_shape[-1])
        self.status_dev = self.res_dev[self.out_bytes:self.out_bytes + 4].view(torch.int32)
        self.res_shape = (B, 1, hq_total, q_shape[-1])
        self.out_dtype = out_dtype
        self.ws: Dict[tuple, Optional[torch.Tensor]] = {}  # by (bucket, split)


class _StepGraph:
    """A captured fast-path step: H2D of the staging buffer, the fused
    append + decode (+ reduce, + gather), D2H of the output and the status
    word.  Holds the output and workspace its kernels were captured with, so
    they stay allocated while the graph exists."""

    def __init__(self, graph, out_dev, workspace):
        self.graph = graph
        self.out_dev = out_dev
        self.workspace = workspace


def q_local_is_whole(lo: int, hi: int, num_kv_heads: int) -> bool:
    return (lo, hi) == (0, num_kv_heads)


def _default_device() -> torch.device:
    if not torch.cuda.is_available():
        raise RuntimeError("B200AttentionBackend requires a CUDA device (no CPU fallback)")
    local = os.environ.get("LOCAL_RANK")
    return torch.device("cuda", int(local) if local is not None else torch.cuda.current_device())


class B200AttentionBackend:
    def __init__(self, *, num_blocks: Optional[int] = None, block_size: int = 16,
                 max_seqs: int = 256, max_seq_len: int = 131072,
                 num_kv_heads: Optional[int] = None, kv_dtype: Optional[torch.dtype] = None,
                 device=None, kv_cache_fraction: float = 0.5, partition_tokens: int = 0,
                 shard=None, check_status: bool = True, shuffle_seed: Optional[int] = None,
                 gather: str = "peer", max_rows_per_call: Optional[int] = None,
                 cuda_graphs: bool = True, max_fast_plans: int = 8, **_unused) -> None:
        self.device = torch.device(device) if device is not None else _default_device()
        if self.device.type != "cuda":
            raise RuntimeError("B200AttentionBackend requires a CUDA device (no CPU fallback)")
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        _lib.lib()  # fail loudly if the CUDA library cannot be built or loaded
        self.block_size = int(block_size)
        self.max_seqs = int(max_seqs)
        self.max_seq_len = int(max_seq_len)
        self.num_blocks = num_blocks
        self.cfg_num_kv_heads = num_kv_heads
        self.kv_dtype = kv_dtype
        self.kv_cache_fraction = float(kv_cache_fraction)
        self.partition_tokens = int(partition_tokens)
        self.shard = shard
        self.check_status = bool(check_status)
        self.shuffle_seed = shuffle_seed
        if gather not in ("peer", "nccl"):
            raise ValueError("gather must be 'peer' or 'nccl'")
        self.gather_mode = gather
        self.max_rows_per_call = int(max_rows_per_call or 4 * self.max_seqs)
        self._peer = None
        self.pool: Optional[PagedKVPool] = None
        self.num_layers = 0
        self.num_kv_heads = 0  # total (all shards)
        self.head_dim = 0
        self.kv_range = (0, 0)
        self._reqs: Dict[str, _Request] = {}
        self.stats = _Stats()
        self._status_host = torch.zeros(1, dtype=torch.int32, pin_memory=True)
        self._kv_esz = 0
        # host-tensor fast-path plans (staging buffers, captured steps) by batch
        # shape, least recently used first; continuous batching changes the
        # batch size from step to step, so only the most recent shapes are kept
        self._fast: "OrderedDict[tuple, _FastPlan]" = OrderedDict()
        self.max_fast_plans = int(max_fast_plans)
        self.cuda_graphs = bool(cuda_graphs)
        # prefill ingestion runs on a side stream; the decode stream waits for
        # these events before it next reads or frees blocks
        self._ingest_stream: Optional[torch.cuda.Stream] = None
        self._pending_ingest: List[torch.cuda.Event] = []

    # ------------------------------------------------------------ setup
    def _ensure_pool(self, num_layers: int, heads: int, head_dim: int, dtype: torch.dtype) -> None:
        if self.pool is not None:
            if (num_layers, head_dim) != (self.num_layers, self.head_dim):
                raise ValueError(
                    f"initial_kv has {num_layers} layers x head_dim {head_dim}; backend holds "
                    f"{self.num_layers} x {self.head_dim}")
            return
        hkv = int(self.cfg_num_kv_heads or heads)
        if heads % hkv:
            raise ValueError(f"initial_kv has {heads} heads, not a multiple of num_kv_heads={hkv}")
        dt = self.kv_dtype or dtype
        if dt not in (torch.float32, torch.float16, torch.bfloat16, torch.float8_e4m3fn):
            raise TypeError(f"unsupported KV dtype {dt}")
        self.num_layers, self.num_kv_heads, self.head_dim, self.kv_dtype = num_layers, hkv, head_dim, dt
        self._kv_esz = torch.empty((), dtype=dt).element_size()
        if self.shard is not None:
            self.kv_range = self.shard.kv_range(hkv)
        else:
            self.kv_range = (0, hkv)
        local = self.kv_range[1] - self.kv_range[0]
        nb = self.num_blocks
        esz = torch.empty((), dtype=dt).element_size()
        per_block = 2 * num_layers * self.block_size * local * head_dim * esz
        if nb is None:
            free, _ = torch.cuda.mem_get_info(self.device)
            nb = max(16, int(free * self.kv_cache_fraction) // per_block)
        width = min(nb, -(-self.max_seq_len // self.block_size) + 1)
        self.pool = PagedKVPool(nb, self.block_size, local, head_dim, num_layers=num_layers,
                                dtype=dt, device=self.device, max_seqs=self.max_seqs,
                                max_blocks_per_seq=width)
        if self.shuffle_seed is not None:
            self.pool.shuffle_free_stack(self.shuffle_seed)

    def _select_heads(self, x: torch.Tensor) -> torch.Tensor:
        """View of [T, H, D] with this rank's KV heads only.  H may be Hkv
        (native) or Hq = Hkv * g (repeat_kv-expanded: one head per group kept)."""
        return select_kv_heads(x, self.kv_range, self.num_kv_heads)

    def _local_kv(self, x: torch.Tensor) -> torch.Tensor:
        """[T, H, D] on device in the cache dtype, local KV heads only."""
        return self._select_heads(x).to(device=self.device, dtype=self.kv_dtype,
                                        non_blocking=True).contiguous()

    def _ingest(self, row: int, initial_kv, T: int) -> None:
        """Every layer's prefill K/V into the pool in one pass: this rank's
        heads of all layers are gathered into one staging buffer [L, K|V, T,
        Hkv_local, D] (pinned host memory for host inputs, so the H2D is one
        asynchronous copy), then one slot computation and one multi-layer
        append.  All of it runs on a side stream, overlapping whatever the
        decode stream is doing; the decode stream waits for it before it next
        reads or frees blocks (_await_ingest)."""
        pool = self.pool
        L = len(initial_kv)
        hl = self.kv_range[1] - self.kv_range[0]
        cur = torch.cuda.current_stream(self.device)
        if self._ingest_stream is None:
            self._ingest_stream = torch.cuda.Stream(self.device)
        ing = self._ingest_stream
        ing.wait_stream(cur)  # the blocks were reserved (and inputs made) on the decode stream
        on_host = not initial_kv[0]["key"].is_cuda
        with torch.cuda.stream(ing):
            shape = (L, 2, T, hl, self.head_dim)
            if on_host:
                stage = torch.empty(shape, dtype=self.kv_dtype, pin_memory=True)
            else:
                stage = torch.empty(shape, dtype=self.kv_dtype, device=self.device)
            for li, layer in enumerate(initial_kv):
                for j, name in ((0, "key"), (1, "value")):
                    src = layer[name]
                    if src.is_cuda:
                        src.record_stream(ing)  # read on this stream after the call returns
                    stage[li, j].copy_(self._select_heads(src))
            dev = stage.to(self.device, non_blocking=True) if on_host else stage
            meta = to_device_i32([row, 0, 0, T], self.device)
            slots = pool.slots(meta[0:1], meta[1:2], meta[2:4], T)
            _lib.kv_append_layers(pool.k, pool.v, dev[:, 0], dev[:, 1], slots, pool.status)
            ev = torch.cuda.Event()
            ev.record(ing)
        self._pending_ingest.append(ev)

    def _await_ingest(self) -> None:
        """Order the decode stream after every prefill ingestion issued so far."""
        cur = torch.cuda.current_stream(self.device)
        for ev in self._pending_ingest:
            cur.wait_event(ev)
        self._pending_ingest.clear()

    # ------------------------------------------------------------ interface
    def init_request(self, request_id: str, initial_kv: List[Dict[str, torch.Tensor]],
                     decode_reserve_tokens: int = 0) -> int:
        if request_id in self._reqs:
            raise ValueError(f"Request {request_id} already exists")
        if not initial_kv:
            raise ValueError("initial_kv must contain at least one layer")
        k0 = initial_kv[0]["key"]
        if k0.dim() != 3:
            raise ValueError(f"initial_kv key must be [T, H, D], got {tuple(k0.shape)}")
        T, H, D = (int(s) for s in k0.shape)
        for layer in initial_kv:
            if tuple(layer["key"].shape) != (T, H, D) or tuple(layer["value"].shape) != (T, H, D):
                raise ValueError("all initial_kv layers must share one [T, H, D] shape")
        self._ensure_pool(len(initial_kv), H, D, k0.dtype)
        pool = self.pool
        row = pool.acquire_row()
        try:
            pool.reserve([row], [T + max(1, int(decode_reserve_tokens))], "OOM: Not enough blocks")
        except Exception:
            pool._free_rows.append(row)
            raise
        if T > 0:
            self._ingest(row, initial_kv, T)
        self._reqs[request_id] = _Request(row=row, layer_len=[T] * self.num_layers, ctx=T)
        return T

    def get_context_len(self, request_id: str) -> int:
        return self._reqs[request_id].ctx

    def free_request(self, request_id: str) -> None:
        req = self._reqs.pop(request_id, None)
        if req is not None:
            if self._pending_ingest:
                self._await_ingest()  # its blocks may still be being written
            self.pool.release_row(req.row)

    def decode_layer(self, request_id: str, layer_idx: int, query: torch.Tensor,
                     key: torch.Tensor, value: torch.Tensor, score_scale: float = 1.0) -> torch.Tensor:
        return self.decode_layer_batch([{"request_id": request_id, "layer_idx": layer_idx,
                                         "query": query, "key": key, "value": value,
                                         "score_scale": score_scale}])[0]

    def decode_layer_batch(self, items: List[Dict[str, object]]) -> List[torch.Tensor]:
        results: List[Optional[torch.Tensor]] = [None] * len(items)
        i = 0
        while i < len(items):
            layer = int(items[i]["layer_idx"])
            scale = float(items[i].get("score_scale", 1.0))
            seen = set()
            j = i
            while j < len(items):
                it = items[j]
                rid = str(it["request_id"])
                if (int(it["layer_idx"]) != layer or float(it.get("score_scale", 1.0)) != scale
                        or rid in seen):
                    break
                seen.add(rid)
                j += 1
            self._run_items(items[i:j], layer, scale, results, i)
            i = j
        return results  # type: ignore[return-value]

    def _run_items(self, items, layer: int, scale: float, results, base: int) -> None:
        reqs_d = self._reqs
        try:
            reqs = [reqs_d[it["request_id"]] for it in items]
        except (KeyError, TypeError):
            reqs = []
            for it in items:
                rid = str(it["request_id"])
                if rid not in reqs_d:
                    raise KeyError(f"Unknown request {rid}") from None
                reqs.append(reqs_d[rid])
        qs = [it["query"] for it in items]
        ks = [it["key"] for it in items]
        vs = [it["value"] for it in items]
        if qs[0].dim() == 3 or ks[0].dim() == 3 or vs[0].dim() == 3:
            sq = lambda t: t.squeeze(0) if t.dim() == 3 else t  # noqa: E731
            qs, ks, vs = [sq(t) for t in qs], [sq(t) for t in ks], [sq(t) for t in vs]
        B = len(items)
        q0, k0 = qs[0], ks[0]
        key = (B, q0.shape, q0.dtype, k0.shape, k0.dtype)
        plan = self._fast.get(key)
        # The fast path gathers fixed byte counts per item into one pinned
        # buffer: every item must be on the host with the first one's shapes
        # and dtypes.
        fast = plan is not None or (not q0.is_cuda and q0.dtype in _HOST_Q_DTYPES)
        if fast:
            if plan is None:
                plan = _FastPlan(self.device, B, q0.shape, q0.dtype, k0.shape, k0.dtype, 3 * B + 1,
                                 q0.dtype, q0.shape[0])
                self._fast[key] = plan
                while len(self._fast) > max(1, self.max_fast_plans):
                    # every call ends with a stream sync: no evicted graph is in flight
                    self._fast.popitem(last=False)
            elif len(self._fast) > 1:
                self._fast.move_to_end(key)
            _, qsh, qdt, ksh, kdt = key
            srcs = plan.srcs
            for i in range(B):
                t, kt, vt = qs[i], ks[i], vs[i]
                if (t.shape != qsh or kt.shape != ksh or vt.shape != ksh or t.dtype != qdt
                        or kt.dtype != kdt or vt.dtype != kdt or t.is_cuda or kt.is_cuda or vt.is_cuda):
                    fast = False
                    break
                if not (t.is_contiguous() and kt.is_contiguous() and vt.is_contiguous()):
                    t, kt, vt = t.contiguous(), kt.contiguous(), vt.contiguous()
                    qs[i], ks[i], vs[i] = t, kt, vt  # keep alive until the gather
                srcs[i] = t.data_ptr()
                srcs[B + i] = kt.data_ptr()
                srcs[2 * B + i] = vt.data_ptr()
        if not fast:  # device tensors (or mixed inputs): no staging, no host sync
            rids = [str(it["request_id"]) for it in items]
            out = self.decode_batch(rids, layer, torch.stack(qs), torch.stack(ks), torch.stack(vs), scale)
            if not qs[0].is_cuda:
                out = out.to("cpu")
            if out.dtype != q0.dtype:
                out = out.to(q0.dtype)
            if self.check_status and not qs[0].is_cuda:
                self.pool.check_status()
            for n in range(len(items)):
                results[base + n] = out[n:n + 1]
            return
        if self._pending_ingest:
            self._await_ingest()
        rows, targets, need = self._plan_single(reqs, layer, q0.shape)
        plan.meta[:] = rows + plan.offs_list + targets
        _lib.host_gather(srcs, plan.sizes, plan.n, plan.host.data_ptr())
        if need:
            # rows and new contexts (the targets) go to the device once, where
            # the reserve kernel reads them ahead of the step
            plan.dev[plan.m_off:].copy_(plan.host[plan.m_off:], non_blocking=True)
            self.pool.commit_reserve(rows, targets, need, plan.rows, plan.ctx)
        pt = self._split(targets, _ONE)
        step = self._step_graph(plan, layer, scale, max(targets), pt) if plan.warm else None
        if step is not None:
            # One graph launch (H2D, fused step); the copy of the output and
            # status word into fresh pinned memory and the host bookkeeping
            # run while the GPU works.
            step.graph.replay()
            res = plan.res_dev.to("cpu", non_blocking=True)
            outs = res[:plan.out_bytes].view(plan.out_dtype).view(plan.res_shape).unbind(0)
            status = res[plan.out_bytes:plan.out_bytes + 4].view(torch.int32)
            self._advance(reqs, layer, None, targets)
            torch.cuda.current_stream(self.device).synchronize()
            code = int(status[0])
            if code:
                plan.status_dev.zero_()
                if self.check_status:
                    self.pool.raise_status(code)
            results[base:base + B] = outs
            return
        plan.dev.copy_(plan.host, non_blocking=True)
        out = self._launch(reqs, layer, [1] * B, targets, plan.q, plan.k, plan.v, plan.rows,
                           plan.offs_d, plan.ctx, scale, check=False, pt=pt)
        # output and status word back behind one synchronisation
        plan.out.copy_(out, non_blocking=True)
        self._status_host.copy_(self.pool.status, non_blocking=True)
        plan.warm = True
        torch.cuda.current_stream(self.device).synchronize()
        if self.check_status and int(self._status_host[0]):
            self.pool.check_status()
        results[base:base + B] = plan.out.clone().split(1)

    def _plan_single(self, reqs, layer: int, q_shape):
        """_plan for one new token per request: validate and count the blocks
        the new tokens need (raising before any state changes when they do
        not fit); returns (table rows, contexts after the step, blocks to
        reserve).  The caller reserves them from the staged metadata."""
        pool = self.pool
        if not 0 <= layer < self.num_layers:
            raise IndexError(f"layer_idx {layer} out of range [0, {self.num_layers})")
        hq, d = int(q_shape[0]), int(q_shape[1])
        if hq % self.num_kv_heads or d != self.head_dim:
            raise ValueError(f"query heads x dim {hq} x {d} do not fit {self.num_kv_heads} KV heads x {self.head_dim}")
        rows = [r.row for r in reqs]
        targets = [r.layer_len[layer] + 1 for r in reqs]
        cap = pool.block_size
        blocks = pool.row_blocks
        # (rows are distinct: decode_layer_batch never puts one request twice in a group)
        for r, t in zip(rows, targets):
            if t > blocks[r] * cap:  # some row crosses into a new block
                need = pool.demand(rows, targets)
                if need > pool.free_count:
                    raise RuntimeError("OOM during append")
                return rows, targets, need
        return rows, targets, 0

    # Context lengths are rounded up to this many tokens for a captured step:
    # the launch's max_ctx_len (and so its partition plan and workspace) is
    # fixed per graph, re-captured when the batch outgrows it.
    _GRAPH_CTX_BUCKET = 512

    def _split(self, targets, n_new) -> int:
        """partition_tokens for this call: the caller's, or the host's choice
        from the batch's contexts (kv_cache.auto_partition)."""
        if self.partition_tokens:
            return self.partition_tokens
        sharded = self.shard is not None and self.shard.world > 1
        return auto_partition(targets, max(n_new), sharded)

    def _step_graph(self, plan: _FastPlan, layer: int, scale: float, max_ctx: int, pt: int):
        """The captured step for this batch shape, layer, scale and context
        bucket, capturing it on first use; None where a step is not captured
        (graphs off, NCCL-gathered shards)."""
        if not self.cuda_graphs:
            return None
        sharded = self.shard is not None and self.shard.world > 1
        if pt < 0 and not sharded and max_ctx <= self.max_seq_len:
            # the balanced split's work follows the contexts themselves; its
            # max_ctx_len only bounds the workspace: one bucket, no re-capture.
            # (A sharded step runs fixed partitions, sized by the bucket.)
            bucket = self.max_seq_len
        else:
            bucket = -(-max_ctx // self._GRAPH_CTX_BUCKET) * self._GRAPH_CTX_BUCKET
        key = (layer, scale, bucket, pt)
        step = plan.graphs.get(key)
        if step is not None:
            return step
        pool = self.pool
        group = plan.q.shape[1] // self.num_kv_heads
        lo, hi = self.kv_range
        q = plan.q if q_local_is_whole(lo, hi, self.num_kv_heads) else plan.q[:, lo * group:hi * group]
        if q.dtype not in (torch.float32, self.kv_dtype) or q.stride(2) != 1 or q.stride(1) != self.head_dim:
            return None
        peer = self._peer_for(q) if sharded else None
        if sharded and peer is None:
            return None  # NCCL gather: stays eager
        B = q.shape[0]
        if plan.k.shape[1] != self.num_kv_heads or plan.k.dtype != self.kv_dtype:
            return None  # K/V need a copy (expanded heads, other dtype): stays eager
        k_loc, v_loc = plan.k[:, lo:hi], plan.v[:, lo:hi]  # token stride spans all heads
        n_seqs = B
        if peer is not None:
            nbytes = _lib.decode_gather_workspace_bytes(n_seqs, B, 1, bucket, q.shape[1], pool.num_kv_heads,
                                                        self.head_dim, pool.block_size, pool.dtype,
                                                        q.dtype, pt)
        else:
            nbytes = _lib.decode_workspace_bytes(n_seqs, B, 1, bucket, q.shape[1], pool.num_kv_heads,
                                                 self.head_dim, pool.block_size, pool.dtype, q.dtype,
                                                 pt)
        for old in [k for k in plan.graphs if k[:2] == key[:2]]:
            del plan.graphs[old]  # an older bucket (or split) of this layer and scale
        live = {k[2:] for k in plan.graphs}
        for b in [b for b in plan.ws if b not in live]:
            del plan.ws[b]  # graphs that still use it keep their own reference
        if key[2:] not in plan.ws:
            plan.ws[key[2:]] = (torch.empty(nbytes, dtype=torch.uint8, device=self.device)
                                if nbytes > 0 else None)
        ws = plan.ws[key[2:]]
        out_dev = plan.out_dev
        g = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(g):
                # H2D of the staging buffer, then the fused step writing the
                # (all-gathered) output and its status bits into the plan's
                # result buffer; the caller copies that back after the launch.
                plan.dev.copy_(plan.host, non_blocking=True)
                if peer is not None:
                    _lib.decode_step_gather(q, pool.k[layer], pool.v[layer], k_loc, v_loc, pool.tables,
                                            plan.offs_d, plan.ctx, peer, max_queries_per_seq=1,
                                            max_ctx_len=bucket, score_scale=scale, seq_rows=plan.rows,
                                            partition_tokens=pt, workspace=ws,
                                            status=plan.status_dev, out=out_dev)
                else:
                    _lib.decode_step(out_dev, q, pool.k[layer], pool.v[layer], k_loc, v_loc, pool.tables,
                                     plan.offs_d, plan.ctx, max_queries_per_seq=1, max_ctx_len=bucket,
                                     score_scale=scale, seq_rows=plan.rows,
                                     partition_tokens=pt, workspace=ws,
                                     status=plan.status_dev, check=False)
        except Exception as e:  # capture is not available here: stay eager from now on
            warnings.warn(f"B200AttentionBackend: CUDA graph capture failed ({e!r}); "
                          "using eager launches", RuntimeWarning)
            self.cuda_graphs = False
            return None
        step = _StepGraph(g, out_dev, ws)
        plan.graphs[key] = step
        return step

    # ------------------------------------------------------------ tensor API
    def decode_batch(self, request_ids: Sequence[str], layer_idx: int, query: torch.Tensor,
                     key: torch.Tensor, value: torch.Tensor, score_scale: float = 1.0,
                     n_new: Optional[Sequence[int]] = None,
                     out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Append ``n_new[b]`` tokens per request and attend causally.

        query [T, Hq, D] (fp32, or the cache dtype), key/value [T, Hkv or Hq, D];
        returns [T, Hq, D] on the GPU in the query dtype (all heads: sharded
        backends all-gather).  Enqueued on the current stream; no host sync.

        ``out``: the consumer's buffer to receive the output instead, e.g. the
        dense node's o_proj input (model_adapter.py:572): a device tensor whose
        T rows each hold Hq * D contiguous values ([T, Hq * D], [T, 1, Hq * D]
        or [T, Hq, D], any row stride), f32/f16/bf16.  A sharded backend's fused
        gather writes every rank's heads straight into it; returned as a
        [T, Hq, D] view.
        """
        B = len(request_ids)
        n_new = [1] * B if n_new is None else [int(n) for n in n_new]
        T = sum(n_new)
        if query.shape[0] != T or key.shape[0] != T or value.shape[0] != T:
            raise ValueError(f"expected {T} new tokens, got q {tuple(query.shape)} k {tuple(key.shape)}")
        if self._pending_ingest:
            self._await_ingest()
        hq = query.shape[1]
        dst = None if out is None else self._consumer_view(out, T, hq)
        q_shape = query.shape[1:]
        # host inputs start their (asynchronous) copies now, so the planning
        # below overlaps them; a sharded rank moves only its own heads
        local = None
        if not (query.is_cuda or key.is_cuda or value.is_cuda) and hq % self.num_kv_heads == 0:
            query, key, value = (self._h2d(x) for x in
                                 local_inputs(query, key, value, self.kv_range, self.num_kv_heads))
            local = hq
        else:
            if not query.is_cuda:
                query = query.to(self.device, non_blocking=True)
            if not key.is_cuda:
                key = key.to(self.device, non_blocking=True)
            if not value.is_cuda:
                value = value.to(self.device, non_blocking=True)
        reqs, rows, targets, offs, ctx_rows = self._plan(request_ids, layer_idx, n_new, q_shape)
        meta = to_device_i32(rows + offs + ctx_rows, self.device)
        res = self._launch(reqs, layer_idx, n_new, targets, query, key, value, meta[0:B],
                           meta[B:2 * B + 1], meta[2 * B + 1:], score_scale, dst=dst, hq=local)
        if dst is not None:
            if res.data_ptr() != dst.data_ptr():
                dst.copy_(res)
            return dst
        # the fused gather's buffer is rewritten by the next call
        return res.clone() if self._peer is not None and res.data_ptr() == self._peer.out.data_ptr() else res

    def _h2d(self, x: torch.Tensor) -> torch.Tensor:
        """A host tensor on this backend's device, copied asynchronously: a
        view of some heads (rows of contiguous values at a wider stride) goes
        through a pinned staging copy, so only those bytes cross PCIe."""
        if not x.is_contiguous():
            stage = torch.empty(x.shape, dtype=x.dtype, pin_memory=True)
            stage.copy_(x)
            x = stage
        return x.to(self.device, non_blocking=True)

    def _consumer_view(self, out: torch.Tensor, T: int, hq: int) -> torch.Tensor:
        """[T, Hq, D] view of a consumer buffer whose T rows hold Hq * D values."""
        D = self.head_dim
        if not out.is_cuda or out.device != self.device:
            raise ValueError(f"out must be on {self.device}")
        if out.dtype not in (torch.float32, torch.float16, torch.bfloat16):
            raise TypeError(f"out dtype {out.dtype} is not f32/f16/bf16")
        if out.dim() < 2 or out.shape[0] != T:
            raise ValueError(f"out must have {T} rows, got {tuple(out.shape)}")
        rows = out.flatten(1) if out.dim() > 2 else out
        if (rows.shape[1] != hq * D or rows.stride(1) != 1
                or (out.dim() > 2 and rows.data_ptr() != out.data_ptr())):
            raise ValueError(f"each row of out must hold {hq} x {D} contiguous values")
        return rows.as_strided((T, hq, D), (rows.stride(0), D, 1))

    def _plan(self, request_ids, layer_idx: int, n_new, q_shape):
        """Validate, reserve blocks for the new tokens and build the metadata
        lists (rows, causal limits).  Raises before any state changes."""
        pool = self.pool
        if pool is None:
            raise KeyError("no request has been initialised")
        reqs = []
        for r in request_ids:
            try:
                reqs.append(self._reqs[r])
            except KeyError:
                raise KeyError(f"Unknown request {r}") from None
        if not 0 <= layer_idx < self.num_layers:
            raise IndexError(f"layer_idx {layer_idx} out of range [0, {self.num_layers})")
        hq, d = int(q_shape[0]), int(q_shape[1])
        if hq % self.num_kv_heads or d != self.head_dim:
            raise ValueError(f"query heads x dim {hq} x {d} do not fit {self.num_kv_heads} KV heads x {self.head_dim}")
        rows = [r.row for r in reqs]
        pos = [r.layer_len[layer_idx] for r in reqs]
        targets = [p + n for p, n in zip(pos, n_new)]
        pool.reserve(rows, targets, "OOM during append")
        offs = [0]
        ctx_rows: List[int] = []
        for p, n in zip(pos, n_new):
            offs.append(offs[-1] + n)
            ctx_rows.extend(range(p + 1, p + n + 1))
        return reqs, rows, targets, offs, ctx_rows

    def _launch(self, reqs, layer_idx, n_new, targets, query, key, value, rows_d, offs_d, ctx_d,
                score_scale, check: bool = True, pt: Optional[int] = None, dst=None,
                hq: Optional[int] = None):
        """``hq`` given: query, key and value are already this rank's heads on
        the device (of ``hq`` query heads in all)."""
        pool = self.pool
        if pt is None:
            pt = self._split(targets, n_new)
        local = hq is not None
        hq = query.shape[1] if hq is None else hq
        group = hq // self.num_kv_heads
        lo, hi = self.kv_range
        q = query.to(self.device, non_blocking=True)
        if q.dtype not in (torch.float32, self.kv_dtype):
            q = q.float()
        if not local and (lo, hi) != (0, self.num_kv_heads):
            q = q[:, lo * group:hi * group]
        if q.stride(2) != 1 or q.stride(1) != self.head_dim:
            q = q.contiguous()
        if local:
            k_loc = key.to(dtype=self.kv_dtype).contiguous()
            v_loc = value.to(dtype=self.kv_dtype).contiguous()
        else:
            k_loc, v_loc = self._local_kv(key), self._local_kv(value)
        sharded = self.shard is not None and self.shard.world > 1
        peer = self._peer_for(q) if sharded else None
        if peer is not None:
            # fused append + decode + reduce with the all-gather over NVLink
            out = pool.decode_step_gather(layer_idx, q, k_loc, v_loc, offs_d, ctx_d, rows_d,
                                          max(n_new), max(targets), score_scale, peer,
                                          partition_tokens=pt, out=dst)
        else:
            # one launch: append each row's token at ctx - 1, then attend (+ reduce)
            direct = dst is not None and not sharded and dst.dtype == q.dtype
            out = pool.decode_step(layer_idx, q, k_loc, v_loc, offs_d, ctx_d, rows_d, max(n_new),
                                   max(targets), score_scale, out=dst if direct else None,
                                   partition_tokens=pt, check=check)
        self._advance(reqs, layer_idx, n_new, targets)
        if sharded and peer is None:
            out = self.shard.gather(out, self.num_kv_heads, group)
        return out

    def _advance(self, reqs, layer_idx, n_new, targets) -> None:
        """Host bookkeeping of a launched step: per-layer lengths, context
        (after the last layer) and counters.  n_new None: one token each."""
        lo, hi = self.kv_range
        last = layer_idx == self.num_layers - 1
        if n_new is None:
            for r in reqs:
                r.layer_len[layer_idx] += 1
                if last:
                    r.ctx += 1
        else:
            for r, n in zip(reqs, n_new):
                r.layer_len[layer_idx] += n
                if last:
                    r.ctx += n
        st = self.stats
        st.batches += 1
        st.items += len(reqs)
        st.tokens += len(reqs) if n_new is None else sum(n_new)
        st.kv_bytes_read += sum(targets) * (hi - lo) * self.head_dim * 2 * self._kv_esz

    def _peer_for(self, q: torch.Tensor):
        """The fused-gather buffers for this call's shape, or None (NCCL)."""
        if self.gather_mode != "peer" or q.shape[0] > self.max_rows_per_call:
            return None
        if self.num_kv_heads % self.shard.world:
            return None  # uneven shards: NCCL gather pads them
        if self._peer is None:
            from .sharded import PeerGather
            self._peer = PeerGather(self.shard, self.max_rows_per_call,
                                    q.shape[1] * self.shard.world, self.head_dim, q.dtype,
                                    self.device)
        return self._peer if self._peer.out.dtype == q.dtype else None

    def close(self) -> None:
        """Release the fused-gather peer buffers (collective under sharding:
        every rank calls it)."""
        if self._peer is not None:
            self._peer.close()
            self._peer = None

    # ------------------------------------------------------------ debug
    def get_debug_info(self) -> dict:
        pool = self.pool
        info = {
            "backend": "b200",
            "library": _lib.lib_path(),
            "device": str(self.device),
            "live_requests": len(self._reqs),
            "stats": dict(self.stats.__dict__),
        }
        if pool is not None:
            info.update({
                "num_layers": self.num_layers, "num_kv_heads": self.num_kv_heads,
                "kv_heads_local": list(self.kv_range), "head_dim": self.head_dim,
                "kv_dtype": str(self.kv_dtype), "block_size": pool.block_size,
                "num_blocks": pool.num_blocks, "free_blocks": pool.free_count,
                "kv_cache_bytes": 2 * pool.k.numel() * pool.k.element_size(),
            })
        if self.shard is not None:
            info["shard"] = {"rank": self.shard.rank, "world": self.shard.world}
        return info
