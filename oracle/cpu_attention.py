"""CPU restatement of CloverInfer's reference attention backend (test oracle).

Follows ``CpuAttentionBackend`` in src/core/attention_backend.py:

* init_request      :68-80   per-layer contiguous ``[T, H, D]`` caches; duplicate id
                             -> ValueError; empty ``initial_kv`` -> ValueError.
* decode_layer      :82-123  unknown id -> KeyError; squeeze 3-D q/k/v (:98-103);
                             append the new token with a concatenation (:105-110);
                             scores = einsum("hd,lhd->hl") in fp32 * score_scale (:116);
                             softmax over the context (:117);
                             context = einsum("hl,lhd->hd") cast to q's dtype (:118);
                             context_len += 1 after the LAST layer only (:120-121).
* decode_layer_batch:125-136 serial loop over item dicts.
* get_context_len / free_request :138-144 (free is idempotent).

The upstream backend only sees as many KV heads as query heads (the model
adapter expands grouped KV with ``repeat_kv`` first, src/core/model_adapter.py:504-507),
so GQA parity cases feed this oracle ``repeat_kv``-expanded K/V.

Test infrastructure only: the product never imports this module.
"""

from __future__ import annotations

from typing import Dict, List

import torch


def repeat_kv(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    """Expand ``[..., Hkv, D]`` to ``[..., Hkv * n_rep, D]``; KV head i serves
    query heads ``i*n_rep .. i*n_rep+n_rep-1`` (HuggingFace ``repeat_kv`` order,
    the expansion src/core/model_adapter.py:504-507 applies before the backend)."""
    if n_rep == 1:
        return x
    *lead, hkv, d = x.shape
    return x.unsqueeze(-2).expand(*lead, hkv, n_rep, d).reshape(*lead, hkv * n_rep, d)


def attend(q: torch.Tensor, keys: torch.Tensor, values: torch.Tensor,
           score_scale: float, out_dtype=None) -> torch.Tensor:
    """The scoring of attention_backend.py:116-118 on one request:
    q [H, D], keys/values [L, H, D] -> [H, D] (fp32 math, cast to ``out_dtype``,
    default q's dtype)."""
    logits = torch.einsum("hd,lhd->hl", q.float(), keys.float()) * float(score_scale)
    probs = torch.softmax(logits, dim=-1)
    return torch.einsum("hl,lhd->hd", probs, values.float()).to(out_dtype or q.dtype)


class CpuAttentionOracle:
    """Same interface and numerics as the upstream ``CpuAttentionBackend``."""

    def __init__(self) -> None:
        self._k: Dict[str, List[torch.Tensor]] = {}
        self._v: Dict[str, List[torch.Tensor]] = {}
        self._ctx: Dict[str, int] = {}

    # attention_backend.py:68-80
    def init_request(self, request_id: str, initial_kv: List[Dict[str, torch.Tensor]],
                     decode_reserve_tokens: int = 0) -> int:
        if request_id in self._k:
            raise ValueError(f"Request {request_id} already exists")
        ks = [layer["key"].detach().cpu().contiguous() for layer in initial_kv]
        vs = [layer["value"].detach().cpu().contiguous() for layer in initial_kv]
        self._k[request_id] = ks
        self._v[request_id] = vs
        if not ks:
            raise ValueError("initial_kv must contain at least one layer")
        self._ctx[request_id] = int(ks[0].shape[0])
        return self._ctx[request_id]

    # attention_backend.py:82-123
    def decode_layer(self, request_id: str, layer_idx: int, query: torch.Tensor,
                     key: torch.Tensor, value: torch.Tensor,
                     score_scale: float = 1.0) -> torch.Tensor:
        if request_id not in self._k:
            raise KeyError(f"Unknown request {request_id}")
        q = query.detach().cpu().contiguous()
        kn = key.detach().cpu().contiguous()
        vn = value.detach().cpu().contiguous()
        q = q.squeeze(0) if q.dim() == 3 else q
        kn = kn.squeeze(0) if kn.dim() == 3 else kn
        vn = vn.squeeze(0) if vn.dim() == 3 else vn

        layers_k, layers_v = self._k[request_id], self._v[request_id]
        layers_k[layer_idx] = torch.cat([layers_k[layer_idx], kn.unsqueeze(0)], dim=0)
        layers_v[layer_idx] = torch.cat([layers_v[layer_idx], vn.unsqueeze(0)], dim=0)
        keys, values = layers_k[layer_idx], layers_v[layer_idx]

        ctx = attend(q, keys, values, score_scale, out_dtype=query.dtype)

        if layer_idx == len(layers_k) - 1:
            self._ctx[request_id] += 1
        return ctx.unsqueeze(0)

    # attention_backend.py:125-136
    def decode_layer_batch(self, items: List[Dict[str, object]]) -> List[torch.Tensor]:
        out = []
        for it in items:
            out.append(self.decode_layer(str(it["request_id"]), int(it["layer_idx"]),
                                         it["query"], it["key"], it["value"],
                                         float(it.get("score_scale", 1.0))))
        return out

    # attention_backend.py:138-144
    def get_context_len(self, request_id: str) -> int:
        return self._ctx[request_id]

    def free_request(self, request_id: str) -> None:
        self._k.pop(request_id, None)
        self._v.pop(request_id, None)
        self._ctx.pop(request_id, None)
