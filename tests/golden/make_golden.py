"""Generate the golden vectors that pin the oracle and the host logic.

Run in a container where the upstream CloverInfer sources are mounted:

    python tests/golden/make_golden.py --reference <path-to-CloverInfer>

It imports the upstream modules THEMSELVES (no Ray needed) and records, on
small seeded inputs:

* ``cpu_backend.pt``  — ``CpuAttentionBackend`` (src/core/attention_backend.py:56-144)
  outputs and context lengths over multi-layer, multi-step, GQA(repeat_kv)
  and sequential multi-token decode scenarios;
* ``kv_manager.pt``   — a seeded stream of ``KVCacheManager`` operations
  (src/core/memory_manager.py:55-173): every ``append_slot`` return value,
  the free stack, block tables and lengths after each op, OOM errors, padded
  ``get_kernel_inputs`` and ``_paged_attention_ref`` outputs (:192-239);
* ``head_groups.json`` — the head-grouping policy
  (src/core/attention_backend.py:320-471): group counts, ranges and placements.

The fixtures are small (well under 1 MB) and committed; nothing at test time
reads the upstream tree.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import random
import sys
import types

import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(root: str):
    sys.dont_write_bytecode = True
    sys.path.insert(0, os.path.join(root, "src"))
    from core.attention_backend import CpuAttentionBackend, PimNaiveAttentionBackend  # noqa
    from core.memory_manager import KVCacheManager  # noqa
    return CpuAttentionBackend, PimNaiveAttentionBackend, KVCacheManager


def _rk(x: torch.Tensor, n_rep: int) -> torch.Tensor:
    if n_rep == 1:
        return x
    *lead, h, d = x.shape
    return x.unsqueeze(-2).expand(*lead, h, n_rep, d).reshape(*lead, h * n_rep, d)


def _backend_scenario(Backend, name, *, seed, ctx0, n_layers, hq, hkv, d, kv_dtype,
                      q_dtype, steps, score_scale, tokens_per_step=1, q_mult=1.0, kv_mult=1.0):
    """Drive the upstream backend; record inputs (un-expanded KV) and outputs."""
    g = torch.Generator().manual_seed(seed)
    rep = hq // hkv
    be = Backend()
    reqs = []
    for r, c in enumerate(ctx0):
        rid = f"{name}-r{r}"
        layers = []
        for _ in range(n_layers):
            k = (torch.randn(c, hkv, d, generator=g) * kv_mult).to(kv_dtype)
            v = (torch.randn(c, hkv, d, generator=g) * kv_mult).to(kv_dtype)
            layers.append({"key": k, "value": v})
        ret = be.init_request(rid, [{"key": _rk(l["key"], rep), "value": _rk(l["value"], rep)}
                                    for l in layers])
        reqs.append({"id": rid, "initial_kv": layers, "init_ret": ret})
    calls = []
    for s in range(steps):
        for layer in range(n_layers):
            for t in range(tokens_per_step):
                items, raw = [], []
                for r in reqs:
                    q = (torch.randn(hq, d, generator=g) * q_mult).to(q_dtype)
                    k = (torch.randn(hkv, d, generator=g) * kv_mult).to(kv_dtype)
                    v = (torch.randn(hkv, d, generator=g) * kv_mult).to(kv_dtype)
                    items.append({"request_id": r["id"], "layer_idx": layer, "query": q,
                                  "key": _rk(k, rep), "value": _rk(v, rep),
                                  "score_scale": score_scale})
                    raw.append({"request_id": r["id"], "layer_idx": layer, "query": q,
                                "key": k, "value": v, "score_scale": score_scale})
                outs = be.decode_layer_batch(items)
                calls.append({"step": s, "layer": layer, "token": t, "items": raw,
                              "outputs": [o.clone() for o in outs],
                              "ctx_after": [be.get_context_len(r["id"]) for r in reqs]})
    return {"name": name, "hq": hq, "hkv": hkv, "d": d, "n_layers": n_layers,
            "score_scale": score_scale, "requests": reqs, "calls": calls}


def make_cpu_backend(Backend):
    scen = [
        # OPT-125m-like: MHA fp32, q pre-scaled upstream so score_scale = 1.0
        _backend_scenario(Backend, "opt", seed=1, ctx0=[9, 21], n_layers=2, hq=4, hkv=4,
                          d=64, kv_dtype=torch.float32, q_dtype=torch.float32, steps=2,
                          score_scale=1.0, q_mult=0.125),
        # Qwen-like GQA (g=7) bf16 KV, fp32 queries so the output stays fp32
        _backend_scenario(Backend, "gqa7", seed=2, ctx0=[40, 17], n_layers=2, hq=14, hkv=2,
                          d=128, kv_dtype=torch.bfloat16, q_dtype=torch.float32, steps=2,
                          score_scale=1.0 / math.sqrt(128), q_mult=0.5, kv_mult=0.5),
        # Llama-like GQA (g=4) bf16 KV with bf16 queries (output in bf16)
        _backend_scenario(Backend, "gqa4bf16", seed=3, ctx0=[31, 16], n_layers=1, hq=8, hkv=2,
                          d=128, kv_dtype=torch.bfloat16, q_dtype=torch.bfloat16, steps=2,
                          score_scale=1.0 / math.sqrt(128)),
        # multi-token append = sequential single-token calls (fp16 KV)
        _backend_scenario(Backend, "multitok", seed=4, ctx0=[15, 33], n_layers=1, hq=8, hkv=2,
                          d=64, kv_dtype=torch.float16, q_dtype=torch.float32, steps=1,
                          score_scale=0.125, tokens_per_step=3),
    ]
    return {"scenarios": scen}


def make_kv_manager(Manager):
    rnd = random.Random(7)
    bs, nb = 4, 20
    mgr = Manager(nb, bs, 2, 8, dtype=torch.float32, device="cpu")
    ops, live, nxt = [], [], 0
    for _ in range(160):
        r = rnd.random()
        op = {}
        try:
            if (r < 0.22 or not live) and len(live) < 8:
                rid = f"q{nxt}"; nxt += 1
                n = rnd.choice([0, 0, 1, 3, 4, 5, 7, 8, 15, 16, 17, 30])
                op = {"op": "allocate", "id": rid, "seq_len": n}
                mgr.allocate(rid, seq_len=n)
                live.append(rid)
            elif r < 0.80:
                rid = rnd.choice(live)
                op = {"op": "append_slot", "id": rid}
                op["ret"] = list(mgr.append_slot(rid))
            else:
                rid = rnd.choice(live)
                op = {"op": "free", "id": rid}
                mgr.free(rid)
                live.remove(rid)
        except RuntimeError as e:
            op["error"] = str(e)
            if op["op"] == "allocate" and op["id"] in mgr.block_tables:
                live.append(op["id"])
        op["free_blocks"] = list(mgr.free_blocks)
        op["tables"] = {k: list(v) for k, v in mgr.block_tables.items()}
        op["ctx"] = dict(mgr.context_lens)
        ops.append(op)
    ids = sorted(mgr.block_tables)
    tables, lens, mx = mgr.get_kernel_inputs(ids) if ids else (torch.zeros(0, 0), torch.zeros(0), 0)

    # The upstream pins (tests/test_kernels.py:8-34, tests/verify_attention.py:88-136),
    # re-expressed with the slow reference as the recorded answer.
    pin = Manager(16, 4, 2, 8, dtype=torch.float32, device="cpu")
    pin.allocate("req_1", seq_len=0)
    for _ in range(5):
        pin.append_slot("req_1")
    pin_tables = list(pin.block_tables["req_1"])
    g = torch.Generator().manual_seed(11)
    ref = Manager(100, 16, 4, 32, dtype=torch.float32, device="cpu")
    ref.allocate("req_test_kernel", seq_len=0)
    k = torch.randn(4, 32, generator=g)
    v = torch.randn(4, 32, generator=g)
    for _ in range(50):
        ref.write_new_kv("req_test_kernel", k, v)
    q = torch.randn(1, 4, 32, generator=g)
    out_ref = ref._paged_attention_ref(q, ["req_test_kernel"])

    # A ragged multi-request paged reference case with distinct tokens.
    rag = Manager(10, 16, 2, 32, dtype=torch.float32, device="cpu")
    rids = ["a", "b", "c"]
    for rid, n in zip(rids, [5, 37, 70]):
        kk = torch.randn(n, 2, 32, generator=g)
        vv = torch.randn(n, 2, 32, generator=g)
        rag.load_initial_kv(rid, kk, vv)
    qq = torch.randn(3, 2, 32, generator=g)
    rag_out = rag._paged_attention_ref(qq, rids)
    rag_tables, rag_lens, rag_max = rag.get_kernel_inputs(rids)
    return {
        "block_size": bs, "num_blocks": nb, "ops": ops,
        "final_ids": ids, "kernel_tables": tables, "kernel_lens": lens, "kernel_max": mx,
        "pin_ctx": pin.context_lens["req_1"], "pin_tables": pin_tables,
        "pin_ref": {"k": k, "v": v, "q": q, "out": out_ref},
        "ragged": {"ids": rids, "k_cache": rag.k_cache.clone(), "v_cache": rag.v_cache.clone(),
                   "tables": rag_tables, "lens": rag_lens, "max": rag_max, "q": qq, "out": rag_out},
    }


def make_head_groups(Pim):
    class _Store:
        def __init__(self):
            self.calls = []

        def allocate_group(self, k_slot, v_slot, k, v, capacity, preferred_dpu, force_host_fallback):
            self.calls.append(preferred_dpu)

    cases = []
    for policy in ["legacy", "balanced", "coarse", "segment_aware", "universal"]:
        for placement in ["identity", "rotated", "rank_spread"]:
            for ndpu in [1, 2, 3, 8, 64]:
                for heads in [1, 7, 8, 12, 32]:
                    for seq in [1, 100, 192, 512]:
                        for hd in [64, 128]:
                            obj = object.__new__(Pim)
                            obj.num_dpus = ndpu
                            obj.head_grouping_policy = policy
                            obj.dpu_placement_policy = placement
                            obj.length = 16
                            obj.max_resident_groups_per_layer = 0
                            obj.resident_store = _Store()
                            n = obj._effective_head_group_count(seq, heads, hd)
                            key = torch.zeros(seq if seq <= 512 else 1, heads, hd, dtype=torch.int8)
                            # _build_head_groups reads seq_len from the tensor shape;
                            # use the real seq_len only where it is cheap.
                            if seq > 512:
                                continue
                            groups = obj._build_head_groups("req-xyz", 3, key, key)
                            cases.append([policy, placement, ndpu, heads, seq, hd, n,
                                          [[gr.head_start, gr.head_end] for gr in groups],
                                          [gr.dpu_id for gr in groups]])
    counts = []
    for policy in ["legacy", "balanced", "coarse", "segment_aware", "universal"]:
        for ndpu in [1, 2, 4, 8, 16, 64, 256]:
            for heads in [1, 8, 12, 28, 32, 40, 64, 96]:
                for seq in [1, 64, 128, 192, 256, 512, 1024, 4096, 32768, 65536]:
                    for hd in [64, 128]:
                        obj = object.__new__(Pim)
                        obj.num_dpus = ndpu
                        obj.head_grouping_policy = policy
                        counts.append([policy, ndpu, heads, seq, hd,
                                       obj._effective_head_group_count(seq, heads, hd)])
    return {"build": cases, "counts": counts}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the CloverInfer checkout")
    a = ap.parse_args()
    Backend, Pim, Manager = _import_reference(a.reference)
    torch.save(make_cpu_backend(Backend), os.path.join(HERE, "cpu_backend.pt"))
    torch.save(make_kv_manager(Manager), os.path.join(HERE, "kv_manager.pt"))
    with open(os.path.join(HERE, "head_groups.json"), "w") as f:
        json.dump(make_head_groups(Pim), f, separators=(",", ":"))
    for fn in ["cpu_backend.pt", "kv_manager.pt", "head_groups.json"]:
        print(fn, os.path.getsize(os.path.join(HERE, fn)))


if __name__ == "__main__":
    main()
