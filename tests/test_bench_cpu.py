"""The bench's parity checker, on the CPU.

``bench.reference_step`` recomputes a step with plain torch fp32 attention over
the paged cache; here it is held to the CPU oracle (``oracle.attend`` over
``repeat_kv``-expanded K/V gathered through the block table) on a small GQA
case with multi-token causal rows, and ``bench.check_parity`` must pass the
oracle's own output, flag a planted error in it, and count a corrupted
appended token.  No GPU is used.
"""

from __future__ import annotations

import dataclasses
import math
from types import SimpleNamespace

import torch

import bench
from cloverinfer_b200.workloads import CONFIGS
from oracle import attend, repeat_kv


def _step(seed=3):
    g = torch.Generator().manual_seed(seed)
    cfg = dataclasses.replace(CONFIGS["c4"], num_q_heads=8, num_kv_heads=2, head_dim=64,
                              block_size=16, dtype=torch.float16)
    hq, hkv, D, bs = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim, cfg.block_size
    lens, n_new = [37, 16, 90], [2, 1, 3]
    nblk = [-(-n // bs) for n in lens]
    nb = sum(nblk) + 3
    k = torch.randn(1, nb, bs, hkv, D, generator=g).half()
    v = torch.randn(1, nb, bs, hkv, D, generator=g).half()
    perm = torch.randperm(nb, generator=g).to(torch.int32)
    tables = torch.full((len(lens), max(nblk) + 1), -1, dtype=torch.int32)
    o = 0
    for i, c in enumerate(nblk):
        tables[i, :c] = perm[o:o + c]
        o += c
    T = sum(n_new)
    q = torch.randn(T, hq, D, generator=g).half().float()
    kn, vn = torch.empty(T, hkv, D).half(), torch.empty(T, hkv, D).half()
    ctx_rows, r = [], 0
    kf, vf = k[0].view(-1, hkv, D), v[0].view(-1, hkv, D)
    for i, (n, c) in enumerate(zip(lens, n_new)):
        for j in range(c):
            pos = n - c + j
            slot = int(tables[i, pos // bs]) * bs + pos % bs
            kn[r + j], vn[r + j] = kf[slot], vf[slot]  # the step appended these
            ctx_rows.append(pos + 1)
        r += c
    st = dict(pool=SimpleNamespace(k=k, v=v, tables=tables), q=q, hq_local=hq, hkv_local=hkv,
              rows=T, n_new=n_new, ctx_rows=ctx_rows, k_new=kn, v_new=vn)
    return cfg, st, lens


def _oracle(cfg, st, lens):
    bs, D, hkv = cfg.block_size, cfg.head_dim, cfg.num_kv_heads
    grp = cfg.num_q_heads // hkv
    kf, vf = st["pool"].k[0].view(-1, hkv, D), st["pool"].v[0].view(-1, hkv, D)
    out, r = [], 0
    for i, (n, c) in enumerate(zip(lens, st["n_new"])):
        slots = [int(st["pool"].tables[i, t // bs]) * bs + t % bs for t in range(n)]
        for j in range(c):
            lim = st["ctx_rows"][r + j]
            out.append(attend(st["q"][r + j], repeat_kv(kf[slots[:lim]], grp),
                              repeat_kv(vf[slots[:lim]], grp), cfg.score_scale, torch.float32))
        r += c
    return torch.stack(out)


def test_reference_step_matches_the_oracle():
    cfg, st, lens = _step()
    ref, mism = bench.reference_step(cfg, st, lens, torch.device("cpu"))
    assert mism == 0
    want = _oracle(cfg, st, lens)
    assert float((ref - want).abs().max()) < 1e-5


def test_check_parity_passes_and_flags():
    cfg, st, lens = _step()
    want = _oracle(cfg, st, lens)
    res = bench.check_parity(cfg, st, lens, 1, torch.device("cpu"), want)
    assert res["pass"] and res["max_abs"] < 1e-5 and res["rows_checked"] == sum(st["n_new"])
    bad = want.clone()
    bad[2, 5, 7] += 5e-3
    res = bench.check_parity(cfg, st, lens, 1, torch.device("cpu"), bad)
    assert not res["pass"] and res["max_abs"] > 4e-3
    st["k_new"][1, 0, 3] += 1.0  # the cache no longer holds this step's token
    res = bench.check_parity(cfg, st, lens, 1, torch.device("cpu"), want)
    assert res["append_mismatches"] == 1 and not res["pass"]
    assert math.isclose(res["tolerance"]["max_abs"], 2e-3)


def test_l2_copies_rule():
    l2 = 132_644_864  # B200: 126.5 MiB
    assert bench.l2_copies(1_073_741_824, l2) == 1            # C3 on one GPU
    assert bench.l2_copies(2 * l2, l2) == 1
    assert bench.l2_copies(134_217_728, l2) == 3               # one rank's C3 share at 8 GPUs
    assert bench.l2_copies(165_150_720, l2) == 3               # C2
    assert bench.l2_copies(8_000_000, l2) == 35                # C1
    assert bench.l2_copies(1, l2) == 64
    for kv in (10_000_000, 100_000_000, 200_000_000):
        n = bench.l2_copies(kv, l2)
        assert (n - 1) * kv >= 2 * l2 or n == 64  # the others fill 2 x L2 between reuses
