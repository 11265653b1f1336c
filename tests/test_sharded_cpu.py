"""Head-sharded output gather on CPU ranks (gloo, world size 2): every rank
ends with the full [T, Hq, D] in head order, for even and uneven KV-head
splits, and the rank -> KV-head map is the upstream balanced split."""

from __future__ import annotations

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, hkv, group, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from cloverinfer_b200.sharded import HeadShardGroup
        sg = HeadShardGroup()
        lo, hi = sg.kv_range(hkv)
        T, D = 3, 4
        full = torch.arange(T * hkv * group * D, dtype=torch.float32).reshape(T, hkv * group, D)
        local = full[:, lo * group:hi * group].contiguous()
        got = sg.gather(local, hkv, group)
        q.put((rank, (lo, hi), bool(torch.equal(got, full))))
    except Exception as e:  # report instead of leaving the parent waiting
        q.put((rank, None, repr(e)))
    finally:
        dist.destroy_process_group()


def _run(hkv, group, world=2):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, hkv, group, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted((q.get(timeout=120) for _ in procs), key=lambda r: r[0])
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return res


def test_gather_even_split():
    res = _run(hkv=8, group=4)
    assert [r[1] for r in res] == [(0, 4), (4, 8)], res
    assert all(r[2] is True for r in res), res


def test_gather_uneven_split():
    res = _run(hkv=3, group=2)
    assert [r[1] for r in res] == [(0, 2), (2, 3)], res
    assert all(r[2] is True for r in res), res
