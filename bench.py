"""Benchmark: paged decode-attention KV-read GB/s (and attention steps/s).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config c3] [--impl b200|reference]

Under torchrun (N > 1) each rank owns Hkv/N KV heads (head sharding) and the
step ends with the all-gather of the per-rank outputs, fused into the split-K
reduce over NVLink (``--gather nccl``: one NCCL all-gather instead).

One "step" = one attention step of one layer for the whole batch at the
configuration's context length: KV append of each sequence's new token fused
with the paged decode (split-K) -> split-K reduce (-> all-gather).  ``value`` times K
such steps on device-resident inputs, captured back to back in one CUDA graph
as consecutive layers run (each step waits for the previous one: they share
the split-K workspace), between CUDA events, max over ranks; W warm-up steps
run the same way before.  ``e2e`` times the same step through the public
``B200AttentionBackend.decode_layer_batch`` API with host (pinned) inputs and
outputs, as the attention node calls it.  The metric is algorithmic KV bytes
read per step (sum_s ctx_s * Hkv * D * 2 * elem) / step time, whole job.

``--impl reference`` times the CPU reference implementation (the oracle port
of CloverInfer's CpuAttentionBackend, all host threads) on a bounded sample of
the same workload and prints the same metric.

After the timed region every rank runs one more (untimed) step and checks the
all-gathered output of EVERY row and head against a plain torch fp32 attention
over the same cache contents (and the appended K/V bit for bit); the worst
error over all ranks is the line's ``parity``.  ``spread`` holds the per-step
times of 30 further, individually timed graph replays, and ``as_configured``
the same measurement with the configuration's own partition length (512
tokens for c3) next to the library's choice.

``--profile-share W`` is the ncu case for one rank of a W-way KV-head shard:
it builds rank ``--profile-rank`` 's share of the step on one GPU and launches
the decode (+ split-K reduce) ``--launches`` times, printing no JSON.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "paged decode-attn KV-read GB/s"

# DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum) of one
# paged_decode_mma_kernel launch from an ncu capture of the same workload and
# kernel build: (config, GPUs, KV dtype option) -> (bytes, summary file).
NCU_TRAFFIC = {
    ("c3", 1, "config"): (1.074150e9 + 9.415e6, "profiles/paged_decode_mma_c3_full.md"),
    ("c3", 8, "config"): (134.347e6 + 4.144e6, "profiles/paged_decode_mma_c3_shard8_full.md"),
    ("c4", 1, "config"): (2.324122e9 + 29.423e6, "profiles/paged_decode_mma_c4_full.md"),
}


def _peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "100"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def config_for(args):
    """The workload of ``--config``, with the KV cache in fp8 under ``--kv-dtype fp8``."""
    import dataclasses
    from cloverinfer_b200.workloads import CONFIGS
    cfg = CONFIGS[args.config]
    if getattr(args, "kv_dtype", "config") == "fp8":
        cfg = dataclasses.replace(cfg, name=cfg.name + "-fp8kv", dtype=torch.float8_e4m3fn)
    return cfg


def _dist_setup():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world > 1:
        import torch.distributed as dist
        local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local),
                                timeout=__import__("datetime").timedelta(seconds=120))
        return dist.get_rank(), world, local
    return 0, 1, 0


def _max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _barrier(world: int):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ------------------------------------------------------------------ CPU baseline
def cpu_reference_seconds_per_step(cfg, lens, sample_seqs: int, calls: int):
    """Time the oracle port of CpuAttentionBackend.decode_layer on a sample of
    the workload's sequences (repeat_kv-expanded KV, as upstream requires);
    return the extrapolated seconds for one whole-batch step."""
    from oracle import CpuAttentionOracle, repeat_kv
    from cloverinfer_b200.workloads import randn
    torch.set_num_threads(os.cpu_count() or 1)
    be = CpuAttentionOracle()
    hq, hkv, D, dt = cfg.num_q_heads, cfg.num_kv_heads, cfg.head_dim, cfg.dtype
    times = []
    sample = lens[:sample_seqs]
    for i, n in enumerate(sample):
        k = repeat_kv(randn((n - 1, hkv, D), 100 + i, cfg.value_scale, dt), cfg.group)
        v = repeat_kv(randn((n - 1, hkv, D), 200 + i, cfg.value_scale, dt), cfg.group)
        be.init_request(f"s{i}", [{"key": k, "value": v}])
    q = randn((hq, D), 1, cfg.value_scale, torch.float32)
    kn = repeat_kv(randn((1, hkv, D), 2, cfg.value_scale, dt), cfg.group)[0]
    vn = repeat_kv(randn((1, hkv, D), 3, cfg.value_scale, dt), cfg.group)[0]
    for c in range(calls + 1):
        t0 = time.perf_counter()
        for i in range(len(sample)):
            be.decode_layer(f"s{i}", 0, q, kn, vn, cfg.score_scale)
        dt_s = time.perf_counter() - t0
        if c > 0:
            times.append(dt_s)
        for i in range(len(sample)):  # keep the sample at the configured length
            be._k[f"s{i}"][0] = be._k[f"s{i}"][0][:-1]
            be._v[f"s{i}"][0] = be._v[f"s{i}"][0][:-1]
    per_sample = statistics.median(times)
    return per_sample * sum(lens) / sum(sample), torch.get_num_threads()


def run_reference(args):
    rank, world, _ = int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")), 0
    if rank != 0:
        return
    from cloverinfer_b200.workloads import CONFIGS, context_lengths, kv_bytes
    cfg = config_for(args)
    lens = context_lengths(cfg, 0)
    nbytes = kv_bytes(lens, cfg.num_kv_heads, cfg.head_dim, cfg.dtype)
    per_step = []
    threads = None
    for _ in range(args.warmup):
        cpu_reference_seconds_per_step(cfg, lens, 1, 1)
    for _ in range(args.steps):
        s, threads = cpu_reference_seconds_per_step(cfg, lens, 1, 1)
        per_step.append(s)
    sec = statistics.median(per_step)
    val = nbytes / sec / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "GB/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(sec * 1e3, 3), "higher_is_better": True, "scaling": "strong",
        "vs_baseline": None, "dtype": str(cfg.dtype).replace("torch.", ""), "data": "synthetic",
        "config": {"workload": cfg.name, "batch": cfg.batch, "ctx": f"{cfg.ctx_lo}-{cfg.ctx_hi}",
                   "num_q_heads": cfg.num_q_heads, "num_kv_heads": cfg.num_kv_heads,
                   "head_dim": cfg.head_dim, "block_size": cfg.block_size},
        "steps_per_s": round(1.0 / sec, 4),
        "cpu_baseline": {"value": round(val, 4), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": "1 of %d sequences per step (full context, repeat_kv-expanded "
                                   "KV, decode_layer incl. the upstream cache concatenation), "
                                   "scaled by total context" % cfg.batch},
        "e2e": {"value": round(val, 4), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------------ B200 arm
def l2_copies(kv_bytes_per_step: int, l2_bytes: int) -> int:
    """Independent copies of a workload the timed steps rotate over: 1 when a
    step's KV is at least twice the L2, else enough that the copies together
    exceed twice the L2 with one to spare (at most 64), so the KV a step
    reads was last touched more than 2 x L2 bytes earlier."""
    if kv_bytes_per_step >= 2 * l2_bytes:
        return 1
    return min(64, -(-2 * l2_bytes // max(kv_bytes_per_step, 1)) + 1)


def build_step(cfg, rank, world, lens, device, seed=0, gather=None, n_new=None, partition_tokens=0):
    from cloverinfer_b200.workloads import build_decode_step
    return build_decode_step(cfg, rank, world, lens, device, seed=seed, gather=gather, n_new=n_new,
                             partition_tokens=partition_tokens)


def _replay_ms(graph, stream, replays: int, steps: int, min_seconds: float = 0.0):
    """Per-step ms of individually timed replays of a `steps`-step graph: at
    least `replays` of them, and more until `min_seconds` have passed (so the
    clock sampler sees the GPU under load)."""
    out = []
    t0 = time.perf_counter()
    while len(out) < replays or time.perf_counter() - t0 < min_seconds:
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
               for _ in range(replays)]
        with torch.cuda.stream(stream):
            for e0, e1 in evs:
                e0.record(stream)
                graph.replay()
                e1.record(stream)
        torch.cuda.synchronize()
        out += [a.elapsed_time(b) / steps for a, b in evs]
    return out


def _spread(ms):
    s = sorted(ms)
    pick = lambda f: s[min(len(s) - 1, max(0, int(round(f * (len(s) - 1)))))]  # noqa: E731
    return {"replays": len(s), "median_ms": round(statistics.median(s), 5),
            "p10_ms": round(pick(0.1), 5), "p90_ms": round(pick(0.9), 5)}


def _bits(t: torch.Tensor) -> torch.Tensor:
    return t.view({1: torch.uint8, 2: torch.int16, 4: torch.int32}[t.element_size()])


def reference_step(cfg, st, lens, device):
    """This rank's heads of the step, recomputed with plain torch fp32
    attention over the cache as the step left it: row r of sequence b attends
    to its first ctx_r tokens (softmax(scale q.K^T).V, the math of
    CpuAttentionBackend.decode_layer, src/core/attention_backend.py:113-118).
    Also counts appended tokens whose cached K or V differ, bit for bit, from
    the step's new K/V.  Returns ([T, Hq_local, D] fp32, mismatches)."""
    pool, q = st["pool"], st["q"]
    hq_l, hkv_l, D, bs = st["hq_local"], st["hkv_local"], cfg.head_dim, cfg.block_size
    grp = hq_l // hkv_l
    K = pool.k[0].view(-1, hkv_l, D)
    V = pool.v[0].view(-1, hkv_l, D)
    T = q.shape[0]
    ref = torch.empty((T, hq_l, D), dtype=torch.float32, device=device)
    ctx = torch.tensor(st["ctx_rows"], dtype=torch.int64, device=device)
    lane = torch.arange(bs, device=device)
    mism = torch.zeros((), dtype=torch.int64, device=device)
    r = 0
    for b, (n, k) in enumerate(zip(lens, st["n_new"])):
        blocks = pool.tables[b, :-(-n // bs)].long()
        slots = (blocks[:, None] * bs + lane).reshape(-1)[:n]
        new = slots[n - k:]
        mism += (_bits(K[new]) != _bits(st["k_new"][r:r + k])).flatten(1).any(1).sum()
        mism += (_bits(V[new]) != _bits(st["v_new"][r:r + k])).flatten(1).any(1).sum()
        kb, vb = K[slots].float(), V[slots].float()
        qb = q[r:r + k].float().view(k, hkv_l, grp, D)
        s = torch.einsum("jhgd,lhd->jhgl", qb, kb) * cfg.score_scale
        masked = torch.arange(n, device=device)[None, :] >= ctx[r:r + k, None]
        s.masked_fill_(masked[:, None, None, :], float("-inf"))
        ref[r:r + k] = torch.einsum("jhgl,lhd->jhgd", torch.softmax(s, dim=-1), vb).reshape(k, hq_l, D)
        r += k
    return ref, int(mism)


def check_parity(cfg, st, lens, world, device, gathered):
    """Worst error of the gathered [T, Hq, D] output (every row and head) on
    every rank against the torch fp32 reference of all ranks' heads; same
    collective sequence on every rank, errors included."""
    err = [float("nan"), float("nan"), 0.0, 0.0]
    ref_local = None
    try:
        ref_local, mism = reference_step(cfg, st, lens, device)
        err[2] = float(mism)
    except Exception as e:  # keep the collectives in step; report the failure
        print(f"parity reference failed: {e!r}", file=sys.stderr)
        err[2] = -1.0
    T, hq_l, D = st["rows"], st["hq_local"], cfg.head_dim
    if ref_local is None:
        ref_local = torch.zeros((T, hq_l, D), dtype=torch.float32, device=device)
    if world > 1:
        import torch.distributed as dist
        allr = torch.empty((world * T, hq_l, D), dtype=torch.float32, device=device)
        dist.all_gather_into_tensor(allr, ref_local.contiguous())
        ref = allr.view(world, T, hq_l, D).permute(1, 0, 2, 3).reshape(T, world * hq_l, D)
    else:
        ref = ref_local
    if err[2] >= 0:
        o = gathered.float()
        e = (o - ref).abs()
        err[0] = float(e.max())
        err[1] = float((e / ref.abs().clamp_min(1e-3)).max())
        err[3] = float((~torch.isfinite(o)).sum())
    t = torch.tensor(err, dtype=torch.float64, device=device)
    if world > 1:
        import torch.distributed as dist
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    max_abs, max_rel, mism, nonfinite = (float(x) for x in t.tolist())
    ok = (mism == 0 and nonfinite == 0 and max_abs <= 2e-3 and max_rel <= 1e-2)
    return {"max_abs": max_abs, "max_rel": max_rel, "rows_checked": T,
            "heads_checked": cfg.num_q_heads, "append_mismatches": int(mism),
            "nonfinite": int(nonfinite), "pass": bool(ok),
            "reference": "torch fp32 attention over the cache contents, all rows and heads, "
                         "checked on every rank (worst rank reported); appended K/V bit-exact",
            "tolerance": {"max_abs": 2e-3, "max_rel_floored": 1e-2}}


def run_profile_share(args):
    """One rank's share of a W-way sharded step on one GPU, decode (+ reduce)
    launched --launches times: the case ncu captures for a multi-GPU rank."""
    from cloverinfer_b200.workloads import build_decode_step, context_lengths, new_tokens
    cfg = config_for(args)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    lens = context_lengths(cfg, 0, args.batch)
    pt = args.partition_tokens if args.partition_tokens is not None else 0
    st = build_decode_step(cfg, args.profile_rank, args.profile_share, lens, dev,
                           n_new=new_tokens(cfg, 0, args.batch), partition_tokens=pt,
                           pool_blocks=0)  # a small device footprint for ncu's replays
    for _ in range(args.launches):
        st["decode_only"]()
    torch.cuda.synchronize()
    st["pool"].check_status()
    msg = ""
    if args.time_share:
        # the share's decode (+ reduce) back to back in one graph, as the timed
        # step chains them (no gather: a single GPU)
        stream = torch.cuda.Stream(dev)
        g = _capture(st["decode_only"], args.launches, stream)
        with torch.cuda.stream(stream):
            g.replay()
        torch.cuda.synchronize()
        reps = _replay_ms(g, stream, args.replays, args.launches)
        g.reset()
        msg = f", per launch {1e3 * statistics.median(reps):.2f} us (median of {len(reps)} replays)"
    print(f"{cfg.name}: rank {args.profile_rank}/{args.profile_share}, {st['hkv_local']} KV heads, "
          f"partition {st['partition_tokens']} tokens, {args.launches} launches ok{msg}")


def _step_runner(st, world, T, cfg, device):
    """The full step of a built workload (the step, plus an NCCL all-gather
    when the fused peer gather is not in use) and a function returning the
    gathered [T, Hq, D] output the last step left."""
    peer = st.get("peer")
    if world == 1:
        return st["step"], lambda: st["out"]
    if peer is not None:
        return st["step"], lambda: peer.out[:T]
    import torch.distributed as dist
    hq_l, D = st["hq_local"], cfg.head_dim
    recv = torch.empty((world * T, hq_l, D), dtype=st["out"].dtype, device=device)

    def full_step():
        st["step"]()
        dist.all_gather_into_tensor(recv, st["out"])

    return full_step, lambda: recv.view(world, T, hq_l, D).permute(1, 0, 2, 3).reshape(T, world * hq_l, D)


def _capture(fn, steps, stream):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        for _ in range(steps):
            fn()
    return g


def run_b200(args):
    from cloverinfer_b200 import _lib
    from cloverinfer_b200.workloads import kv_bytes, new_tokens, context_lengths

    rank, world, local = _dist_setup()
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    _lib.lib()
    cfg = config_for(args)
    lens = context_lengths(cfg, 0, args.batch)
    n_new = new_tokens(cfg, 0, args.batch)
    B = len(lens)
    T = sum(n_new)
    total_kv = kv_bytes(lens, cfg.num_kv_heads, cfg.head_dim, cfg.dtype)
    peer = None
    if world > 1 and args.gather == "peer":
        from cloverinfer_b200.sharded import HeadShardGroup, PeerGather
        peer = PeerGather(HeadShardGroup(), T, cfg.num_q_heads, cfg.head_dim, torch.float32, device)
    pt_arg = args.partition_tokens if args.partition_tokens is not None else 0
    st = build_step(cfg, rank, world, lens, device, gather=peer, n_new=n_new, partition_tokens=pt_arg)
    st["peer"] = peer
    local_kv = kv_bytes(lens, st["hkv_local"], cfg.head_dim, cfg.dtype)
    # A step whose KV fits twice in L2 (C1, C2) would find it there on the
    # next step: the timed steps then rotate over independent copies of the
    # workload (own pool, tables and buffers), more than 2 x L2 in all.
    l2 = torch.cuda.get_device_properties(device).L2_cache_size
    n_copies = l2_copies(local_kv, l2)
    copies = [st] + [dict(build_step(cfg, rank, world, lens, device, seed=c, gather=peer, n_new=n_new,
                                     partition_tokens=pt_arg), peer=peer) for c in range(1, n_copies)]
    runners = [_step_runner(c, world, T, cfg, device) for c in copies]
    full_step, gathered = runners[0]
    rot = {"i": 0}

    def step_rot():
        # the next copy's step (the order is fixed when a graph captures it)
        runners[rot["i"] % n_copies][0]()
        rot["i"] += 1

    def decode_rot():
        copies[rot["i"] % n_copies]["decode_only"]()
        rot["i"] += 1

    stream = torch.cuda.Stream(device)
    stream.wait_stream(torch.cuda.current_stream(device))
    launches_per_step = 1 + (1 if st["workspace_bytes"] > 0 or peer is not None else 0)
    gather_kind = "none" if world == 1 else ("fused-peer-stores" if peer is not None else "nccl")

    with torch.cuda.stream(stream):
        for _ in range(3):  # eager warm-up (module load, tensor maps, NCCL comm init)
            for run, _ in runners:
                run()
    torch.cuda.synchronize(device)
    # K timed steps back to back in one CUDA graph: one graph launch per K
    # steps, and programmatic dependent launch between a step's reduce and the
    # next step's decode.  The warm-up replays the same graph (its first launch
    # also uploads it), so at least W steps run untimed.
    rot["i"] = 0
    graph = None if args.no_graph else _capture(step_rot, args.steps, stream)
    warm_replays = -(-args.warmup // args.steps)
    warm_steps = warm_replays * args.steps if graph is not None else args.warmup

    def run_steps(n):
        if graph is not None:
            graph.replay()
        else:
            for _ in range(n):
                step_rot()

    with torch.cuda.stream(stream):
        for _ in range(warm_replays if graph is not None else 1):
            run_steps(args.warmup)
    torch.cuda.synchronize(device)
    for c in copies:
        c["pool"].check_status()

    vis = os.environ.get("CUDA_VISIBLE_DEVICES")
    clocks = ClockSampler(vis.split(",")[local] if vis else str(local))
    clocks.start()
    time.sleep(0.3)
    _barrier(world)
    torch.cuda.synchronize(device)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        run_steps(args.steps)
        e1.record(stream)
    torch.cuda.synchronize(device)
    _barrier(world)
    ms = e0.elapsed_time(e1) / args.steps
    ms = _max_over_ranks(ms, world)

    # Spread: further replays of the same graph, each timed on its own.
    spread = None
    if graph is not None:
        _barrier(world)
        reps = _replay_ms(graph, stream, args.replays, args.steps, min_seconds=1.0)
        # every rank times the same number of replays: the max is taken replay by replay
        n = int(_max_over_ranks(float(len(reps)), world))
        while len(reps) < n:
            reps += _replay_ms(graph, stream, 1, args.steps)
        spread = _spread([_max_over_ranks(x, world) for x in reps[:n]])

    # Dominant kernel alone: decode (+ its split-K reduce) launches back to back
    # in one graph, timed between CUDA events on the launching stream (median
    # of the individually timed replays).
    rot["i"] = 0
    dec_graph = _capture(decode_rot, args.steps, stream)
    with torch.cuda.stream(stream):
        dec_graph.replay()
    torch.cuda.synchronize(device)
    dec_reps = _replay_ms(dec_graph, stream, args.replays, args.steps)
    dec_ms = statistics.median(dec_reps)
    clk = clocks.stop()
    for c in copies:
        c["pool"].check_status()
    used_graph = graph is not None
    # Release every graph (one may hold NCCL work) before anything else: a
    # live graph with NCCL calls makes destroy_process_group wait for good.
    if graph is not None:
        graph.reset()
    dec_graph.reset()
    del graph, dec_graph
    torch.cuda.synchronize(device)

    # Parity: one more step, then every row and head against torch fp32.
    with torch.cuda.stream(stream):
        full_step()
    torch.cuda.synchronize(device)
    st["pool"].check_status()
    parity = check_parity(cfg, st, lens, world, device, gathered())

    # The configuration's own partition length next to the library's choice.
    as_cfg = None
    if cfg.partition_tokens and not args.no_graph and cfg.partition_tokens != st["partition_tokens"]:
        st2 = build_step(cfg, rank, world, lens, device, gather=peer, n_new=n_new,
                         partition_tokens=cfg.partition_tokens)
        st2["peer"] = peer
        step2, gathered2 = _step_runner(st2, world, T, cfg, device)
        with torch.cuda.stream(stream):
            step2()
        torch.cuda.synchronize(device)
        g2 = _capture(step2, args.steps, stream)
        with torch.cuda.stream(stream):
            for _ in range(warm_replays):
                g2.replay()
        torch.cuda.synchronize(device)
        _barrier(world)
        reps2 = [_max_over_ranks(x, world) for x in _replay_ms(g2, stream, args.replays, args.steps)]
        g2.reset()
        del g2
        torch.cuda.synchronize(device)
        st2["pool"].check_status()
        with torch.cuda.stream(stream):
            step2()
        torch.cuda.synchronize(device)
        par2 = check_parity(cfg, st2, lens, world, device, gathered2())
        med2 = statistics.median(reps2)
        as_cfg = {"partition_tokens": st2["partition_tokens"],
                  "l2": "one copy of the workload (KV %.0f MB per GPU)" % (local_kv / 1e6),
                  "value": round(total_kv / (med2 * 1e-3) / 1e9, 2), "unit": "GB/s",
                  "ms_per_step": round(med2, 5), "spread": _spread(reps2),
                  "parity": {k: par2[k] for k in ("max_abs", "max_rel", "pass")}}
        del st2
        torch.cuda.empty_cache()

    # ---------------- e2e through the public API (host buffers in, host out)
    e2e = run_e2e(cfg, lens, n_new, rank, world, device, args)

    hbm_peak, peak_kind = _peaks()
    achieved = local_kv / (dec_ms * 1e-3) / 1e9
    value = total_kv / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 5),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
        "dtype": "bf16" if cfg.dtype == torch.bfloat16 else str(cfg.dtype).replace("torch.", ""),
        "data": "synthetic",
        "config": {"workload": cfg.name, "batch": B, "new_tokens": T, "ctx": f"{cfg.ctx_lo}-{cfg.ctx_hi}",
                   "num_q_heads": cfg.num_q_heads, "num_kv_heads": cfg.num_kv_heads,
                   "head_dim": cfg.head_dim, "block_size": cfg.block_size,
                   "partition_tokens": st["partition_tokens"], "pool_blocks": st["pool_blocks"],
                   "split": ("balanced over all resident warps" if st["partition_tokens"] < 0
                             else "%d-token partitions" % st["partition_tokens"]),
                   "parallelism": f"kv-head-shard{world}", "gather": gather_kind,
                   "cuda_graph": ("%d steps per graph" % args.steps) if used_graph else "none",
                   "warmup_steps_run": warm_steps,
                   "l2": ("inputs > L2 (KV %.0f MB per GPU)" % (local_kv / 1e6)) if n_copies == 1 else
                         ("KV %.1f MB per GPU < 2 x L2 (%.0f MB): the timed steps rotate over %d independent "
                          "copies of the workload (%.0f MB in all)"
                          % (local_kv / 1e6, l2 / 1e6, n_copies, n_copies * local_kv / 1e6))},
        "steps_per_s": round(1e3 / ms, 2),
        "tokens_per_s": round(T * 1e3 / ms, 2),
        "pct_hbm_peak_per_gpu": round(100.0 * value / world / hbm_peak, 2),
        "spread": spread,
        "parity": parity,
        "as_configured": as_cfg,
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                     "frac": round(achieved / hbm_peak, 4),
                     "traffic": NCU_TRAFFIC.get((args.config, world, args.kv_dtype), (None,))[0],
                     "traffic_source": NCU_TRAFFIC.get((args.config, world, args.kv_dtype),
                                                       (None, None))[1],
                     "kernel": ("paged_decode_stream_kernel" if st["partition_tokens"] < 0
                                else "paged_decode_mma_kernel") + " + splitk_reduce_kernel",
                     "launch_ms": round(dec_ms, 5), "launch_spread": _spread(dec_reps),
                     "peak_kind": peak_kind},
        "clocks": clk,
        "gpu_launches": launches_per_step * args.steps,
        "e2e": e2e,
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        sec, threads = cpu_reference_seconds_per_step(cfg, lens, 1, 2)
        line["cpu_baseline"] = {"value": round(total_kv / sec / 1e9, 4), "unit": "GB/s",
                                "cores": threads, "kind": "port",
                                "sample": "1 of %d sequences, 2 timed calls (median), scaled by total "
                                          "context; repeat_kv-expanded KV as upstream" % B}
    if rank == 0:
        print(json.dumps(line), flush=True)
    if peer is not None:
        peer.close()
    if world > 1:
        import torch.distributed as dist
        torch.cuda.synchronize(device)
        dist.barrier()
        dist.destroy_process_group()


def run_e2e(cfg, lens, n_new, rank, world, device, args):
    """The public API with host tensors: decode_layer_batch (per-item tensors, as
    AttentionNode calls it) for one new token per sequence, decode_batch (host
    [T, H, D] tensors) for multi-token steps."""
    from cloverinfer_b200 import B200AttentionBackend, HeadShardGroup
    from cloverinfer_b200.workloads import kv_bytes
    shard = HeadShardGroup() if world > 1 else None
    B, D, dt = len(lens), cfg.head_dim, cfg.dtype
    T = sum(n_new)
    steps_total = args.steps + args.warmup
    be = B200AttentionBackend(num_blocks=sum(-(-(n + 4 * steps_total + 16) // cfg.block_size)
                                             for n in lens) + 64,
                              block_size=cfg.block_size, num_kv_heads=cfg.num_kv_heads, kv_dtype=dt,
                              device=device, max_seqs=B, shard=shard, shuffle_seed=77,
                              partition_tokens=0,
                              max_seq_len=max(lens) + 4 * steps_total + 4096, gather=args.gather,
                              max_rows_per_call=T)
    g = torch.Generator(device=device).manual_seed(99)
    lo, hi = (0, cfg.num_kv_heads) if shard is None else shard.kv_range(cfg.num_kv_heads)
    for i, (n, k) in enumerate(zip(lens, n_new)):
        # prefill KV built on the device for speed; heads outside this rank's
        # shard are never read, so they are left as zeros
        kk = torch.zeros((n - k, cfg.num_kv_heads, D), dtype=dt, device=device)
        vv = torch.zeros_like(kk)
        kk[:, lo:hi] = (torch.randn((n - k, hi - lo, D), generator=g, device=device) * cfg.value_scale).to(dt)
        vv[:, lo:hi] = (torch.randn((n - k, hi - lo, D), generator=g, device=device) * cfg.value_scale).to(dt)
        be.init_request(f"r{i}", [{"key": kk, "value": vv}])  # one layer: a step is one layer
        del kk, vv
    hg = torch.Generator().manual_seed(5)
    ids = [f"r{i}" for i in range(B)]
    single = all(k == 1 for k in n_new)
    if single:
        items = [{"request_id": rid, "layer_idx": 0,
                  "query": torch.randn((cfg.num_q_heads, D), generator=hg).pin_memory(),
                  "key": torch.randn((cfg.num_kv_heads, D), generator=hg).to(dt).pin_memory(),
                  "value": torch.randn((cfg.num_kv_heads, D), generator=hg).to(dt).pin_memory(),
                  "score_scale": cfg.score_scale} for rid in ids]
        call = lambda: be.decode_layer_batch(items)  # noqa: E731
    else:
        qh = torch.randn((T, cfg.num_q_heads, D), generator=hg).pin_memory()
        kh = torch.randn((T, cfg.num_kv_heads, D), generator=hg).to(dt).pin_memory()
        vh = torch.randn((T, cfg.num_kv_heads, D), generator=hg).to(dt).pin_memory()
        # Every rank holds the whole gathered output; the job reads it back
        # once, each rank its own share of the rows.
        r0, r1 = T * rank // world, T * (rank + 1) // world

        def call():
            # the output back into pinned host memory, then one stream sync
            out = be.decode_batch(ids, 0, qh, kh, vh, cfg.score_scale, n_new=n_new)
            host = out[r0:r1].to("cpu", non_blocking=True)
            torch.cuda.current_stream(device).synchronize()
            return host
    esz = torch.empty((), dtype=dt).element_size()
    if single:
        h2d = T * cfg.num_q_heads * D * 4 + 2 * T * cfg.num_kv_heads * D * esz
        d2h = T * cfg.num_q_heads * D * 4
    else:
        # per rank: its heads of the inputs (decode_batch copies no others)
        # and its share of the output rows
        h2d = (T * cfg.num_q_heads * D * 4 + 2 * T * cfg.num_kv_heads * D * esz) * (hi - lo) \
            // cfg.num_kv_heads
        d2h = (r1 - r0) * cfg.num_q_heads * D * 4
    for _ in range(args.warmup):
        call()
    torch.cuda.synchronize(device)
    _barrier(world)
    lens_before = [be.get_context_len(rid) for rid in ids]
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        call()
    e1.record()
    torch.cuda.synchronize(device)
    ms = _max_over_ranks(e0.elapsed_time(e1) / args.steps, world)
    # bytes actually attended over (contexts grow by n_new tokens per step)
    attended = sum(kv_bytes([n + (s + 1) * k for n, k in zip(lens_before, n_new)],
                            cfg.num_kv_heads, D, dt) for s in range(args.steps)) / args.steps
    for rid in ids:
        be.free_request(rid)
    be.close()
    del be
    torch.cuda.empty_cache()
    return {"value": round(attended / (ms * 1e-3) / 1e9, 2), "unit": "GB/s",
            "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h, "ms_per_step": round(ms, 5),
            "bytes": "per rank" + ("" if single or world == 1 else
                                   "; each rank copies its heads' inputs and reads 1/N of the "
                                   "gathered output rows"),
            "api": ("B200AttentionBackend.decode_layer_batch (per-item host tensors)" if single
                    else "B200AttentionBackend.decode_batch (host tensors, multi-token)"),
            "gather": "none" if world == 1 else args.gather}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="c3")
    ap.add_argument("--batch", type=int, default=0)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-graph", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--kv-dtype", default="config", choices=["config", "fp8"],
                    help="KV cache dtype: the configuration's, or fp8 (e4m3) on the same workload")
    ap.add_argument("--gather", default="peer", choices=["peer", "nccl"],
                    help="N>1 output all-gather: fused NVLink peer stores or NCCL")
    ap.add_argument("--partition-tokens", type=int, default=None,
                    help="split-K partition length (default: the library's choice; -1 balanced)")
    ap.add_argument("--replays", type=int, default=30,
                    help="individually timed graph replays behind spread and the roofline time")
    ap.add_argument("--profile-share", type=int, default=0,
                    help="ncu case: one rank's share of a W-way shard on one GPU (no JSON)")
    ap.add_argument("--profile-rank", type=int, default=0)
    ap.add_argument("--launches", type=int, default=6)
    ap.add_argument("--time-share", action="store_true",
                    help="with --profile-share: also time the launches chained in one graph")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)
    if args.profile_share:
        run_profile_share(args)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_b200(args)


if __name__ == "__main__":
    main()
