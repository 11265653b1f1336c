"""Run one rank's share of a configuration's decode step on one GPU.

    python -m cloverinfer_b200.profile_case --config c3 --world 8 --launches 6

Builds the step of rank ``--rank`` of a ``--world``-way KV-head-sharded run
(its KV heads, the library's partition choice for that share) and launches the
decode (+ split-K reduce) ``--launches`` times — the case an ncu capture of a
multi-GPU rank's kernel runs on a single GPU.
"""

from __future__ import annotations

import argparse

import torch

from .workloads import CONFIGS, build_decode_step, context_lengths, new_tokens


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--config", default="c3")
    ap.add_argument("--world", type=int, default=1)
    ap.add_argument("--rank", type=int, default=0)
    ap.add_argument("--launches", type=int, default=6)
    a = ap.parse_args()
    cfg = CONFIGS[a.config]
    dev = torch.device("cuda", 0)
    lens = context_lengths(cfg, 0)
    st = build_decode_step(cfg, a.rank, a.world, lens, dev, n_new=new_tokens(cfg, 0))
    for _ in range(a.launches):
        st["decode_only"]()
    torch.cuda.synchronize()
    st["pool"].check_status()
    print(f"{cfg.name}: rank {a.rank}/{a.world}, {st['hkv_local']} KV heads, "
          f"partition {st['partition_tokens']} tokens, {a.launches} launches ok")


if __name__ == "__main__":
    main()
