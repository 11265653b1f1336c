"""The balanced split's decomposition, restated on the CPU.

paged_decode_stream.cu gives worker w the unit range [w*per, (w+1)*per) of
all (sequence, KV head x column chunk, block) units, and the host sizes the
split-K workspace for at most
    max_parts = min(ceil(workers / hc) + 1, ceil(max_ctx / block_size))
parts per segment (paged_decode.cu, make_plan).  A segment cut into more
parts than that would lose partials (the kernel flags it), so this checks the
bound over random batches, and that the ranges cover every unit exactly once.
"""

from __future__ import annotations

import math
import random


def _plan(ctx, hc, bs, workers, min_units=8):
    n = [(c + bs - 1) // bs if c > 0 else 0 for c in ctx]
    U = sum(n) * hc
    weff = max(1, min(workers, -(-U // min_units)))
    per = -(-U // weff) if U > 0 else 1
    return n, U, per


def _check(ctx, hc, bs, workers):
    n, U, per = _plan(ctx, hc, bs, workers)
    max_parts = min(-(-workers // hc) + 1, max(1, -(-max(ctx) // bs)))
    start = 0
    for nb in n:
        for _ in range(hc):
            if nb:
                first, last = start // per, (start + nb - 1) // per
                count = last - first + 1
                assert count <= max_parts, (count, max_parts, nb, per, hc)
                assert count <= nb
            start += nb
    assert start == U
    # worker ranges partition [0, U)
    covered = sum(max(0, min(U, (w + 1) * per) - w * per) for w in range(workers) if w * per < U)
    assert covered == U


def test_part_count_bound_holds_on_random_batches():
    rng = random.Random(0)
    for _ in range(400):
        B = rng.choice([1, 2, 8, 33, 256, 1024])
        hc = rng.choice([1, 2, 4, 8, 16])
        bs = rng.choice([16, 32])
        workers = rng.choice([148 * 6 * 2, 148 * 3 * 2, 148 * 2, 64])
        kind = rng.random()
        if kind < 0.3:
            ctx = [rng.randint(0, 70000)] * B
        elif kind < 0.6:
            ctx = [int(math.exp(rng.uniform(math.log(1), math.log(65536)))) for _ in range(B)]
        else:
            ctx = [rng.choice([0, 1, 15, 16, 17, 4097, 40000]) for _ in range(B)]
        if max(ctx) == 0:
            ctx[0] = 1
        _check(ctx, hc, bs, workers)


def test_single_long_sequence_split_over_every_worker():
    # one 40k-token sequence on one KV head: the worst case for parts per segment
    _check([40000], 1, 16, 148 * 6 * 2)
    _check([40000, 1, 0, 3], 1, 16, 148 * 6 * 2)
