"""Synthetic workloads and bench configuration helpers (no GPU)."""

from __future__ import annotations

import argparse
import math

import torch

from cloverinfer_b200 import _lib
from cloverinfer_b200.workloads import CONFIGS, context_lengths, kv_bytes, new_tokens


def test_config_shapes_follow_the_reference_configs():
    c3 = CONFIGS["c3"]
    assert (c3.num_q_heads, c3.num_kv_heads, c3.head_dim, c3.block_size, c3.batch) == (32, 8, 128, 16, 8)
    assert context_lengths(c3, 0) == [32768] * 8
    # 8 x 32768 x 8 KV heads x 128 x (K, V) x 2 bytes
    assert kv_bytes(context_lengths(c3, 0), 8, 128, torch.bfloat16) == 1073741824
    c2 = CONFIGS["c2"]
    lens = context_lengths(c2, 0)
    assert len(lens) == 32 and min(lens) >= 1024 and max(lens) <= 4096 and c2.group == 7
    c4 = CONFIGS["c4"]
    lens, nn = context_lengths(c4, 0), new_tokens(c4, 0)
    assert len(lens) == 256 and min(lens) >= 16 and max(lens) <= 16384
    assert set(nn) <= {1, 2, 3, 4} and c4.block_size == 32
    assert math.isclose(CONFIGS["c1"].score_scale, 1 / 8)


def test_seeded_inputs_are_reproducible():
    c5 = CONFIGS["c5"]
    assert context_lengths(c5, 3) == context_lengths(c5, 3)
    assert context_lengths(c5, 3) != context_lengths(c5, 4)


def test_fp8_kv_option_and_dtype_codes():
    import bench
    cfg = bench.config_for(argparse.Namespace(config="c3", kv_dtype="fp8"))
    assert cfg.dtype == torch.float8_e4m3fn and cfg.name.endswith("-fp8kv")
    assert bench.config_for(argparse.Namespace(config="c3", kv_dtype="config")).dtype == torch.bfloat16
    assert kv_bytes([10], 2, 128, torch.float8_e4m3fn) == 10 * 2 * 128 * 2
    assert _lib.dtype_code(torch.float8_e4m3fn) == _lib.FP8_E4M3 == 3
    assert (_lib.F32, _lib.F16, _lib.BF16) == (0, 1, 2)
