"""Shared test configuration.

Markers: ``gpu`` — needs a CUDA device (B200); everything else runs on CPU.

Tolerance used by every attention parity check (fp16/bf16 KV vs the fp32
oracle, fp32 queries so neither side rounds the output):
    max |err|                        <= 2e-3   (absolute)
    max |err| / max(|ref|, 1e-3)     <= 1e-2   (elementwise relative, floored)
When the query (and so the output) is 16-bit, the output's own rounding,
half an ulp (|ref| * 2^-8 for bf16, 2^-11 for fp16), is added to both bounds.
fp32 KV caches are held to 1e-4 absolute.
"""

from __future__ import annotations

import os
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)
GOLDEN = os.path.join(ROOT, "tests", "golden")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")


def load_golden(name: str):
    return torch.load(os.path.join(GOLDEN, name), weights_only=False)


def has_gpu() -> bool:
    return torch.cuda.is_available()


def attn_errors(out: torch.Tensor, ref: torch.Tensor):
    out = out.detach().float().cpu()
    ref = ref.detach().float().cpu()
    err = (out - ref).abs()
    rel = err / ref.abs().clamp_min(1e-3)
    return float(err.max()) if err.numel() else 0.0, float(rel.max()) if rel.numel() else 0.0


def assert_attn_close(out: torch.Tensor, ref: torch.Tensor, *, kv_dtype=torch.bfloat16,
                      out_dtype=torch.float32, what: str = "") -> None:
    out_f = out.detach().float().cpu()
    ref_f = ref.detach().float().cpu()
    assert out_f.shape == ref_f.shape, f"{what}: shape {tuple(out_f.shape)} vs {tuple(ref_f.shape)}"
    assert torch.isfinite(out_f).all(), f"{what}: non-finite output"
    err = (out_f - ref_f).abs()
    if kv_dtype == torch.float32 and out_dtype == torch.float32:
        assert float(err.max()) <= 1e-4, f"{what}: max abs err {float(err.max()):.3g} > 1e-4"
        return
    ulp = {torch.bfloat16: 2.0 ** -8, torch.float16: 2.0 ** -11}.get(out_dtype, 0.0)
    abs_bound = 2e-3 + ref_f.abs() * ulp
    rel_bound = 1e-2 + ulp * ref_f.abs() / ref_f.abs().clamp_min(1e-3)
    rel = err / ref_f.abs().clamp_min(1e-3)
    bad_abs = err > abs_bound
    bad_rel = rel > rel_bound
    assert not bad_abs.any(), (f"{what}: max abs err {float(err.max()):.3g} "
                               f"(bound 2e-3 + out-dtype rounding)")
    assert not bad_rel.any(), (f"{what}: max floored rel err {float(rel.max()):.3g} "
                               f"(bound 1e-2 + out-dtype rounding)")


gpu = pytest.mark.gpu
