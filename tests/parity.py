"""Tolerances and comparison helpers for the GPU parity tests.

The bars are the project's stated parity targets against the CPU oracle:

* fp32 outputs within 1e-4 relative, element by element:
  ``|a - b| <= 1e-4 * |b| + floor``.  The floor is 1e-6 times the largest
  magnitude of the operands (by default the largest ``|b|``), about eight
  fp32 ulps of that magnitude: the level at which two fp32 evaluations that
  only sum in a different order already differ.  Without it an output that
  comes out of a cancellation (a rotated coordinate near zero, a row mean
  near zero) would demand bit equality.
* bf16 outputs within 2e-2 max-abs.  The bar is absolute wherever half a
  bf16 ulp is below it, i.e. for ``|ref| < 8``.  From 8 up a correctly
  rounded bf16 value can already sit half an ulp (1/32 at 8..16) from the
  fp32 reference, so there the bound is that half ulp plus a quarter of the
  bar (5e-3) for the kernel's own fp32 error.
* fp32 recurrent / final states within 1e-3 relative (Frobenius norm).

``assert_bf16_rel`` adds, for outputs whose scale is small next to 2e-2 (the
gated delta rule's o is ~1e-3 to 1e-1), a relative Frobenius bound of 1e-2,
about ten times the rounding of a bf16 output, so that the check still says
something about such outputs.

Every failure message gives the measured max-abs and max-relative errors.
"""

import os

import torch

FP32_REL = 1e-4
FP32_FLOOR = 1e-6
BF16_MAXABS = 2e-2
STATE_REL = 1e-3
OUT_REL = 1e-2

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def golden(name):
    return torch.load(os.path.join(GOLD, name + ".pt"), weights_only=False)["cases"]


def _cpu(a, b):
    return a.detach().float().cpu(), b.detach().float().cpu()


def maxabs(a, b):
    return (a.detach().float().cpu() - b.detach().float().cpu()).abs().max().item() if a.numel() else 0.0


def rel_fro(a, b):
    a, b = _cpu(a, b)
    d = (a - b).norm().item()
    n = b.norm().item()
    return d / n if n > 0 else d


def _errors(a, b):
    err = (a - b).abs()
    rel = err / b.abs().clamp(min=torch.finfo(torch.float32).tiny)
    return err.max().item(), rel.max().item()


def assert_fp32(a, b, tol=FP32_REL, scale=None):
    """Element-wise ``|a - b| <= tol * |b| + 1e-6 * scale``, where ``scale``
    is the operands' largest magnitude (default: ``max |b|``)."""
    a, b = _cpu(a, b)
    assert a.shape == b.shape, f"shape {tuple(a.shape)} != {tuple(b.shape)}"
    if not b.numel():
        return
    s = b.abs().max().item() if scale is None else float(scale)
    err = (a - b).abs()
    bound = tol * b.abs() + FP32_FLOOR * s
    worst = (err - bound).max().item()
    if worst > 0:
        e_abs, e_rel = _errors(a, b)
        idx = int((err - bound).argmax())
        raise AssertionError(
            f"fp32 mismatch: max-abs {e_abs:.3e}, max-rel {e_rel:.3e} (tol {tol} relative + "
            f"floor {FP32_FLOOR * s:.2e}); worst element {idx}: got {a.reshape(-1)[idx].item():.7g}, "
            f"ref {b.reshape(-1)[idx].item():.7g}")


def bf16_bound(b, tol=BF16_MAXABS):
    """Per-element bound for a bf16 output against an fp32 reference ``b``."""
    mag = b.abs()
    # half an ulp of bf16 at |b|: 2^(floor(log2|b|) - 8)
    half_ulp = torch.exp2(torch.floor(torch.log2(mag.clamp(min=1e-30))) - 8)
    return torch.where(mag < 8, torch.full_like(mag, tol), half_ulp + tol / 4)


def assert_bf16(a, b, tol=BF16_MAXABS):
    """bf16 outputs: ``|a - b| <= tol`` for ``|b| < 8``; above that, half a
    bf16 ulp of ``|b|`` plus ``tol / 4`` (see the module docstring)."""
    a, b = _cpu(a, b)
    assert a.shape == b.shape, f"shape {tuple(a.shape)} != {tuple(b.shape)}"
    if not a.numel():
        return
    err = (a - b).abs()
    bound = bf16_bound(b, tol)
    worst = (err - bound).max().item()
    if worst > 0 or torch.isnan(a).any():
        e_abs, e_rel = _errors(a, b)
        idx = int((err - bound).nan_to_num(float("inf")).argmax())
        raise AssertionError(
            f"bf16 mismatch: max-abs {e_abs:.4e} (bar {tol} for |ref| < 8), max-rel {e_rel:.3e}; "
            f"worst element {idx}: got {a.reshape(-1)[idx].item():.6g}, "
            f"ref {b.reshape(-1)[idx].item():.6g}")


def assert_state(a, b, tol=STATE_REL):
    r = rel_fro(a, b)
    if not r <= tol:
        x, y = _cpu(a, b)
        raise AssertionError(f"state relative (Frobenius) error {r:.3e} > {tol}; "
                             f"max-abs {maxabs(x, y):.3e}")


def assert_bf16_rel(a, b, tol=BF16_MAXABS, rel=OUT_REL):
    """``assert_bf16`` plus a relative Frobenius bound (see the module docstring)."""
    assert_bf16(a, b, tol)
    r = rel_fro(a, b)
    assert r <= rel, f"relative (Frobenius) error {r:.3e} > {rel}"
