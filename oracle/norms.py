"""Norm oracles (test infrastructure only; see ``oracle/__init__.py``)."""

import torch

from . import _out


def layer_norm_fwd(x, weight, bias=None, eps=1e-6, z=None, group_size=None,
                   norm_before_gate=True, is_rms_norm=False):
    """Grouped LayerNorm / RMSNorm with an optional SiLU gate ``z``.

    Follows the golden reference ``_golden_ref``
    (triton_npu/triton_src/test_layernorm_fwd.py:1529-1564) and the
    statistics layout of ``layer_norm_fwd_kernel``
    (triton_npu/triton_src/test_layernorm_fwd.py:1125-1187): for every row
    and every group of ``group_size`` columns,

        x'   = x * silu(z)               (only when z is given and the gate
                                           comes before the norm)
        mean = sum(x') / G               (LayerNorm only)
        rstd = 1 / sqrt(var(x') + eps)   (var about 0 for RMSNorm)
        y    = x_hat * w [+ b]           (w, b indexed by the full column)
        y   *= silu(z)                   (when the gate comes after the norm)

    ``mean`` and ``rstd`` are fp32 vectors of length ngroups*M stored at
    ``group * M + row`` (test_layernorm_fwd.py:1163-1165).
    Returns ``(y, mean, rstd)``; ``y`` has x's dtype, ``mean`` is None for
    RMSNorm.
    """
    shape = x.shape
    n = shape[-1]
    x2 = x.reshape(-1, n).to(torch.float32)
    m = x2.shape[0]
    if group_size is None or group_size < 0:
        group_size = n
    ng = n // group_size
    z2 = z.reshape(-1, n).to(torch.float32) if z is not None else None
    if z2 is not None and not norm_before_gate:
        x2 = x2 * (z2 * torch.sigmoid(z2))
    xg = x2.reshape(m, ng, group_size)
    if is_rms_norm:
        mean = None
        var = (xg * xg).mean(dim=-1, keepdim=True)
        xhat = xg * torch.rsqrt(var + eps)
    else:
        mu = xg.mean(dim=-1, keepdim=True)
        xc = xg - mu
        var = (xc * xc).mean(dim=-1, keepdim=True)
        xhat = xc * torch.rsqrt(var + eps)
        mean = mu.reshape(m, ng).t().contiguous().reshape(-1)
    rstd = torch.rsqrt(var + eps).reshape(m, ng).t().contiguous().reshape(-1)
    y = xhat.reshape(m, n) * weight.to(torch.float32)
    if bias is not None:
        y = y + bias.to(torch.float32)
    if z2 is not None and norm_before_gate:
        y = y * (z2 * torch.sigmoid(z2))
    return _out.out(y, x.dtype).reshape(shape), mean, rstd


def gemma_rms_norm(x, gamma, eps=1e-6):
    """Gemma RMSNorm: ``y = x * rsqrt(mean(x^2) + eps) * (1 + gamma)``.

    Parity unpinned: the reference calls the closed CANN operator
    ``aclnnGemmaRmsNorm`` (ascendc_npu/gemma_rms_norm.cpp:54) and its only test
    checks shapes (npu_python_extension/test_npu_examples.py:25-55).  This is
    the public Gemma definition, computed in fp32.  The normalised axes are
    the trailing ``gamma.dim()`` axes; ``rstd`` is fp32 with shape
    ``x.shape[:-gamma.dim()] + (1,) * gamma.dim()``
    (ascendc_npu/gemma_rms_norm.cpp:35-49).  Returns ``(rstd, y)`` in the
    order of the pybind schema (npu_python_extension/op_register.cpp:28-35).
    """
    gd = gamma.dim()
    lead = x.shape[: x.dim() - gd]
    n = gamma.numel()
    xf = x.reshape(-1, n).to(torch.float32)
    rstd = torch.rsqrt((xf * xf).mean(dim=-1, keepdim=True) + eps)
    y = xf * rstd * (1.0 + gamma.reshape(-1).to(torch.float32))
    rstd_shape = tuple(lead) + (1,) * gd if x.dim() > gd else (1,) * x.dim()
    return rstd.reshape(rstd_shape), _out.out(y, x.dtype).reshape(x.shape)


def l2norm_last_dim(x, eps=1e-6):
    """``x * rsqrt(sum(x^2) + eps)`` over the last axis, computed in fp32 and
    cast back (``l2norm_ref``, triton_npu/triton_src/test_l2norm.py:95-98)."""
    xf = x.to(torch.float32)
    return _out.out(xf * torch.rsqrt((xf * xf).sum(dim=-1, keepdim=True) + eps), x.dtype)
