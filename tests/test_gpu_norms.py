"""GPU parity: layer_norm_fwd (LN / RMS / gated), gemma_rms_norm, l2norm."""

import pytest
import torch

import oracle
import torch_npu_ops_b200 as ops
from parity import assert_bf16, assert_fp32, golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _to(t):
    return None if t is None else t.to(DEV)


@pytest.mark.parametrize("case", golden("layer_norm_fwd"), ids=lambda c: c["name"])
def test_layer_norm_golden(case):
    a = case["args"]
    y = ops.layer_norm_fwd(_to(a["x"]), _to(a["weight"]), _to(a["bias"]), a["eps"], _to(a["z"]),
                           a["group_size"], a["norm_before_gate"], a["is_rms_norm"])
    ref, _, _ = oracle.layer_norm_fwd(a["x"], a["weight"], a["bias"], a["eps"], a["z"],
                                      a["group_size"], a["norm_before_gate"], a["is_rms_norm"])
    if a["x"].dtype == torch.float32:
        assert_fp32(y, ref)
        assert_fp32(y, case["out"]["y"])
    else:
        assert_bf16(y, ref)


CASES = [  # (M, N, group, rms, bias, z, before, xdtype, wdtype)
    (8192, 128, 128, True, False, True, True, torch.bfloat16, torch.bfloat16),  # gated RMSNorm cfg4
    (256, 2048, 2048, False, True, False, True, torch.bfloat16, torch.bfloat16),  # LayerNorm cfg4
    (1024, 128, 128, True, False, True, True, torch.bfloat16, torch.float32),
    (300, 512, 128, False, True, True, False, torch.float32, torch.float32),
    (37, 4096, 4096, True, True, False, True, torch.bfloat16, torch.float32),
    (5, 8192, 8192, False, False, True, False, torch.float32, torch.float32),
    (64, 96, 96, True, False, False, True, torch.float32, torch.float32),
    # streaming (bulk-copy) path: 16-bit, contiguous rows, >= 8192 segments
    (2048, 512, 64, False, True, True, False, torch.bfloat16, torch.bfloat16),  # LN, gate first
    (4100, 512, 128, True, True, True, True, torch.bfloat16, torch.float32),     # partial tile
    (1000, 2048, 256, True, False, True, True, torch.float16, torch.float16),
    (3000, 768, 256, False, False, False, True, torch.bfloat16, torch.bfloat16),  # LN, no gate
    # wide streaming path: one warp per segment, >= 4 MB of x
    (1100, 2048, 2048, False, True, False, True, torch.bfloat16, torch.bfloat16),  # LN cfg4 row
    (600, 4096, 1024, True, False, True, False, torch.bfloat16, torch.float32),    # gate first
    (520, 8192, 8192, False, True, True, True, torch.float16, torch.float16),      # 1 seg / tile
    (4200, 1024, 512, True, True, False, True, torch.bfloat16, torch.bfloat16),    # 4 / warp
    (130, 16384, 16384, False, False, False, True, torch.bfloat16, torch.bfloat16),
    (4099, 1040, 520, False, True, False, True, torch.bfloat16, torch.bfloat16),   # odd tiles
    # few wide segments (< 4 MB): one CTA per segment
    (40, 512, 512, False, True, True, False, torch.bfloat16, torch.bfloat16),      # 64 threads
    (100, 2048, 1024, True, False, True, True, torch.float16, torch.float16),      # 2 groups
    (8, 8192, 8192, False, True, False, True, torch.bfloat16, torch.float32),      # 4 vectors
]


@pytest.mark.parametrize("M,N,G,rms,bias,z,before,xdt,wdt", CASES)
def test_layer_norm_vs_oracle(M, N, G, rms, bias, z, before, xdt, wdt):
    g = torch.Generator().manual_seed(M * 7 + N)
    x = torch.randn(M, N, generator=g).to(xdt)
    w = (1 + 0.1 * torch.randn(N, generator=g)).to(wdt)
    b = (0.1 * torch.randn(N, generator=g)).to(wdt) if bias else None
    zz = torch.randn(M, N, generator=g).to(xdt) if z else None
    y, mean, rstd = ops.layer_norm_fwd_with_stats(_to(x), _to(w), _to(b), 1e-6, _to(zz), G,
                                                  before, rms)
    ry, rmean, rrstd = oracle.layer_norm_fwd(x, w, b, 1e-6, zz, G, before, rms)
    (assert_fp32 if xdt == torch.float32 else assert_bf16)(y, ry)
    assert_fp32(rstd, rrstd)
    if not rms:
        # a row mean comes out of a cancellation: its floor is set by the
        # magnitude of the summed elements, not by the mean itself
        assert_fp32(mean, rmean, scale=x.float().abs().max().item())


def test_layer_norm_strided_rows():
    x = torch.randn(64, 256, dtype=torch.bfloat16)
    full = torch.randn(64, 512, dtype=torch.bfloat16)
    full[:, :256] = x
    w = torch.randn(256, dtype=torch.bfloat16)
    y = ops.layer_norm_fwd(full.to(DEV)[:, :256], w.to(DEV), None, 1e-6, None, 128, True, True)
    assert_bf16(y, oracle.layer_norm_fwd(x, w, None, 1e-6, None, 128, True, True)[0])


@pytest.mark.parametrize("shape,dt", [((256, 2048), torch.bfloat16), ((4, 128, 4096), torch.float16),
                                      ((4, 128, 4096), torch.float32), ((3, 100), torch.bfloat16),
                                      ((2048, 2048), torch.bfloat16),   # wide streaming path
                                      ((1100, 4000), torch.float16),
                                      ((9000, 128), torch.bfloat16),    # narrow streaming path
                                      ((300, 1024), torch.bfloat16)])   # CTA per row
def test_gemma_rms_norm(shape, dt):
    g = torch.Generator().manual_seed(1234)
    x = torch.randn(*shape, generator=g).to(dt)
    gamma = (0.1 * torch.randn(shape[-1], generator=g)).to(dt)
    rstd, y = ops.npu_gemma_rms_norm(x.to(DEV), gamma.to(DEV), 1e-6)
    rr, ry = oracle.gemma_rms_norm(x, gamma, 1e-6)
    assert rstd.shape == rr.shape and y.shape == x.shape
    assert_fp32(rstd, rr)
    (assert_fp32 if dt == torch.float32 else assert_bf16)(y, ry)
    rstd2, y2 = ops.npu_python_extension_lib.gemma_rms_norm(x.to(DEV), gamma.to(DEV), 1e-6)
    assert torch.equal(y2, y)


@pytest.mark.parametrize("xshape,gshape", [((4, 8, 16, 128), (16, 128)), ((6, 32, 64), (32, 64)),
                                           ((32, 64), (32, 64)), ((3, 2, 4, 256), (2, 4, 256))])
def test_gemma_rms_norm_multidim_gamma(xshape, gshape):
    """gamma over the trailing gamma.dim() axes: rstd has shape
    x.shape[:-gamma.dim()] + (1,) * gamma.dim() (ascendc_npu/gemma_rms_norm.cpp:35-49)."""
    g = torch.Generator().manual_seed(77)
    x = torch.randn(*xshape, generator=g).to(torch.bfloat16)
    gamma = (0.1 * torch.randn(*gshape, generator=g)).to(torch.bfloat16)
    rstd, y = ops.npu_gemma_rms_norm(x.to(DEV), gamma.to(DEV), 1e-6)
    rr, ry = oracle.gemma_rms_norm(x, gamma, 1e-6)
    lead = xshape[: len(xshape) - len(gshape)]
    expect = tuple(lead) + (1,) * len(gshape) if len(xshape) > len(gshape) else (1,) * len(xshape)
    assert tuple(rstd.shape) == tuple(rr.shape) == expect and y.shape == x.shape
    assert_fp32(rstd, rr)
    assert_bf16(y, ry)
    rstd2, y2 = ops.npu_python_extension_lib.gemma_rms_norm(x.to(DEV), gamma.to(DEV), 1e-6)
    assert tuple(rstd2.shape) == expect and torch.equal(y2, y)


@pytest.mark.parametrize("case", golden("l2norm"), ids=lambda c: c["name"])
def test_l2norm_golden(case):
    x = case["args"]["x"]
    y = ops.npu_l2norm_last_dim(x.to(DEV), case["args"]["eps"])
    ref = oracle.l2norm_last_dim(x, case["args"]["eps"])
    (assert_fp32 if x.dtype == torch.float32 else assert_bf16)(y, ref)


@pytest.mark.parametrize("shape", [(20000, 128), (9000, 64), (9000, 256), (3000, 1024), (700, 4104),
                                   (50, 2048)])
def test_l2norm_streaming(shape):
    """bf16 rows on the bulk-copy streaming paths (narrow and wide) and, below
    4 MB, the CTA-per-row path."""
    from torch_npu_ops_b200 import _lib
    g = torch.Generator().manual_seed(shape[0] + shape[1])
    x = (3 * torch.randn(*shape, generator=g)).to(torch.bfloat16)
    y = ops.npu_l2norm_last_dim(x.to(DEV), 1e-6)
    assert_bf16(y, oracle.l2norm_last_dim(x, 1e-6))
    assert _lib.load().xops_device_error_count() == 0
