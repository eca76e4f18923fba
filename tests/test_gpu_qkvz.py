"""GPU parity: fused_qkvzba_split_reshape_cat (the de-interleave of the GDN
input projections).  The op is a permutation, so every check is bit-exact."""

import pytest
import torch

import oracle
import torch_npu_ops_b200 as ops
from parity import golden

pytestmark = pytest.mark.gpu
DEV = "cuda"
NAMES = ("mixed_qkv", "z", "b", "a")


@pytest.mark.parametrize("case", golden("fused_qkvzba_split_reshape_cat"), ids=lambda c: c["name"])
def test_qkvzba_golden(case):
    a = case["args"]
    outs = ops.npu_fused_qkvzba_split_reshape_cat(a["mixed_qkvz"].to(DEV), a["mixed_ba"].to(DEV),
                                                  a["num_heads_qk"], a["num_heads_v"],
                                                  a["head_qk"], a["head_v"])
    for got, name in zip(outs, NAMES):
        assert torch.equal(got.cpu(), case["out"][name]), name


# the reference test's (batch, nqk, nv) list with head_qk = head_v = 128
# (test_fused_qkvzba_split_reshape.py:518-555)
REF = [(1, 8, 16), (4, 8, 16), (8, 8, 16), (1, 16, 16), (1, 16, 32), (1, 16, 48), (1, 16, 64),
       (4, 16, 32), (8, 16, 32), (64, 16, 16), (64, 8, 8), (64, 4, 4), (64, 2, 2), (64, 16, 32),
       (64, 8, 16), (64, 4, 8), (64, 2, 4), (64, 16, 48), (64, 8, 24), (64, 4, 12), (64, 2, 6),
       (64, 16, 64), (64, 8, 32), (64, 4, 16), (64, 2, 8), (4096, 2, 4), (4096, 16, 16),
       (4096, 4, 8), (4096, 8, 16), (4096, 16, 32), (4096, 16, 48), (4096, 16, 64)]


def _check(rows, nqk, nv, hqk, hv, dt=torch.bfloat16, dba=torch.bfloat16, seed=0):
    r = nv // nqk
    g = torch.Generator().manual_seed(seed + rows + 7 * nqk + nv)
    qkvz = torch.randn(rows, nqk * (2 * hqk + 2 * r * hv), generator=g).to(dt)
    ba = torch.randn(rows, nqk * 2 * r, generator=g).to(dba)
    outs = ops.npu_fused_qkvzba_split_reshape_cat(qkvz.to(DEV), ba.to(DEV), nqk, nv, hqk, hv)
    refs = oracle.fused_qkvzba_split_reshape_cat(qkvz, ba, nqk, nv, hqk, hv)
    for got, ref, name in zip(outs, refs, NAMES):
        assert got.shape == ref.shape and got.dtype == ref.dtype, name
        assert torch.equal(got.cpu(), ref), name


@pytest.mark.parametrize("rows,nqk,nv", REF)
def test_qkvzba_reference_shapes(rows, nqk, nv):
    _check(rows, nqk, nv, 128, 128)


@pytest.mark.parametrize("rows,nqk,nv,hqk,hv,dt,dba", [
    (33, 4, 12, 36, 20, torch.bfloat16, torch.bfloat16),   # 8-byte vectors
    (17, 2, 6, 6, 10, torch.float16, torch.float32),       # element-wise path
    (9, 3, 9, 64, 32, torch.float32, torch.float16),       # fp32 projections
    (0, 2, 4, 128, 128, torch.bfloat16, torch.bfloat16),   # no rows
])
def test_qkvzba_odd_shapes(rows, nqk, nv, hqk, hv, dt, dba):
    _check(rows, nqk, nv, hqk, hv, dt, dba)


def test_qkvzba_ratio_check_and_cpp():
    from torch_npu_ops_b200 import _C as C
    x = torch.randn(2, 2 * (256 + 10 * 128), dtype=torch.bfloat16, device=DEV)
    ba = torch.randn(2, 2 * 10, dtype=torch.bfloat16, device=DEV)
    with pytest.raises(RuntimeError, match="v_heads_per_qk in"):
        ops.npu_fused_qkvzba_split_reshape_cat(x, ba, 2, 10, 128, 128)
    qkvz = torch.randn(5, 4 * (256 + 512), dtype=torch.bfloat16, device=DEV)
    ba = torch.randn(5, 4 * 4, dtype=torch.bfloat16, device=DEV)
    o1 = C.npu_fused_qkvzba_split_reshape_cat(qkvz, ba, 4, 8, 128, 128)
    o2 = ops.npu_fused_qkvzba_split_reshape_cat(qkvz, ba, 4, 8, 128, 128)
    assert all(torch.equal(p, q) for p, q in zip(o1, o2))
    assert C.kernel_entry_point("fused_qkvzba_split_reshape_cat_gqa_r3_kernel") == \
        "xops_fused_qkvzba_split_reshape_cat"
