"""GPU parity: fused_gdn_gating and fused_sigmoid_gating_delta_rule_update
(the gates computed from the projections inside the recurrent step), through
the Python host API, the C++ torch API and the golden fixtures."""

import pytest
import torch

import oracle
import torch_npu_ops_b200 as ops
from parity import assert_bf16, assert_fp32, assert_state, golden

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _to(t):
    return None if t is None else t.to(DEV)


@pytest.mark.parametrize("case", golden("fused_gdn_gating"), ids=lambda c: c["name"])
def test_gdn_gating_golden(case):
    a = case["args"]
    g, beta = ops.npu_fused_gdn_gating(_to(a["A_log"]), _to(a["a"]), _to(a["b"]),
                                       _to(a["dt_bias"]), a["beta"], a["threshold"])
    assert g.shape == case["out"]["g"].shape and g.dtype == torch.float32
    assert beta.shape == case["out"]["beta"].shape and beta.dtype == a["b"].dtype
    assert_fp32(g, case["out"]["g"])
    # sigmoid rounded to b's dtype: at most one ulp apart
    assert_bf16(beta, case["out"]["beta"], tol=8e-3)


@pytest.mark.parametrize("rows,heads,dt,off", [
    (1, 64, torch.bfloat16, 0), (65536, 32, torch.bfloat16, 0),   # decode row, cfg5 prefill
    (333, 7, torch.float16, 0), (129, 6, torch.float32, 0),
    (100, 5, torch.bfloat16, 1),                                  # unaligned views: scalar path
])
def test_gdn_gating_shapes(rows, heads, dt, off):
    g0 = torch.Generator().manual_seed(rows + heads)
    A_log = torch.rand(heads, generator=g0) * 2.7
    dt_bias = torch.rand(heads, generator=g0)
    a = (8 * torch.randn(rows * heads + off, generator=g0)).to(dt)[off:].view(rows, heads)
    b = torch.randn(rows * heads + off, generator=g0).to(dt)[off:].view(rows, heads)
    ad, bd = a.to(DEV), b.to(DEV)
    if off:  # keep the odd offset on the device too
        ad = torch.empty(rows * heads + off, dtype=dt, device=DEV)[off:].view(rows, heads)
        bd = torch.empty(rows * heads + off, dtype=dt, device=DEV)[off:].view(rows, heads)
        ad.copy_(a)
        bd.copy_(b)
    g, beta = ops.npu_fused_gdn_gating(_to(A_log), ad, bd, _to(dt_bias))
    rg, rb = oracle.fused_gdn_gating(A_log, a, b, dt_bias)
    assert_fp32(g, rg)
    if dt == torch.float32:
        assert_fp32(beta, rb)
    else:
        assert_bf16(beta, rb, tol=8e-3)


@pytest.mark.parametrize("case", golden("fused_sigmoid_gating_delta_rule_update"),
                         ids=lambda c: c["name"])
def test_sigmoid_gating_golden(case):
    a = case["args"]
    st = a["initial_state_source"].clone().to(DEV)
    o = ops.npu_fused_sigmoid_gating_delta_rule_update(
        _to(a["A_log"]), _to(a["a"]), _to(a["dt_bias"]), _to(a["q"]), _to(a["k"]), _to(a["v"]),
        _to(a["b"]), st, _to(a["initial_state_indices"]), _to(a["cu_seqlens"]), a["scale"],
        a["use_qk_l2norm_in_kernel"])
    # the reference test's own bounds against its torch path
    # (test_fused_sigmoid_gating_delta_rule_update.py:299-304)
    torch.testing.assert_close(o.cpu().float(), case["out"]["o"].float(), rtol=5e-3, atol=1e-2)
    torch.testing.assert_close(st.cpu(), case["out"]["state"], rtol=5e-2, atol=2e-2)
    # and this build's bounds against the fp32 oracle
    st_ref = a["initial_state_source"].clone()
    ro = oracle.fused_sigmoid_gating_delta_rule_update(
        a["A_log"], a["a"], a["dt_bias"], a["q"], a["k"], a["v"], a["b"], st_ref,
        a["initial_state_indices"], a["cu_seqlens"], a["scale"], a["use_qk_l2norm_in_kernel"])
    assert_bf16(o, ro)
    assert_state(st, st_ref)


# the reference test's (batch, H, HV) list, K = V = 128, one token per row
# (test_fused_sigmoid_gating_delta_rule_update.py:225-251)
REF_SHAPES = [(1, 8, 16), (2, 8, 16), (4, 8, 16), (8, 8, 16), (4, 16, 16), (4, 8, 8), (4, 4, 4),
              (4, 2, 2), (4, 16, 32), (4, 4, 8), (4, 2, 4), (4, 16, 48), (4, 8, 24), (4, 4, 12),
              (4, 2, 6), (4, 16, 64), (4, 8, 32), (4, 4, 16), (4, 2, 8), (4, 1, 8)]


def _inputs(batch, T, H, HV, K, seed, a_dtype=torch.bfloat16):
    g = torch.Generator().manual_seed(seed)
    return dict(
        q=torch.randn(batch, T, H, K, generator=g).to(torch.bfloat16),
        k=torch.randn(batch, T, H, K, generator=g).to(torch.bfloat16),
        v=torch.randn(batch, T, HV, K, generator=g).to(torch.bfloat16),
        a=torch.randn(batch, T, HV, generator=g).to(a_dtype),
        b=torch.randn(batch, T, HV, generator=g).to(a_dtype),
        A_log=torch.randn(HV, generator=g), dt_bias=torch.randn(HV, generator=g),
        h0=torch.randn(batch, HV, K, K, generator=g))


@pytest.mark.parametrize("batch,H,HV", REF_SHAPES)
def test_sigmoid_gating_reference_shapes(batch, H, HV):
    d = _inputs(batch, 1, H, HV, 128, 47 + batch + H + HV)
    idx = torch.arange(batch, dtype=torch.int32)
    cu = torch.arange(batch + 1, dtype=torch.int32)
    st = d["h0"].clone().to(DEV)
    o = ops.npu_fused_sigmoid_gating_delta_rule_update(
        _to(d["A_log"]), _to(d["a"]), _to(d["dt_bias"]), _to(d["q"]), _to(d["k"]), _to(d["v"]),
        _to(d["b"]), st, _to(idx), _to(cu), None, True)
    st_ref = d["h0"].clone()
    ro = oracle.fused_sigmoid_gating_delta_rule_update(
        d["A_log"], d["a"], d["dt_bias"], d["q"], d["k"], d["v"], d["b"], st_ref, idx, cu, None,
        True)
    assert o.shape == (batch, 1, HV, 128)
    assert_bf16(o, ro)
    assert_state(st, st_ref)


@pytest.mark.parametrize("a_dtype", [torch.bfloat16, torch.float32])
def test_sigmoid_gating_varlen_slots(a_dtype):
    """Varlen multi-token rows, a permuted slot table with a negative entry
    (zero start, no write-back), an empty sequence, spare slots untouched,
    K = V = 64, no in-kernel L2 norm and a custom softplus."""
    lens = [3, 0, 5, 1]
    N, H, HV, K = len(lens), 2, 6, 64
    T = sum(lens)
    d = _inputs(1, T, H, HV, K, 99, a_dtype)
    h0 = torch.randn(6, HV, K, K, generator=torch.Generator().manual_seed(3))
    idx = torch.tensor([4, 1, -1, 0], dtype=torch.int32)
    cu = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    st = h0.clone().to(DEV)
    o = ops.npu_fused_sigmoid_gating_delta_rule_update(
        _to(d["A_log"]), _to(d["a"]), _to(d["dt_bias"]), _to(d["q"]), _to(d["k"]), _to(d["v"]),
        _to(d["b"]), st, _to(idx), _to(cu), 0.2, False, 2.0, 5.0)
    st_ref = h0.clone()
    ro = oracle.fused_sigmoid_gating_delta_rule_update(
        d["A_log"], d["a"], d["dt_bias"], d["q"], d["k"], d["v"], d["b"], st_ref, idx, cu, 0.2,
        False, 2.0, 5.0)
    assert_bf16(o, ro)
    assert_state(st, st_ref)
    for s in (2, 3, 5):  # the negative row's and the unused slots
        assert torch.equal(st[s].cpu(), h0[s])


def test_gating_via_cpp_api():
    from torch_npu_ops_b200 import _C as C
    d = _inputs(4, 1, 2, 8, 128, 5)
    a2, b2 = _to(d["a"][:, 0]).contiguous(), _to(d["b"][:, 0]).contiguous()
    g1, b1 = C.npu_fused_gdn_gating(_to(d["A_log"]), a2, b2, _to(d["dt_bias"]))
    g2, bb2 = ops.npu_fused_gdn_gating(_to(d["A_log"]), a2, b2, _to(d["dt_bias"]))
    assert torch.equal(g1, g2) and torch.equal(b1, bb2)
    idx = torch.arange(4, dtype=torch.int32, device=DEV)
    cu = torch.arange(5, dtype=torch.int32, device=DEV)
    s1, s2 = d["h0"].clone().to(DEV), d["h0"].clone().to(DEV)
    args = [_to(d[n]) for n in ("A_log", "a", "dt_bias", "q", "k", "v", "b")]
    o1 = C.npu_fused_sigmoid_gating_delta_rule_update(*args, s1, idx, cu, None, True)
    o2 = ops.npu_fused_sigmoid_gating_delta_rule_update(*args, s2, idx, cu, None, True)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    assert C.kernel_entry_point("fused_gdn_gating_decode_kernel") == "xops_fused_gdn_gating"


def test_recurrent_negative_slot():
    """The plain recurrent op gives a negative slot the same meaning."""
    d = _inputs(1, 4, 2, 4, 128, 8)
    g = -torch.rand(1, 4, 4)
    beta = torch.rand(1, 4, 4)
    cu = torch.tensor([0, 1, 4], dtype=torch.int32)
    idx = torch.tensor([-1, 1], dtype=torch.int32)
    h0 = torch.randn(2, 4, 128, 128)
    st = h0.clone().to(DEV)
    o, _ = ops.npu_fused_recurrent_gated_delta_rule(_to(d["q"]), _to(d["k"]), _to(d["v"]), _to(g),
                                                    _to(beta), None, st, True, _to(cu), _to(idx),
                                                    None, True)
    assert torch.equal(st[0].cpu(), h0[0])  # no write-back for the negative slot
    z = torch.zeros(1, 4, 128, 128)
    ro0, _ = oracle.fused_recurrent_gated_delta_rule(d["q"][:, :1], d["k"][:, :1], d["v"][:, :1],
                                                     g[:, :1], beta[:, :1], None, z, True, None,
                                                     None, True)
    assert_bf16(o[:, :1], ro0)
