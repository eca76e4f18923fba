"""The C++ torch API (xllm::kernel::npu / npu_ops, pybind module
torch_npu_ops_b200._C) gives the same results as the ctypes host API and
the oracle, and keeps the reference's pybind schemas."""

import pytest
import torch

import oracle
import torch_npu_ops_b200 as ops
from parity import assert_bf16, assert_fp32, assert_state
from torch_npu_ops_b200 import workloads

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module")
def C():
    from torch_npu_ops_b200 import _C
    return _C


def test_schemas_match_reference(C):
    x = torch.randn(4, 128, 4096, dtype=torch.bfloat16, device=DEV)
    gamma = torch.randn(4096, dtype=torch.bfloat16, device=DEV)
    rstd, y = C.gemma_rms_norm(x, gamma, 1e-6)
    assert y.shape == x.shape and rstd.shape == (4, 128, 1) and rstd.dtype == torch.float32
    rr, ry = oracle.gemma_rms_norm(x.cpu(), gamma.cpu(), 1e-6)
    assert_bf16(y, ry)
    out = C.layer_norm_fwd(x=x.reshape(-1, 4096), weight=gamma, bias=None, eps=1e-6, z=None,
                           group_size=128, norm_before_gate=True, is_rms_norm=True)
    ref, _, _ = oracle.layer_norm_fwd(x.cpu().reshape(-1, 4096), gamma.cpu(), None, 1e-6, None,
                                      128, True, True)
    assert_bf16(out, ref)


def test_chunk_and_recurrent_via_cpp(C):
    w = workloads.chunk_config3(hk=2, hv=4, lengths=[100, 300], seed=12)
    d = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in w.items()}
    o1, h1 = C.npu_chunk_gated_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], None,
                                          d["initial_state"], True, d["cu_seqlens"], False, False)
    o2, h2 = ops.npu_chunk_gated_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"], None,
                                            d["initial_state"], True, d["cu_seqlens"])
    assert torch.equal(o1, o2) and torch.equal(h1, h2)
    dec = workloads.decode_config4(batch=8, hk=2, hv=4)
    st1 = dec["state"].clone().to(DEV)
    st2 = dec["state"].clone().to(DEV)
    a = {k: (v.to(DEV) if torch.is_tensor(v) else v) for k, v in dec.items()}
    oa, _ = C.npu_fused_recurrent_gated_delta_rule(a["q"], a["k"], a["v"], a["g"], a["beta"], None,
                                                   st1, True, a["cu_seqlens"],
                                                   a["ssm_state_indices"],
                                                   use_qk_l2norm_in_kernel=True)
    ob, _ = ops.npu_fused_recurrent_gated_delta_rule(a["q"], a["k"], a["v"], a["g"], a["beta"],
                                                     None, st2, True, a["cu_seqlens"],
                                                     a["ssm_state_indices"], None, True)
    assert torch.equal(oa, ob) and torch.equal(st1, st2)


def test_conv_and_rope_via_cpp(C):
    w = workloads.conv_prefill_config2(total=2048, nseq=4, dim=1024)
    st = w["conv_state"].clone().to(DEV)
    y = C.npu_causal_conv1d_update_v2(w["x"].to(DEV), st, w["weight"].to(DEV), True,
                                      w["bias"].to(DEV), None, w["query_start_loc"].to(DEV))
    st_ref = w["conv_state"].clone()
    ref = oracle.causal_conv1d_varlen(w["x"], st_ref, w["weight"], w["bias"], True,
                                      w["query_start_loc"])
    assert_bf16(y, ref)
    assert torch.equal(st.cpu(), st_ref)
    r = workloads.rope_config1()
    q, k, v = C.npu_split_rmsnorm_rope(*[t.to(DEV) for t in r["tensors"]], **r["kwargs"])
    rq, rk, _ = oracle.split_rmsnorm_rope(*r["tensors"], **r["kwargs"])
    assert_fp32(q, rq)
    assert_fp32(k, rk)


def test_registry_maps_reference_kernel_names(C):
    assert C.kernel_entry_point("chunk_gated_delta_rule_fwd_kernel_h_blockdim64") == \
        "xops_chunk_gated_delta_rule_fwd_h"
    assert C.kernel_entry_point("layer_norm_fwd_kernel_fast_rms_bf16_z_nobias_nomask") == \
        "xops_layer_norm_fwd"
    assert C.kernel_entry_point("rope_inplace_kernel") == "xops_rope_inplace"
    assert C.kernel_entry_point("a_kernel_the_reference_does_not_have") == ""
