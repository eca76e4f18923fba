"""The reference runtime's launch path, OperationBase::execute through
OperationFactory, packing the argument lists of the reference's call sites
(triton_npu/torch_api/*.cpp), launches the same kernels as the torch API and
matches the oracle."""

import pytest
import torch
import torch.nn.functional as F

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


def _p(t):
    return ("ptr", None if t is None else t.data_ptr())


def _execute(C, name, grid, args):
    rc, err, _ = C._runtime_execute(name, *grid, args, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert rc == 0, f"{name}: {rc} {err}"


@pytest.mark.parametrize("z", [False, True])
def test_factory_layer_norm_fwd_execute(C, z):
    """OperationFactory::instance().layer_norm_fwd().execute(...) with the
    reference's group_size > 128 argument list: RMSNorm, optional gate."""
    g = torch.Generator().manual_seed(31)
    M, N, G = 300, 1024, 512
    x = torch.randn(M, N, generator=g).to(torch.bfloat16)
    w = (1 + 0.1 * torch.randn(N, generator=g)).to(torch.bfloat16)
    zz = torch.randn(M, N, generator=g).to(torch.bfloat16) if z else None
    y, rstd = C._runtime_layer_norm_fwd(x.to(DEV), w.to(DEV), None if zz is None else zz.to(DEV),
                                        1e-6, G)
    ry, _, rrstd = oracle.layer_norm_fwd(x, w, None, 1e-6, zz, G, True, True)
    assert_bf16(y, ry)
    assert_fp32(rstd, rrstd.reshape(-1))


# (kernel name, rms, bf16, z, bias) of the reference's fast variants
FAST = [
    ("layer_norm_fwd_kernel_fast", False, False, False, True),
    ("layer_norm_fwd_kernel_fast_bf16", False, True, False, True),
    ("layer_norm_fwd_kernel_fast_rms_bias", True, False, False, True),
    ("layer_norm_fwd_kernel_fast_rms_bf16_nobias", True, True, False, False),
    ("layer_norm_fwd_kernel_fast_z", False, False, True, True),
    ("layer_norm_fwd_kernel_fast_bf16_z", False, True, True, False),
    ("layer_norm_fwd_kernel_fast_rms_z_nobias", True, False, True, False),
    ("layer_norm_fwd_kernel_fast_rms_bf16_z_bias", True, True, True, True),
    ("layer_norm_fwd_kernel_fast_rms_bf16_z_nobias_nomask", True, True, True, False),
]


@pytest.mark.parametrize("name,rms,bf16,z,bias", FAST, ids=[f[0] for f in FAST])
def test_layer_norm_fast_variants(C, name, rms, bf16, z, bias):
    """Argument lists of npu_triton_layernorm_fwd.cpp:154-257 (gate z, bias and
    mean slots as each variant packs them)."""
    g = torch.Generator().manual_seed(len(name))
    M, G, ng = 1030, 128, 2
    N = G * ng
    dt = torch.bfloat16 if bf16 else torch.float32
    x = torch.randn(M, N, generator=g).to(dt)
    w = (1 + 0.1 * torch.randn(N, generator=g)).to(dt)
    b = (0.1 * torch.randn(N, generator=g)).to(dt) if bias else None
    zz = torch.randn(M, N, generator=g).to(dt) if z else None
    xd, wd = x.to(DEV), w.to(DEV)
    bd, zd = (None if b is None else b.to(DEV)), (None if zz is None else zz.to(DEV))
    y = torch.empty_like(xd)
    mean = torch.empty(ng * M, device=DEV)
    rstd = torch.empty(ng * M, device=DEV)
    args = [_p(xd), _p(y), _p(wd)]
    if bias or not rms:
        args.append(_p(bd))
    if z:
        args.append(_p(zd))
    if not rms:
        args.append(_p(mean))
    args += [_p(rstd), ("i32", N), ("i32", N), ("i32", N if z else 0), ("i32", M), ("i32", G),
             ("f32", 1e-6), ("i32", 40)]
    _execute(C, name, (40, ng, 1), args)
    ry, rmean, rrstd = oracle.layer_norm_fwd(x, w, b, 1e-6, zz, G, True, rms)
    (assert_bf16 if bf16 else assert_fp32)(y, ry)
    assert_fp32(rstd, rrstd.reshape(-1))
    if not rms:
        assert_fp32(mean, rmean.reshape(-1), scale=x.float().abs().max().item())


def test_l2norm_execute(C):
    x = torch.randn(777, 128, dtype=torch.bfloat16, device=DEV)
    y = torch.empty_like(x)
    _execute(C, "l2norm_fwd_kernel2_loop", (40, 1, 1),
             [_p(x), _p(y), ("f32", 1e-6), ("i32", 777), ("i32", 128), ("i32", 1), ("i32", 1)])
    assert torch.equal(y, ops.npu_l2norm_last_dim(x, 1e-6))


def test_gdn_gating_execute(C):
    g0 = torch.Generator().manual_seed(3)
    B, H = 256, 32
    A_log = (torch.rand(H, generator=g0) * 2.7).to(DEV)
    dtb = torch.rand(H, generator=g0).to(DEV)
    a = torch.randn(B, H, generator=g0).to(torch.bfloat16).to(DEV)
    b = torch.randn(B, H, generator=g0).to(torch.bfloat16).to(DEV)
    g = torch.empty(1, B, H, device=DEV)
    beta = torch.empty(1, B, H, dtype=torch.bfloat16, device=DEV)
    _execute(C, "fused_gdn_gating_decode_kernel", (B, 1, (H + 7) // 8),
             [_p(g), _p(beta), _p(A_log), _p(a), _p(b), _p(dtb), ("i32", H)])
    rg, rb = ops.npu_fused_gdn_gating(A_log, a, b, dtb)
    assert torch.equal(g, rg) and torch.equal(beta, rb)


def test_split_rmsnorm_rope_execute(C):
    T, qh, kvh, hd = 64, 4096, 512, 256
    g0 = torch.Generator().manual_seed(4)
    inp = torch.randn(T, qh + 2 * kvh, generator=g0).to(torch.bfloat16).to(DEV)
    sin, cos = workloads.neox_sin_cos(torch.arange(T), hd, 1e6)
    sin, cos = sin.to(torch.bfloat16).to(DEV), cos.to(torch.bfloat16).to(DEV)
    qw = (1 + 0.1 * torch.randn(hd, generator=g0)).to(torch.bfloat16).to(DEV)
    kw = (1 + 0.1 * torch.randn(hd, generator=g0)).to(torch.bfloat16).to(DEV)
    q = torch.empty(T, qh, dtype=torch.bfloat16, device=DEV)
    k = torch.empty(T, kvh, dtype=torch.bfloat16, device=DEV)
    v = torch.empty(T, kvh, dtype=torch.bfloat16, device=DEV)
    # the name the reference builds for eps 1e-6 (std::to_string -> "0.000001")
    name = f"split_rmsnorm_rope_kernel_bias0_eps0000001_hd{hd}_qh{qh}_kvh{kvh}"
    _execute(C, name, (20, kvh // hd, 1),
             [_p(inp), _p(sin), _p(cos), _p(q), _p(k), _p(v), _p(qw), ("ptr", None), _p(kw),
              ("ptr", None), ("i32", T)])
    rq, rk, rv = ops.npu_split_rmsnorm_rope(inp, sin, cos, qw, kw, qh, kvh, hd, 1e-6)
    assert torch.equal(q, rq) and torch.equal(k, rk) and torch.equal(v, rv)


def test_conv_qwen_decode_execute(C):
    d = workloads.conv_decode_config2(batch=64)
    x = d["x"].to(DEV).unsqueeze(-1).contiguous()
    st = d["conv_state"].to(DEV)
    st2 = st.clone()
    w = d["weight"].to(DEV)
    out = torch.empty_like(x)
    _execute(C, "_causal_conv1d_update_qwen_decode_kernel", (64, 8192 // 256, 1),
             [_p(x), _p(st), _p(w), ("ptr", None), _p(out), ("i32", -1), ("i32", 64),
              ("i32", 8192)])
    ro = ops.npu_causal_conv1d_update(x, st2, w, True, None)
    assert torch.equal(out, ro) and torch.equal(st, st2)


def test_recurrent_execute(C):
    w = workloads.decode_config4(batch=32)
    d = {n: (t.to(DEV) if torch.is_tensor(t) else t) for n, t in w.items()}
    st = d["state"].clone()
    o = torch.empty(1, 1, 32, 32, 128, dtype=torch.bfloat16, device=DEV)
    N, H, HV = 32, 16, 32
    _execute(C, "fused_recurrent_gated_delta_rule_fwd_kernel", (1, 2, N * HV),
             [_p(d["q"]), _p(d["k"]), _p(d["v"]), _p(d["g"]), _p(d["beta"]), _p(o), _p(st), _p(st),
              _p(d["cu_seqlens"]), _p(d["ssm_state_indices"]), ("f32", 128 ** -0.5),
              ("i64", N), ("i64", 32), ("i64", H), ("i64", HV), ("i64", st.stride(0)),
              ("i64", st.stride(0))])
    st_ref = w["state"].clone()
    ro, _ = oracle.fused_recurrent_gated_delta_rule(w["q"], w["k"], w["v"], w["g"], w["beta"],
                                                    None, st_ref, True, w["cu_seqlens"],
                                                    w["ssm_state_indices"], True)
    assert_bf16(o.reshape(ro.shape), ro)
    assert_state(st, st_ref)
