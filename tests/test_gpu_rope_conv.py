"""GPU parity: split_rmsnorm_rope (full and partial rotary) and causal conv1d
(varlen prefill + decode update)."""

import pytest
import torch

import oracle
import torch_npu_ops_b200 as ops
from parity import assert_bf16, assert_fp32, golden
from torch_npu_ops_b200 import workloads

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _to(t):
    return None if t is None else t.to(DEV)


@pytest.mark.parametrize("case", golden("split_rmsnorm_rope"), ids=lambda c: c["name"])
def test_rope_golden(case):
    a = case["args"]
    q, k, v = ops.npu_split_rmsnorm_rope(_to(a["input"]), _to(a["sin"]), _to(a["cos"]),
                                         _to(a["q_weight"]), _to(a["k_weight"]),
                                         a["q_hidden_size"], a["kv_hidden_size"], a["head_dim"],
                                         a["eps"], _to(a["q_bias"]), _to(a["k_bias"]), a["bias"])
    assert_fp32(q, case["out"]["q"])
    assert_fp32(k, case["out"]["k"])
    assert torch.equal(v.cpu(), case["out"]["v"])


def test_rope_config1():
    w = workloads.rope_config1()
    q, k, v = ops.npu_split_rmsnorm_rope(*[_to(t) for t in w["tensors"]], **w["kwargs"])
    rq, rk, rv = oracle.split_rmsnorm_rope(*w["tensors"], **w["kwargs"])
    assert_fp32(q, rq)
    assert_fp32(k, rk)
    assert torch.equal(v.cpu(), rv)


@pytest.mark.parametrize("T,qh,kvh,hd,rd,dt,bias", [
    (333, 8, 1, 128, 128, torch.bfloat16, False),
    (17, 4, 4, 64, 32, torch.float32, False),
    (64, 16, 2, 256, 64, torch.bfloat16, False),
    # >= 4 MB of input: the bulk-copy streaming path
    (1024, 16, 2, 256, 64, torch.float32, False),    # cfg1 heads at 1024 tokens
    (2000, 8, 1, 128, 128, torch.float32, True),     # full rotary, bias
    (1500, 16, 2, 256, 64, torch.bfloat16, True),
    (700, 4, 2, 512, 200, torch.float32, False),     # rotary half not a lane multiple
    (800, 4, 2, 256, 42, torch.float32, True),       # cos/sin rows not 16-byte multiples
])
def test_rope_shapes(T, qh, kvh, hd, rd, dt, bias):
    g = torch.Generator().manual_seed(T)
    inp = torch.randn(T, (qh + 2 * kvh) * hd, generator=g).to(dt)
    qw = (1 + 0.1 * torch.randn(hd, generator=g)).to(dt)
    kw = (1 + 0.1 * torch.randn(hd, generator=g)).to(dt)
    qb = (0.1 * torch.randn(hd, generator=g)).to(dt) if bias else None
    kb = (0.1 * torch.randn(hd, generator=g)).to(dt) if bias else None
    sin, cos = workloads.neox_sin_cos(torch.arange(T) * 7, rd, 1e6)
    q, k, v = ops.npu_split_rmsnorm_rope(_to(inp), _to(sin), _to(cos), _to(qw), _to(kw), qh * hd,
                                         kvh * hd, hd, 1e-6, _to(qb), _to(kb), bias)
    rq, rk, rv = oracle.split_rmsnorm_rope(inp, sin, cos, qw, kw, qh * hd, kvh * hd, hd, 1e-6,
                                           qb, kb, bias)
    check = assert_fp32 if dt == torch.float32 else assert_bf16
    check(q, rq)
    check(k, rk)
    assert torch.equal(v.cpu(), rv)


@pytest.mark.parametrize("case", golden("causal_conv1d"), ids=lambda c: c["name"])
def test_conv_golden(case):
    a = case["args"]
    st = a["conv_state"].clone().to(DEV)
    if case["kind"] == "update":
        y = ops.npu_causal_conv1d_update(_to(a["x"]), st, _to(a["weight"]), True, _to(a["bias"]))
    else:
        y = ops.npu_causal_conv1d_update_v2(_to(a["x"]), st, _to(a["weight"]), True, _to(a["bias"]),
                                            query_start_loc=_to(a["query_start_loc"]))
    st_ref = a["conv_state"].clone()
    if case["kind"] == "update":
        ref = oracle.causal_conv1d_update(a["x"], st_ref, a["weight"], a["bias"], True)
    else:
        ref = oracle.causal_conv1d_varlen(a["x"], st_ref, a["weight"], a["bias"], True,
                                          a["query_start_loc"])
    (assert_fp32 if a["x"].dtype == torch.float32 else assert_bf16)(y, ref)
    assert torch.equal(st.cpu(), st_ref)
    assert torch.equal(st.cpu(), case["out"]["conv_state"])


def test_conv_prefill_config2():
    w = workloads.conv_prefill_config2()
    x, st, wt, b, qsl = w["x"], w["conv_state"], w["weight"], w["bias"], w["query_start_loc"]
    st_d = st.clone().to(DEV)
    y = ops.npu_causal_conv1d_update_v2(x.to(DEV), st_d, wt.to(DEV), True, b.to(DEV),
                                        query_start_loc=qsl.to(DEV))
    st_ref = st.clone()
    ref = oracle.causal_conv1d_varlen(x, st_ref, wt, b, True, qsl)
    assert_bf16(y, ref)
    assert torch.equal(st_d.cpu(), st_ref)


@pytest.mark.parametrize("lens,dim,width,dt", [
    ([300, 5, 1000], 264, 2, torch.bfloat16),   # partial 256-channel slab, width 2
    ([129, 31, 2], 520, 6, torch.float16),      # width 6 (5-row halo), fp16
    ([33, 64, 95], 1024, 4, torch.bfloat16),    # tiles ending mid-box
])
def test_conv_varlen_widths_and_slabs(lens, dim, width, dt):
    g = torch.Generator().manual_seed(dim + width)
    T = sum(lens)
    x = torch.randn(T, dim, generator=g).to(dt)
    st = torch.randn(len(lens), dim, width - 1, generator=g).to(dt)
    wt = (0.5 * torch.randn(dim, width, generator=g)).to(dt)
    b = (0.5 * torch.randn(dim, generator=g)).to(dt)
    qsl = torch.tensor([0] + torch.cumsum(torch.tensor(lens), 0).tolist(), dtype=torch.int32)
    st_d = st.clone().to(DEV)
    y = ops.npu_causal_conv1d_update_v2(x.to(DEV), st_d, wt.to(DEV), True, b.to(DEV),
                                        query_start_loc=qsl.to(DEV))
    st_ref = st.clone()
    ref = oracle.causal_conv1d_varlen(x, st_ref, wt, b, True, qsl)
    assert_bf16(y, ref)
    assert torch.equal(st_d.cpu(), st_ref)


def test_conv_varlen_ragged_and_slots():
    g = torch.Generator().manual_seed(11)
    lens = [1, 2, 3, 64, 65, 0, 200, 7]
    dim, width = 256, 4
    T = sum(lens)
    x = torch.randn(T, dim, generator=g).to(torch.bfloat16)
    st = torch.randn(12, dim, width - 1, generator=g).to(torch.bfloat16)
    wt = (0.5 * torch.randn(dim, width, generator=g)).to(torch.bfloat16)
    b = (0.5 * torch.randn(dim, generator=g)).to(torch.bfloat16)
    qsl = torch.tensor([0] + torch.cumsum(torch.tensor(lens), 0).tolist(), dtype=torch.int32)
    slots = torch.tensor([3, 0, 11, 5, -1, 7, 2, 9], dtype=torch.int32)  # one padded slot
    st_d = st.clone().to(DEV)
    y = ops.npu_causal_conv1d_update_v2(x.to(DEV), st_d, wt.to(DEV), True, b.to(DEV),
                                        conv_state_indices=slots.to(DEV),
                                        query_start_loc=qsl.to(DEV), pad_slot_id=-1)
    st_ref = st.clone()
    ref = oracle.causal_conv1d_varlen(x, st_ref, wt, b, True, qsl, slots, pad_slot_id=-1)
    keep = torch.ones(T, dtype=torch.bool)
    keep[int(qsl[4]):int(qsl[5])] = False  # padded sequence: output unspecified
    assert_bf16(y.cpu()[keep], ref[keep])
    assert torch.equal(st_d.cpu(), st_ref)


@pytest.mark.parametrize("B,dim,L,width,state_len,bias,dt", [
    (256, 8192, 1, 4, 3, True, torch.bfloat16),  # config 2 decode
    (16, 2048, 1, 4, 3, False, torch.bfloat16),
    (7, 64, 3, 4, 5, True, torch.float32),
    (4, 128, 2, 3, 2, True, torch.float16),
])
def test_conv_decode(B, dim, L, width, state_len, bias, dt):
    g = torch.Generator().manual_seed(B + dim)
    x = torch.randn(B, dim, L, generator=g).to(dt)
    st = torch.randn(B + 3, dim, state_len, generator=g).to(dt)
    wt = (0.5 * torch.randn(dim, width, generator=g)).to(dt)
    b = (0.5 * torch.randn(dim, generator=g)).to(dt) if bias else None
    slots = torch.randperm(B + 3, generator=g)[:B].to(torch.int32)
    st_d = st.clone().to(DEV)
    y = ops.npu_causal_conv1d_update(x.to(DEV), st_d, wt.to(DEV), True, _to(b),
                                     conv_state_indices=slots.to(DEV))
    st_ref = st.clone()
    ref = oracle.causal_conv1d_update(x, st_ref, wt, b, True, slots)
    (assert_fp32 if dt == torch.float32 else assert_bf16)(y, ref)
    assert torch.equal(st_d.cpu(), st_ref)


def test_conv_decode_pad_slot_untouched():
    x = torch.randn(3, 64, dtype=torch.bfloat16)
    st = torch.randn(3, 64, 3, dtype=torch.bfloat16)
    wt = torch.randn(64, 4, dtype=torch.bfloat16)
    slots = torch.tensor([2, -1, 0], dtype=torch.int32)
    st_d = st.clone().to(DEV)
    ops.npu_causal_conv1d_update(x.to(DEV), st_d, wt.to(DEV), True, None,
                                 conv_state_indices=slots.to(DEV), pad_slot_id=-1)
    assert torch.equal(st_d.cpu()[1], st[1])
