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
    # partner in the same lane's chunk half / (32 V) rows away
    (1200, 8, 2, 256, 256, torch.float32, True),
    (600, 4, 2, 512, 512, torch.float32, False),
    (900, 4, 2, 512, 256, torch.float32, False),
    (700, 4, 2, 512, 512, torch.bfloat16, False),
    (800, 4, 2, 512, 128, torch.bfloat16, True),     # partner lane of chunk 0, two chunks
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
    (9, 512, 1, 4, 3, True, torch.float16),   # odd batch on the two-rows-per-thread path
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


@pytest.mark.parametrize("B,bias", [(5, False), (4096, True)])
def test_conv_decode_rows_without_slots(B, bias):
    # rows map to their own state lines; an odd batch leaves the second row
    # of the last thread empty
    g = torch.Generator().manual_seed(B)
    dim = 8192 if B > 64 else 128
    x = torch.randn(B, dim, generator=g).to(torch.bfloat16)
    st = torch.randn(B, dim, 3, generator=g).to(torch.bfloat16)
    wt = (0.5 * torch.randn(dim, 4, generator=g)).to(torch.bfloat16)
    b = (0.5 * torch.randn(dim, generator=g)).to(torch.bfloat16) if bias else None
    st_d = st.clone().to(DEV)
    y = ops.npu_causal_conv1d_update(x.to(DEV), st_d, wt.to(DEV), True, _to(b))
    st_ref = st.clone()
    ref = oracle.causal_conv1d_update(x, st_ref, wt, b, True)
    assert_bf16(y, ref)
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


# ------------------------------------- conv v2 slot tables (spec decode, APC)
@pytest.mark.parametrize("case", golden("causal_conv1d_slots"), ids=lambda c: c["name"])
def test_conv_slots_golden(case):
    a = case["args"]
    st = a["conv_state"].clone().to(DEV)
    y = ops.npu_causal_conv1d_update_v2(
        _to(a["x"]), st, _to(a["weight"]), a["activation"], _to(a["bias"]),
        _to(a["conv_state_indices"]), _to(a["query_start_loc"]), a["max_query_len"],
        a["pad_slot_id"], _to(a["block_idx_last_scheduled_token"]), _to(a["initial_state_idx"]),
        False, _to(a["num_accepted_tokens"]))
    assert torch.equal(st.cpu(), case["out"]["conv_state"])
    # the reference test's own output bound (it convolves in bf16)
    torch.testing.assert_close(y.cpu().float(), case["out"]["out"].float(), rtol=1e-2, atol=5e-2)


@pytest.mark.parametrize("dt", [torch.bfloat16, torch.float32])
def test_conv_slots_varlen_spec(dt):
    """Varlen speculative decoding with different lengths per sequence (each
    sequence's window from its own length), a [B, blocks] table with
    prefix-cache read / write blocks, and a padded row."""
    g = torch.Generator().manual_seed(31)
    dim, width, lens = 320, 4, [3, 1, 0, 2]
    B = len(lens)
    x = torch.randn(sum(lens), dim, generator=g).to(dt)
    lines = 8
    st = torch.randn(lines, dim, width - 1 + max(lens) - 1, generator=g).to(dt)
    w = torch.randn(dim, width, generator=g).to(dt)
    b = torch.randn(dim, generator=g).to(dt)
    qsl = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    idx = torch.tensor([[1, 2, 3], [4, 5, 6], [-1, -1, -1], [7, 0, 0]], dtype=torch.int32)
    ini = torch.tensor([0, 1, 0, 0], dtype=torch.int32)
    last = torch.tensor([2, 1, 0, 1], dtype=torch.int32)
    acc = torch.tensor([2, 1, 1, 3], dtype=torch.int32)
    st_d = st.clone().to(DEV)
    y = ops.npu_causal_conv1d_update_v2(_to(x), st_d, _to(w), True, _to(b), _to(idx), _to(qsl),
                                        max(lens), -1, _to(last), _to(ini), False, _to(acc))
    st_ref = st.clone()
    ref = oracle.causal_conv1d_update_v2_slots(x, st_ref, w, b, True, qsl, idx, acc, ini, last, -1)
    (assert_fp32 if dt == torch.float32 else assert_bf16)(y, ref)
    assert torch.equal(st_d.cpu(), st_ref)


def test_conv_slots_wide_state_no_spec_and_cpp():
    """A cache wider than width - 1 without speculative decoding rewrites
    only the first width - 1 columns; the C++ API takes the same path."""
    from torch_npu_ops_b200 import _C as C
    g = torch.Generator().manual_seed(32)
    B, dim, width, T = 3, 256, 4, 2
    x = torch.randn(B, dim, T, generator=g).to(torch.bfloat16)
    st = torch.randn(B, dim, 6, generator=g).to(torch.bfloat16)
    w = torch.randn(dim, width, generator=g).to(torch.bfloat16)
    idx = torch.tensor([2, 0, 1], dtype=torch.int32)
    s1, s2 = st.clone().to(DEV), st.clone().to(DEV)
    y1 = ops.npu_causal_conv1d_update_v2(_to(x), s1, _to(w), True, None, _to(idx))
    y2 = C.npu_causal_conv1d_update_v2(_to(x), s2, _to(w), True, None, _to(idx))
    assert torch.equal(y1, y2) and torch.equal(s1, s2)
    st_ref = st.clone()
    xt = x.transpose(1, 2).reshape(B * T, dim)
    qsl = torch.arange(B + 1, dtype=torch.int32) * T
    ref = oracle.causal_conv1d_update_v2_slots(xt, st_ref, w, None, True, qsl, idx)
    assert_bf16(y1.transpose(1, 2).reshape(B * T, dim), ref)
    assert torch.equal(s1.cpu(), st_ref)
    assert torch.equal(s1.cpu()[:, :, width - 1:], st[:, :, width - 1:])  # columns 3.. untouched


# -------------------------------------------------------------- rope_inplace
@pytest.mark.parametrize("case", golden("rope_inplace"), ids=lambda c: c["name"])
def test_rope_inplace_golden(case):
    a = case["args"]
    x = a["x"].clone().to(DEV)
    y = ops.rope_inplace(x, _to(a["sin"]), _to(a["cos"]), a["rope_dim"])
    assert y.data_ptr() == x.data_ptr()
    assert_bf16(x, case["out"]["x"])
    pre = a["x"].shape[-1] - a["rope_dim"]
    assert torch.equal(x.cpu()[..., :pre], a["x"][..., :pre])  # the head part is untouched


@pytest.mark.parametrize("dt,sdt", [(torch.float32, torch.float32), (torch.bfloat16, torch.float32),
                                    (torch.float16, torch.float16)])
def test_rope_inplace_strided_views(dt, sdt):
    """q_pe-style views: the rotated vectors are slices of a wider packed
    tensor (row and head strides), sin / cos rows wider than rope_dim."""
    g = torch.Generator().manual_seed(9)
    bsz, heads, hidden, rd = 5, 3, 192, 64
    packed = torch.randn(bsz, heads, 2 * hidden, generator=g).to(dt)
    sin = torch.randn(bsz, 96, generator=g).to(sdt)
    cos = torch.randn(bsz, 96, generator=g).to(sdt)
    pd = packed.clone().to(DEV)
    view = pd[:, :, hidden:]
    ops.rope_inplace(view, _to(sin), _to(cos), rd)
    ref = packed.clone()
    oracle.rope_inplace(ref[:, :, hidden:], sin, cos, rd)
    (assert_fp32 if dt == torch.float32 else assert_bf16)(pd, ref)
    assert torch.equal(pd.cpu()[:, :, :hidden], packed[:, :, :hidden])


def test_rope_inplace_cpp():
    from torch_npu_ops_b200 import _C as C
    g = torch.Generator().manual_seed(10)
    x = torch.randn(4, 8, 512, generator=g).to(torch.bfloat16)
    sin = torch.randn(4, 64, generator=g).to(torch.bfloat16)
    cos = torch.randn(4, 64, generator=g).to(torch.bfloat16)
    x1, x2 = x.clone().to(DEV), x.clone().to(DEV)
    C.rope_inplace(x1, _to(sin), _to(cos), 64)
    ops.rope_inplace(x2, _to(sin), _to(cos), 64)
    assert torch.equal(x1, x2)


@pytest.mark.parametrize("lens,dim,qk,dt", [
    ([300, 5, 1000], 1024, 512, torch.bfloat16),    # ragged, half the channels normalised
    ([4096, 2048], 8192, 4096, torch.bfloat16),     # the GDN layer's channel split
    ([129, 64], 768, 256, torch.float16),
])
def test_conv_varlen_qk_l2norm(lens, dim, qk, dt):
    """The fused conv + q/k L2 norm against the reference's two steps: the conv
    output rounded to the activation dtype, then x / sqrt(sum x^2 + eps) per
    128-channel head (l2norm_ref, test_l2norm.py:95) on the first qk channels."""
    g = torch.Generator().manual_seed(dim + qk)
    T = sum(lens)
    x = torch.randn(T, dim, generator=g).to(dt)
    wt = (0.5 * torch.randn(dim, 4, generator=g)).to(dt)
    b = (0.5 * torch.randn(dim, generator=g)).to(dt)
    st = torch.randn(len(lens), dim, 3, generator=g).to(dt)
    qsl = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
    st_d = st.clone().to(DEV)
    y = ops.causal_conv1d_varlen_qk_l2norm(x.to(DEV), st_d, wt.to(DEV), b.to(DEV), qsl.to(DEV), qk)
    st_ref = st.clone()
    with oracle.fp32_outputs():
        ref = oracle.causal_conv1d_varlen(x, st_ref, wt, b, True, qsl)
    y16 = ref.to(dt)  # the reference stores the conv output in the activation dtype
    with oracle.fp32_outputs():
        qk_ref = oracle.l2norm_last_dim(y16[:, :qk].reshape(-1, 128), 1e-6).reshape(T, qk)
    assert_bf16(y[:, :qk], qk_ref)
    assert_bf16(y[:, qk:], ref[:, qk:])
    assert torch.equal(st_d.cpu(), st_ref)
    # the un-normalised channels are exactly those of the plain conv
    st2 = st.clone().to(DEV)
    y2 = ops.npu_causal_conv1d_update_v2(x.to(DEV), st2, wt.to(DEV), True, b.to(DEV),
                                         query_start_loc=qsl.to(DEV))
    assert torch.equal(y[:, qk:], y2[:, qk:])
    if dt == torch.bfloat16:  # the separate l2norm operator takes bf16, as the reference's
        assert_bf16(y[:, :qk],
                    ops.npu_l2norm_last_dim(y2[:, :qk].reshape(-1, 128), 1e-6).reshape(T, qk))
