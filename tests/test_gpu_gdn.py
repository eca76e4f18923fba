"""GPU parity: chunked gated delta rule (fused op and the sub-operator
pipeline) and the fused recurrent (decode) rule, against the CPU oracle and
the reference's golden fixtures."""

import pytest
import torch
import torch.nn.functional as F

import oracle
import torch_npu_ops_b200 as ops
from parity import BF16_MAXABS, assert_bf16, assert_bf16_rel, assert_fp32, assert_state, golden, rel_fro
from torch_npu_ops_b200 import workloads

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _to(t):
    return None if t is None else t.to(DEV)


def _run_chunk(inp, l2=False, scale=None):
    o, ht = ops.npu_chunk_gated_delta_rule(
        _to(inp["q"]), _to(inp["k"]), _to(inp["v"]), _to(inp["g"]), _to(inp["beta"]), scale,
        _to(inp["initial_state"]), True, _to(inp["cu_seqlens"]), False, l2)
    torch.cuda.synchronize()
    return o.cpu(), ht.cpu()


def _oracle_chunk(inp, l2=False, scale=None):
    return oracle.chunk_gated_delta_rule(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"], scale,
                                         inp["initial_state"], True, inp["cu_seqlens"], l2)


@pytest.mark.parametrize("case", golden("chunk_gated_delta_rule"), ids=lambda c: c["name"])
def test_chunk_golden(case):
    a = case["args"]
    if a["q"].shape[-1] != 128 or a["v"].shape[-1] != 128:
        pytest.skip("compiled for head_dim 128 (the reference kernels' constraint)")
    inp = dict(a)
    o, ht = _run_chunk(inp, a["use_qk_l2norm_in_kernel"])
    ro, rh = _oracle_chunk(inp, a["use_qk_l2norm_in_kernel"])
    assert_bf16_rel(o, ro)
    assert_state(ht, rh)
    # and the reference's own output, within its test tolerance (1e-2)
    assert_bf16(o, case["out"]["o"], tol=2e-2)


def test_chunk_config3():
    inp = workloads.chunk_config3()
    o, ht = _run_chunk(inp)
    ro, rh = _oracle_chunk(inp)
    assert_bf16_rel(o, ro)
    assert_state(ht, rh)


@pytest.mark.parametrize("lens,hk,hv,l2,h0", [
    ([1, 63, 64, 65, 0, 129, 7], 2, 4, False, True),     # ragged tails, empty sequence
    ([300], 1, 1, True, False),                         # in-kernel L2 norm, no initial state
    ([64] * 5, 4, 4, False, True),                      # no GQA, exact chunk multiples
    ([1000, 24], 2, 6, True, True),                     # GQA group 3
])
def test_chunk_varlen_edges(lens, hk, hv, l2, h0):
    inp = workloads.chunk_config3(hk=hk, hv=hv, lengths=lens, seed=sum(lens))
    if not h0:
        inp["initial_state"] = None
    if l2:  # raw (un-normalised) q/k so the in-kernel norm matters
        g = torch.Generator().manual_seed(9)
        inp["q"] = torch.randn(inp["q"].shape, generator=g).to(torch.bfloat16)
        inp["k"] = torch.randn(inp["k"].shape, generator=g).to(torch.bfloat16)
    o, ht = ops.npu_chunk_gated_delta_rule(
        _to(inp["q"]), _to(inp["k"]), _to(inp["v"]), _to(inp["g"]), _to(inp["beta"]), None,
        _to(inp["initial_state"]), True, _to(inp["cu_seqlens"]), False, l2)
    ro, rh = oracle.chunk_gated_delta_rule(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"],
                                           None, inp["initial_state"], True, inp["cu_seqlens"], l2)
    assert_bf16_rel(o, ro)
    keep = [i for i, L in enumerate(lens) if L > 0 or h0]
    assert_state(ht.cpu()[keep], rh[keep])


def _segmented(B, T, N, hk, hv, varlen):
    """True when the host plan cuts the chain into segments (the workspace
    then carries segment states beyond the per-chunk part)."""
    from torch_npu_ops_b200 import _lib
    lib = _lib.load()
    chunks = T // 64 + N if varlen else B * ((T + 63) // 64)
    return lib.xops_chunk_gated_delta_rule_workspace_size(B, T, N, hk, hv, 128, 0, int(varlen)) > \
        chunks * hv * 33280


@pytest.mark.parametrize("lens,hk,hv,l2", [
    ([8192], 1, 2, False),                     # one long sequence: 16 segments of 8 chunks
    ([5000, 130, 64, 1, 0, 3000], 1, 2, True),  # long and short sequences share the plan
    ([16384], 2, 4, False),                    # GQA, longer segments
    ([16384], 8, 16, True),                    # 16 heads, in-kernel L2 norm
])
def test_chunk_segmented_chain(lens, hk, hv, l2):
    """Long sequences on few heads run as local / transition / output passes
    over segments plus a combine of the segment states; results match the
    serial recurrence of the oracle."""
    assert _segmented(1, sum(lens), len(lens), hk, hv, True)
    inp = workloads.chunk_config3(hk=hk, hv=hv, lengths=lens, seed=len(lens) + hv)
    o, ht = ops.npu_chunk_gated_delta_rule(
        _to(inp["q"]), _to(inp["k"]), _to(inp["v"]), _to(inp["g"]), _to(inp["beta"]), None,
        _to(inp["initial_state"]), True, _to(inp["cu_seqlens"]), False, l2)
    ro, rh = oracle.chunk_gated_delta_rule(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"],
                                           None, inp["initial_state"], True, inp["cu_seqlens"], l2)
    assert_bf16_rel(o, ro)
    assert_state(ht, rh)


def test_chunk_segmented_batched_no_cu():
    """Equal-length batch without cu_seqlens on the segmented plan."""
    B, T, hk, hv = 2, 4096, 1, 2
    assert _segmented(B, T, B, hk, hv, False)
    g = torch.Generator().manual_seed(21)
    q = F.normalize(torch.randn(B, T, hk, 128, generator=g), dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(B, T, hk, 128, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, T, hv, 128, generator=g).to(torch.bfloat16)
    gate, beta = workloads.gdn_gates(B * T, hv, g)
    gate, beta = gate.reshape(B, T, hv), beta.reshape(B, T, hv)
    h0 = 0.02 * torch.randn(B, hv, 128, 128, generator=g)
    o, ht = ops.npu_chunk_gated_delta_rule(_to(q), _to(k), _to(v), _to(gate), _to(beta), None,
                                           _to(h0), True, None)
    ro, rh = oracle.chunk_gated_delta_rule(q, k, v, gate, beta, None, h0, True, None)
    assert_bf16_rel(o, ro)
    assert_state(ht, rh)


def test_chunk_batched_no_cu_and_scale():
    g = torch.Generator().manual_seed(21)
    B, T = 3, 150
    q = F.normalize(torch.randn(B, T, 2, 128, generator=g), dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(B, T, 2, 128, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(B, T, 4, 128, generator=g).to(torch.bfloat16)
    gate = F.logsigmoid(torch.randn(B, T, 4, generator=g))
    beta = torch.sigmoid(torch.randn(B, T, 4, generator=g))
    h0 = 0.1 * torch.randn(B, 4, 128, 128, generator=g)
    o, ht = ops.npu_chunk_gated_delta_rule(_to(q), _to(k), _to(v), _to(gate), _to(beta), 0.05,
                                           _to(h0), True, None)
    ro, rh = oracle.chunk_gated_delta_rule(q, k, v, gate, beta, 0.05, h0, True, None)
    assert_bf16_rel(o, ro)
    assert_state(ht, rh)


def test_chunk_strided_qkv_views():
    """q/k/v as slices of one packed [T, (2*Hk + Hv) * 128] tensor (the conv
    output layout) give the same result as contiguous inputs."""
    inp = workloads.chunk_config3(hk=2, hv=4, lengths=[200, 77], seed=4)
    T = 277
    packed = torch.cat([inp["q"].reshape(T, -1), inp["k"].reshape(T, -1), inp["v"].reshape(T, -1)],
                       dim=1).to(DEV)
    qv = packed[:, :256].view(1, T, 2, 128)
    kv = packed[:, 256:512].view(1, T, 2, 128)
    vv = packed[:, 512:].view(1, T, 4, 128)
    o1, h1 = ops.npu_chunk_gated_delta_rule(qv, kv, vv, _to(inp["g"]), _to(inp["beta"]), None,
                                            _to(inp["initial_state"]), True, _to(inp["cu_seqlens"]))
    o2, h2 = ops.npu_chunk_gated_delta_rule(_to(inp["q"]), _to(inp["k"]), _to(inp["v"]),
                                            _to(inp["g"]), _to(inp["beta"]), None,
                                            _to(inp["initial_state"]), True, _to(inp["cu_seqlens"]))
    assert torch.equal(o1, o2) and torch.equal(h1, h2)


def test_chunk_strided_l2_streaming():
    """In-kernel q/k L2 norm on >= 8192 (token, head) rows goes through the
    bulk-copy streaming pre-pass; strided q/k views (one copy per token row)
    and contiguous inputs (one copy per tile) agree bit for bit and match the
    oracle."""
    inp = workloads.chunk_config3(hk=2, hv=4, lengths=[3000, 1200], seed=5)
    T = 4200
    g = torch.Generator().manual_seed(10)
    inp["q"] = torch.randn(inp["q"].shape, generator=g).to(torch.bfloat16)
    inp["k"] = torch.randn(inp["k"].shape, generator=g).to(torch.bfloat16)
    packed = torch.cat([inp["q"].reshape(T, -1), inp["k"].reshape(T, -1), inp["v"].reshape(T, -1)],
                       dim=1).to(DEV)
    qv = packed[:, :256].view(1, T, 2, 128)
    kv = packed[:, 256:512].view(1, T, 2, 128)
    vv = packed[:, 512:].view(1, T, 4, 128)
    args = (_to(inp["g"]), _to(inp["beta"]), None, _to(inp["initial_state"]), True,
            _to(inp["cu_seqlens"]), False, True)
    o1, h1 = ops.npu_chunk_gated_delta_rule(qv, kv, vv, *args)
    o2, h2 = ops.npu_chunk_gated_delta_rule(_to(inp["q"]), _to(inp["k"]), _to(inp["v"]), *args)
    assert torch.equal(o1, o2) and torch.equal(h1, h2)
    ro, rh = oracle.chunk_gated_delta_rule(inp["q"], inp["k"], inp["v"], inp["g"], inp["beta"],
                                           None, inp["initial_state"], True, inp["cu_seqlens"], True)
    assert_bf16_rel(o1, ro)
    assert_state(h1, rh)


@pytest.mark.parametrize("lens,hk,hv", [([130, 1, 64, 250], 2, 4), ([300, 64], 1, 4),
                                         ([700], 4, 4), ([129, 63], 2, 16)])
def test_chunk_subops_pipeline(lens, hk, hv):
    """cumsum -> kkt -> solve_tril -> w/u -> fwd_h -> fwd_o on the GPU, each
    stage against the oracle's same stage, and the composition against the
    fused op."""
    inp = workloads.chunk_config3(hk=hk, hv=hv, lengths=lens, seed=8)
    q, k, v, g, beta, h0, cu = (inp[n] for n in ("q", "k", "v", "g", "beta", "initial_state",
                                                 "cu_seqlens"))
    gc = ops.npu_chunk_local_cumsum(_to(g), 64, _to(cu))
    rgc = oracle.chunk_local_cumsum(g, 64, cu)
    assert_fp32(gc, rgc)
    A = ops.npu_chunk_scaled_dot_kkt_fwd(_to(k), _to(beta), gc, 64, _to(cu))
    rA = oracle.chunk_scaled_dot_kkt_fwd(k, beta, rgc, 64, cu)
    assert_fp32(A, rA)
    Ai = ops.npu_solve_tril(A, 64, _to(cu), torch.float32)
    rAi = oracle.solve_tril(rA, 64, cu)
    assert rel_fro(Ai, rAi) < 1e-3
    w, u = ops.npu_recompute_w_u_fwd(_to(k), _to(v), _to(beta), gc, Ai, _to(cu))
    rw, ru = oracle.recompute_w_u_fwd(k, v, beta, rgc, rAi, cu)
    assert_bf16(w, rw)
    assert_bf16(u, ru)
    h, vn, ht = ops.npu_chunk_gated_delta_rule_fwd_h(_to(k), w, u, gc, _to(h0), True, 64, True,
                                                     _to(cu))
    rh, rvn, rht = oracle.chunk_gated_delta_rule_fwd_h(k, w.cpu(), u.cpu(), rgc, h0, True, 64, True,
                                                       cu)
    assert h.shape == rh.shape
    assert_bf16(h, rh)
    assert_bf16(vn, rvn)
    assert_state(ht, rht)
    o = ops.npu_chunk_fwd_o(_to(q), _to(k), vn, h, gc, 128 ** -0.5, 64, _to(cu))
    ro = oracle.chunk_fwd_o(q, k, vn.cpu(), h.cpu(), rgc, 128 ** -0.5, 64, cu)
    assert_bf16_rel(o, ro)
    of, _ = ops.npu_chunk_gated_delta_rule(_to(q), _to(k), _to(v), _to(g), _to(beta), None,
                                           _to(h0), True, _to(cu))
    assert_bf16(o, of, tol=2 * BF16_MAXABS)


@pytest.mark.parametrize("case", golden("fused_recurrent_gated_delta_rule"), ids=lambda c: c["name"])
def test_recurrent_golden(case):
    a = case["args"]
    st = a["initial_state"].clone().to(DEV)
    idx = torch.arange(st.shape[0], dtype=torch.int32, device=DEV)
    o, ht = ops.npu_fused_recurrent_gated_delta_rule(
        _to(a["q"]), _to(a["k"]), _to(a["v"]), _to(a["g"]), _to(a["beta"]), a["scale"], st, True,
        _to(a["cu_seqlens"]), idx, None, a["use_qk_l2norm_in_kernel"])
    assert ht.data_ptr() == st.data_ptr()
    st_ref = a["initial_state"].clone()
    ro, _ = oracle.fused_recurrent_gated_delta_rule(a["q"], a["k"], a["v"], a["g"], a["beta"],
                                                    a["scale"], st_ref, True, a["cu_seqlens"],
                                                    idx.cpu(), a["use_qk_l2norm_in_kernel"])
    assert_bf16_rel(o, ro)
    assert_state(st, st_ref)


def test_recurrent_config4_inplace():
    w = workloads.decode_config4()
    st = w["state"].clone().to(DEV)
    o, ht = ops.npu_fused_recurrent_gated_delta_rule(
        _to(w["q"]), _to(w["k"]), _to(w["v"]), _to(w["g"]), _to(w["beta"]), None, st, True,
        _to(w["cu_seqlens"]), _to(w["ssm_state_indices"]), None, True)
    st_ref = w["state"].clone()
    ro, _ = oracle.fused_recurrent_gated_delta_rule(w["q"], w["k"], w["v"], w["g"], w["beta"], None,
                                                    st_ref, True, w["cu_seqlens"],
                                                    w["ssm_state_indices"], True)
    assert_bf16_rel(o, ro)
    assert_state(st, st_ref)


def test_recurrent_slots_not_inplace_multitoken():
    g = torch.Generator().manual_seed(5)
    N, H, HV, D = 3, 2, 4, 128
    lens = [2, 5, 1]
    T = sum(lens)
    q = torch.randn(1, T, H, D, generator=g).to(torch.bfloat16)
    k = torch.randn(1, T, H, D, generator=g).to(torch.bfloat16)
    v = torch.randn(1, T, HV, D, generator=g).to(torch.bfloat16)
    gate = F.logsigmoid(torch.randn(1, T, HV, generator=g))
    beta = torch.sigmoid(torch.randn(1, T, HV, generator=g))
    pool = torch.randn(7, HV, D, D, generator=g)
    slots = torch.tensor([5, 0, 3], dtype=torch.int32)
    cu = torch.tensor([0, 2, 7, 8], dtype=torch.int32)
    pool_d = pool.clone().to(DEV)
    o, fin = ops.npu_fused_recurrent_gated_delta_rule(_to(q), _to(k), _to(v), _to(gate), _to(beta),
                                                      0.3, pool_d, False, _to(cu), _to(slots),
                                                      None, True)
    assert torch.equal(pool_d.cpu(), pool)  # not in place: pool untouched
    ro, rfin = oracle.fused_recurrent_gated_delta_rule(q, k, v, gate, beta, 0.3, pool.clone(),
                                                       False, cu, slots, True)
    assert_bf16_rel(o, ro)
    assert_state(fin, rfin)


# ------------------------------------------------------ speculative decoding
@pytest.mark.parametrize("case", golden("fused_recurrent_spec"), ids=lambda c: c["name"])
def test_recurrent_spec_golden(case):
    a = case["args"]
    st = a["initial_state"].clone().to(DEV)
    o, ht = ops.npu_fused_recurrent_gated_delta_rule(
        _to(a["q"]), _to(a["k"]), _to(a["v"]), _to(a["g"]), _to(a["beta"]), a["scale"], st, True,
        _to(a["cu_seqlens"]), _to(a["ssm_state_indices"]), _to(a["num_accepted_tokens"]),
        a["use_qk_l2norm_in_kernel"])
    assert ht.data_ptr() == st.data_ptr()
    per_token = st[a["ssm_state_indices"].reshape(-1).long().to(DEV)]
    # the reference test's bounds against its torch path
    torch.testing.assert_close(o.cpu().float(), case["out"]["o"].reshape(o.shape).float(),
                               rtol=5e-3, atol=1e-2)
    torch.testing.assert_close(per_token.cpu(), case["out"]["token_states"], rtol=5e-2, atol=1e-2)
    st_ref = a["initial_state"].clone()
    ro, _ = oracle.fused_recurrent_gated_delta_rule(
        a["q"], a["k"], a["v"], a["g"], a["beta"], a["scale"], st_ref, True, a["cu_seqlens"],
        a["ssm_state_indices"], a["use_qk_l2norm_in_kernel"], a["num_accepted_tokens"])
    assert_bf16_rel(o, ro)
    assert_state(st, st_ref)


def _spec_inputs(N, T, H, HV, D, slots, seed):
    g0 = torch.Generator().manual_seed(seed)
    return dict(
        q=torch.randn(1, N * T, H, D, generator=g0).to(torch.bfloat16),
        k=torch.randn(1, N * T, H, D, generator=g0).to(torch.bfloat16),
        v=torch.randn(1, N * T, HV, D, generator=g0).to(torch.bfloat16),
        g=F.logsigmoid(torch.rand(1, N * T, HV, generator=g0)),
        beta=torch.sigmoid(torch.rand(1, N * T, HV, generator=g0)),
        h0=torch.randn(slots, HV, D, D, generator=g0))


# the reference's spec test head pairs (test_fused_recurrent_gated_delta_rule.py:755-772)
@pytest.mark.parametrize("H,HV", [(16, 16), (8, 8), (4, 4), (2, 2), (16, 32), (8, 16), (4, 8),
                                  (2, 4), (16, 48), (8, 24), (4, 12), (2, 6), (16, 64), (8, 32),
                                  (4, 16), (2, 8), (1, 8)])
def test_recurrent_spec_shapes(H, HV):
    N, T, D = 2, 3, 128
    d = _spec_inputs(N, T, H, HV, D, N * T, H + HV)
    idx = torch.arange(N * T, dtype=torch.int32).reshape(N, T)
    acc = torch.tensor([1, 2], dtype=torch.int32)
    cu = torch.arange(N + 1, dtype=torch.int32) * T
    st = d["h0"].clone().to(DEV)
    o, _ = ops.npu_fused_recurrent_gated_delta_rule(
        _to(d["q"]), _to(d["k"]), _to(d["v"]), _to(d["g"]), _to(d["beta"]), None, st, True,
        _to(cu), _to(idx), _to(acc), True)
    st_ref = d["h0"].clone()
    ro, _ = oracle.fused_recurrent_gated_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"],
                                                    None, st_ref, True, cu, idx, True, acc)
    assert_bf16_rel(o, ro)
    assert_state(st, st_ref)


@pytest.mark.parametrize("mode", ["plain_2d_inplace", "spec_1d", "spec_not_inplace", "spec_ragged"])
def test_recurrent_slot_tables(mode):
    """Per-token index tables outside speculative decoding, a flat [N] table
    under speculative decoding (read with token stride 1, as the reference
    kernel addresses it), speculative decoding into a separate state tensor,
    and ragged sequences with a negative (skipped) token slot."""
    N, T, H, HV, D = 3, 2, 1, 2, 64
    d = _spec_inputs(N, T, H, HV, D, 12, 77)
    cu = torch.arange(N + 1, dtype=torch.int32) * T
    acc = None
    inplace = True
    if mode == "plain_2d_inplace":
        idx = torch.tensor([[3, 7], [0, 5], [9, 1]], dtype=torch.int32)
    elif mode == "spec_1d":
        # one-token rows: a flat [N] table under speculative decoding reads
        # and writes entry n + t = n
        idx = torch.tensor([4, 6, 8], dtype=torch.int32)
        acc = torch.tensor([1, 1, 1], dtype=torch.int32)
        cu = torch.tensor([0, 1, 2, 3], dtype=torch.int32)
    elif mode == "spec_not_inplace":
        # the per-token stores land in the new [N, HV, K, V] tensor; each
        # sequence keeps to its own row so no two sequences write one slot
        idx = torch.tensor([[0, 0], [1, 1], [2, 2]], dtype=torch.int32)
        acc = torch.tensor([2, 1, 1], dtype=torch.int32)
        inplace = False
    else:
        idx = torch.tensor([[2, -1, 4], [5, 6, 7], [8, 9, 10]], dtype=torch.int32)
        acc = torch.tensor([1, 2, 1], dtype=torch.int32)
        cu = torch.tensor([0, 3, 4, 6], dtype=torch.int32)
    st = d["h0"].clone().to(DEV)
    o, fin = ops.npu_fused_recurrent_gated_delta_rule(
        _to(d["q"]), _to(d["k"]), _to(d["v"]), _to(d["g"]), _to(d["beta"]), 0.3, st, inplace,
        _to(cu), _to(idx), _to(acc), True)
    st_ref = d["h0"].clone()
    ro, rfin = oracle.fused_recurrent_gated_delta_rule(d["q"], d["k"], d["v"], d["g"], d["beta"],
                                                       0.3, st_ref, inplace, cu, idx, True, acc)
    n_tok = int(cu[-1])
    assert_bf16(o[:, :n_tok], ro[:, :n_tok])
    assert_state(st, st_ref)
    if not inplace:
        assert_state(fin, rfin)
        assert torch.equal(st.cpu(), d["h0"])


def test_recurrent_spec_via_cpp():
    from torch_npu_ops_b200 import _C as C
    N, T, H, HV, D = 2, 3, 2, 4, 128
    d = _spec_inputs(N, T, H, HV, D, N * T, 5)
    idx = _to(torch.arange(N * T, dtype=torch.int32).reshape(N, T))
    acc = _to(torch.tensor([2, 1], dtype=torch.int32))
    cu = _to(torch.arange(N + 1, dtype=torch.int32) * T)
    s1, s2 = d["h0"].clone().to(DEV), d["h0"].clone().to(DEV)
    args = [_to(d[n]) for n in ("q", "k", "v", "g", "beta")]
    o1, _ = C.npu_fused_recurrent_gated_delta_rule(*args, None, s1, True, cu, idx, acc, True)
    o2, _ = ops.npu_fused_recurrent_gated_delta_rule(*args, None, s2, True, cu, idx, acc, True)
    assert torch.equal(o1, o2) and torch.equal(s1, s2)
    assert C.kernel_entry_point("fused_recurrent_gated_delta_rule_spec_fwd_kernel") == \
        "xops_fused_recurrent_gated_delta_rule"


# ------------------------------------------------- gating fused into the rule
def _gating_inputs(T, H, adt, bdt, seed):
    g = torch.Generator().manual_seed(seed)
    A_log = torch.rand(H, generator=g) * 2.7
    a = torch.randn(T, H, generator=g).to(adt)
    b = torch.randn(T, H, generator=g).to(bdt)
    dt_bias = torch.rand(H, generator=g)
    return A_log, a, b, dt_bias


@pytest.mark.parametrize("lens,hk,hv,adt,bdt,l2", [
    ([1, 63, 64, 65, 0, 129, 700], 4, 8, torch.bfloat16, torch.bfloat16, False),  # pair prep
    ([900, 33], 2, 8, torch.float16, torch.float32, True),                          # per-head prep
    ([4096], 16, 32, torch.float32, torch.bfloat16, False),                         # cfg3 heads
    ([8192], 1, 2, torch.bfloat16, torch.bfloat16, False),                          # segmented chain
])
def test_chunk_gated_equals_gating_then_rule(lens, hk, hv, adt, bdt, l2):
    """npu_fused_gdn_gating followed by npu_chunk_gated_delta_rule and the
    fused-gating entry give the same bits; both match the composed oracle."""
    inp = workloads.chunk_config3(hk=hk, hv=hv, lengths=lens, seed=11)
    T = sum(lens)
    A_log, a, b, dt_bias = _gating_inputs(T, hv, adt, bdt, seed=len(lens) + hv)
    g, beta = ops.npu_fused_gdn_gating(_to(A_log), _to(a), _to(b), _to(dt_bias))
    o1, h1 = ops.npu_chunk_gated_delta_rule(
        _to(inp["q"]), _to(inp["k"]), _to(inp["v"]), g, beta.float(), None,
        _to(inp["initial_state"]), True, _to(inp["cu_seqlens"]), False, l2)
    o2, h2 = ops.chunk_gated_delta_rule_gated(
        _to(inp["q"]), _to(inp["k"]), _to(inp["v"]), _to(A_log), _to(a[None]), _to(b), _to(dt_bias),
        None, _to(inp["initial_state"]), True, _to(inp["cu_seqlens"]), l2)
    torch.cuda.synchronize()
    assert torch.equal(o1, o2) and torch.equal(h1, h2)
    rg, rb = oracle.fused_gdn_gating(A_log, a, b, dt_bias)
    rb = rb.to(bdt).float()  # beta as the gating operator stores it (b's dtype)
    ro, rh = oracle.chunk_gated_delta_rule(inp["q"], inp["k"], inp["v"], rg, rb, None,
                                           inp["initial_state"], True, inp["cu_seqlens"], l2)
    assert_bf16_rel(o2.cpu(), ro)
    assert_state(h2.cpu(), rh)


def test_gdn_prefill_gating_option():
    """The layer pipeline with the gating folded into the rule equals the
    pipeline fed by npu_fused_gdn_gating, bit for bit (a head shard of the
    bench configuration, 8192 tokens)."""
    from torch_npu_ops_b200.pipeline import gdn_prefill
    w = workloads.long_config5_shard(0, 8, T=8192)
    hv, hk = w["heads"][1] - w["heads"][0], w["k_heads"][1] - w["k_heads"][0]
    T = w["T"]
    A_log, a, b, dt_bias = _gating_inputs(T, hv, torch.bfloat16, torch.bfloat16, seed=5)
    g, beta = ops.npu_fused_gdn_gating(_to(A_log), _to(a), _to(b), _to(dt_bias))
    outs = []
    for gating in (None, (_to(A_log), _to(a), _to(b), _to(dt_bias))):
        st = torch.zeros(1, w["x"].shape[1], 3, dtype=torch.bfloat16, device=DEV)
        gg, bb = (g, beta.float()) if gating is None else (None, None)
        outs.append(gdn_prefill(_to(w["x"]), st, _to(w["weight"]), _to(w["bias"]), gg, bb,
                                _to(w["initial_state"]), _to(w["z"]), _to(w["norm_w"]), hk, hv,
                                gating=gating, fuse_norm=False))
    torch.cuda.synchronize()
    for x1, x2 in zip(*outs):
        assert torch.equal(x1, x2)


@pytest.mark.parametrize("T,hk,hv,lens", [
    (8192, 2, 4, None),             # a head shard of the bench configuration: one segment plan
    (65536, 2, 4, None),            # the 8-GPU shard: segmented chain (phase 1 + phase 3 outputs)
    (3000, 4, 8, [1000, 64, 1936]),  # varlen, chunks cut by sequence ends
    (4160, 4, 8, [77, 4000, 83]),   # short sequences and partial 16-token row groups
])
def test_out_norm_fused_equals_rule_then_norm(T, hk, hv, lens):
    """The gated RMSNorm inside the chain's output epilogue
    (chunk_gated_delta_rule_out_norm) equals npu_chunk_gated_delta_rule
    followed by layer_norm_fwd (its streaming kernel, which every shape
    here takes) bit for bit: y, the final state, and o when it is asked
    for; asking for o leaves y unchanged."""
    from torch_npu_ops_b200.pipeline import gdn_prefill
    g = torch.Generator().manual_seed(T + 7 * hv)
    d = 128
    C = (2 * hk + hv) * d
    x = torch.randn(T, C, generator=g).to(torch.bfloat16)
    cw = (0.5 * torch.randn(C, 4, generator=g)).to(torch.bfloat16)
    cb = (0.5 * torch.randn(C, generator=g)).to(torch.bfloat16)
    gate, beta = workloads.gdn_gates(T, hv, g)
    lens = lens or [T]
    assert sum(lens) == T
    N = len(lens)
    h0 = 0.02 * torch.randn(N, hv, d, d, generator=g)
    z = torch.randn(T, hv, d, generator=g).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    qsl = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=DEV)
    outs = []
    for fuse, ret_o in ((True, False), (True, True), (False, True)):
        st = torch.zeros(N, C, 3, dtype=torch.bfloat16, device=DEV)
        outs.append(gdn_prefill(_to(x), st, _to(cw), _to(cb), _to(gate)[None], _to(beta)[None],
                                _to(h0), _to(z), _to(nw), hk, hv, query_start_loc=qsl,
                                return_o=ret_o, fuse_norm=fuse))
    torch.cuda.synchronize()
    assert _lib_errors() == 0
    (y0, o0, h0a, n0), (y1, o1, h1, n1), (y2, o2, h2, n2) = outs
    assert o0 is None
    assert torch.equal(y0, y2) and torch.equal(y1, y2)
    assert torch.equal(o1, o2)
    assert torch.equal(h0a, h2) and torch.equal(h1, h2)
    assert torch.equal(n0, n2), (n0.float() - n2.float()).abs().max().item()
    assert torch.equal(n1, n2)


def _lib_errors():
    from torch_npu_ops_b200 import _lib
    return _lib.load().xops_device_error_count()


@pytest.mark.parametrize("T,hk,hv,lens", [(8192, 2, 4, None), (3000, 4, 8, [1000, 64, 1936]),
                                          (4096, 2, 8, None)])
def test_gdn_layer_prefill_from_projections(T, hk, hv, lens):
    """Conv, gating and gated norm read the un-split projections in place
    (the norm inside the rule's chain kernel); the results equal split ->
    conv -> gating -> rule -> norm bit for bit, and the rule's output
    matches the composed oracle."""
    from torch_npu_ops_b200.pipeline import gdn_layer_prefill, gdn_prefill
    g = torch.Generator().manual_seed(T + hv)
    d, r = 128, hv // hk
    mixed_qkvz = torch.randn(T, hk * (2 + 2 * r) * d, generator=g).to(torch.bfloat16)
    mixed_ba = torch.randn(T, hk * 2 * r, generator=g).to(torch.bfloat16)
    C = (2 * hk + hv) * d
    w = (0.5 * torch.randn(C, 4, generator=g)).to(torch.bfloat16)
    cb = (0.5 * torch.randn(C, generator=g)).to(torch.bfloat16)
    A_log = torch.rand(hv, generator=g) * 2.7
    dt_bias = torch.rand(hv, generator=g)
    nw = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    lens = lens or [T]
    N = len(lens)
    h0 = 0.02 * torch.randn(N, hv, d, d, generator=g)
    qsl = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32, device=DEV)
    st1 = torch.zeros(N, C, 3, dtype=torch.bfloat16, device=DEV)
    st2 = st1.clone()
    fused = gdn_layer_prefill(_to(mixed_qkvz), _to(mixed_ba), st1, _to(w), _to(cb), _to(A_log),
                              _to(dt_bias), _to(h0), _to(nw), hk, hv, query_start_loc=qsl,
                              return_o=True)
    # the layer's own call (o not written) gives the same normalised output
    st3 = torch.zeros(N, C, 3, dtype=torch.bfloat16, device=DEV)
    lean = gdn_layer_prefill(_to(mixed_qkvz), _to(mixed_ba), st3, _to(w), _to(cb), _to(A_log),
                             _to(dt_bias), _to(h0), _to(nw), hk, hv, query_start_loc=qsl)
    assert lean[1] is None
    mixed_qkv, z, b, a = ops.npu_fused_qkvzba_split_reshape_cat(_to(mixed_qkvz), _to(mixed_ba), hk,
                                                                hv, d, d)
    gt, beta = ops.npu_fused_gdn_gating(_to(A_log), a, b, _to(dt_bias))
    plain = gdn_prefill(mixed_qkv, st2, _to(w), _to(cb), gt, beta.float(), _to(h0), z, _to(nw), hk,
                        hv, query_start_loc=qsl, fuse_norm=False)
    torch.cuda.synchronize()
    for x1, x2 in zip(fused, plain):
        assert torch.equal(x1, x2)
    assert torch.equal(st1, st2)
    assert torch.equal(lean[3], plain[3]) and torch.equal(lean[2], plain[2])
    # the rule's output against the oracle, from the conv output both paths share
    y = fused[0].cpu()
    q = y[:, : hk * d].view(1, T, hk, d)
    k = y[:, hk * d: 2 * hk * d].view(1, T, hk, d)
    v = y[:, 2 * hk * d:].view(1, T, hv, d)
    rg, rb = oracle.fused_gdn_gating(A_log, a.cpu(), b.cpu(), dt_bias)
    ro, rh = oracle.chunk_gated_delta_rule(q, k, v, rg, rb.to(torch.bfloat16).float(), None, h0, True,
                                           qsl.cpu() if N > 1 else None, False)
    assert_bf16_rel(fused[1].cpu(), ro)
    assert_state(fused[2].cpu(), rh)
