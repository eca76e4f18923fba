"""Generate the golden fixtures in this directory from the reference's OWN
torch-native implementations.

Runs only where the reference project is importable: ``--ref-root`` names its
checkout (the directory holding ``triton_npu/``); the fixtures it writes
travel with the repository, so nothing else ever needs the reference at run
time.

The reference's test modules import ``torch_npu`` and Ascend-only Triton
extensions at module level; two empty stand-in modules are registered in
``sys.modules`` so those imports succeed on a CPU-only machine.  Only the
pure-torch reference functions are called -- never a Triton kernel.

Fixtures: ``<op>.pt`` = ``{"cases": [{"name", "args": {...}, "out": {...}}]}``.
Usage: ``python tests/golden/make_golden.py --ref-root DIR [--only ...]``.
"""

import argparse
import importlib
import os
import sys
import types

import torch
import torch.nn.functional as F

HERE = os.path.dirname(os.path.abspath(__file__))


def _import_reference(ref_root):
    sys.dont_write_bytecode = True
    sys.modules.setdefault("torch_npu", types.ModuleType("torch_npu"))
    cann = types.ModuleType("triton.language.extra.cann")
    ext = types.ModuleType("triton.language.extra.cann.extension")
    ext.extract_slice = lambda *a, **k: None
    ext.insert_slice = lambda *a, **k: None
    cann.extension = ext
    sys.modules["triton.language.extra.cann"] = cann
    sys.modules["triton.language.extra.cann.extension"] = ext
    sys.path.insert(0, os.path.join(ref_root, "triton_npu", "triton_src"))
    names = ["test_chunk_gated_delta_rule", "test_fused_recurrent_gated_delta_rule",
             "test_layernorm_fwd", "test_causal_conv1d_update",
             "test_causal_conv1d_update_v2", "test_split_rmsnorm_rope", "test_l2norm",
             "test_fused_gdn_gating", "test_fused_sigmoid_gating_delta_rule_update",
             "test_fused_qkvzba_split_reshape", "test_rope_inplace"]
    return {n: importlib.import_module(n) for n in names}


def _save(name, cases):
    path = os.path.join(HERE, name + ".pt")
    torch.save({"cases": cases}, path)
    print(f"wrote {path}: {len(cases)} cases, {os.path.getsize(path) / 1024:.0f} KB")


def gen_layernorm(m):
    ref = m["test_layernorm_fwd"]._golden_ref
    cases = []
    specs = [  # (name, M, N, group, bias, z, before, rms, dtype)
        ("ln_bias_f32", 16, 128, 128, True, False, True, False, torch.float32),
        ("rms_nobias_f32", 16, 128, 128, False, False, True, True, torch.float32),
        ("rms_z_before_f32", 16, 256, 128, False, True, True, True, torch.float32),
        ("rms_z_after_f32", 16, 256, 128, False, True, False, True, torch.float32),
        ("ln_z_bias_f32", 12, 256, 64, True, True, True, False, torch.float32),
        ("ln_bias_big_group_f32", 8, 2048, 2048, True, False, True, False, torch.float32),
        ("rms_z_before_bf16", 64, 128, 128, False, True, True, True, torch.bfloat16),
        ("ln_bias_big_group_bf16", 8, 2048, 2048, True, False, True, False, torch.bfloat16),
        ("rms_z_after_bias_bf16", 10, 384, 128, True, True, False, True, torch.bfloat16),
    ]
    g = torch.Generator().manual_seed(42)
    for name, M, N, G, bias, z, before, rms, dt in specs:
        x = torch.randn(M, N, generator=g).to(dt)
        w = (1 + 0.1 * torch.randn(N, generator=g)).to(dt)
        b = (0.1 * torch.randn(N, generator=g)).to(dt) if bias else None
        zz = torch.randn(M, N, generator=g).to(dt) if z else None
        y = ref(x, w, b, 1e-6, z=zz, group_size=G, norm_before_gate=before, is_rms_norm=rms)
        cases.append({"name": name, "args": {"x": x, "weight": w, "bias": b, "z": zz,
                      "eps": 1e-6, "group_size": G, "norm_before_gate": before,
                      "is_rms_norm": rms}, "out": {"y": y}})
    _save("layer_norm_fwd", cases)


def gen_l2norm(m):
    ref = m["test_l2norm"].l2norm_ref
    cases = []
    g = torch.Generator().manual_seed(0)
    for shape in [(1, 31, 4, 64), (1, 31, 4, 128), (2, 17, 3, 192)]:
        for dt in (torch.bfloat16, torch.float32):
            x = torch.randn(*shape, generator=g).to(dt)
            cases.append({"name": f"{shape}_{dt}", "args": {"x": x, "eps": 1e-6},
                          "out": {"y": ref(x, 1e-6)}})
    _save("l2norm", cases)


def gen_rope(m):
    mod = m["test_split_rmsnorm_rope"]
    cases = []
    g = torch.Generator().manual_seed(0)
    # full-width rotary: the reference function as is
    for (T, qh, kvh, hd, bias) in [(16, 4, 1, 128, False), (9, 8, 2, 64, True)]:
        qkv = torch.randn(T, (qh + 2 * kvh) * hd, generator=g)
        qw = 1 + 0.1 * torch.randn(hd, generator=g)
        kw = 1 + 0.1 * torch.randn(hd, generator=g)
        qb = 0.1 * torch.randn(hd, generator=g)
        kb = 0.1 * torch.randn(hd, generator=g)
        sin = torch.randn(T, hd, generator=g)
        cos = torch.randn(T, hd, generator=g)
        q, k, v = mod.split_rmsnorm_rope_ref(qkv, sin, cos, qw, kw, qh * hd, kvh * hd, hd,
                                             1e-6, q_bias=qb, k_bias=kb, bias=bias)
        cases.append({"name": f"full_T{T}_qh{qh}_kvh{kvh}_hd{hd}_b{int(bias)}",
                      "args": {"input": qkv, "sin": sin, "cos": cos, "q_weight": qw,
                               "k_weight": kw, "q_hidden_size": qh * hd,
                               "kv_hidden_size": kvh * hd, "head_dim": hd, "eps": 1e-6,
                               "q_bias": qb, "k_bias": kb, "bias": bias},
                      "out": {"q": q, "k": k, "v": v}})
    # partial rotary (rotary_dim < head_dim): the reference's rms_norm followed by
    # its custom_rope applied to the first rotary_dim dims (composition of the
    # reference's own pieces; the pass-through convention is an assumption)
    T, qh, kvh, hd, rd = 12, 4, 1, 256, 64
    qkv = torch.randn(T, (qh + 2 * kvh) * hd, generator=g)
    qw = 1 + 0.1 * torch.randn(hd, generator=g)
    kw = 1 + 0.1 * torch.randn(hd, generator=g)
    pos = torch.arange(T, dtype=torch.float64)
    inv = 1.0 / (1e7 ** (torch.arange(0, rd, 2, dtype=torch.float64) / rd))
    ang = torch.cat([pos[:, None] * inv, pos[:, None] * inv], -1)
    sin, cos = torch.sin(ang).float(), torch.cos(ang).float()
    qn = mod.rms_norm(qkv[:, : qh * hd].reshape(-1, hd), qw, 1e-6).reshape(T, 1, qh, hd)
    kn = mod.rms_norm(qkv[:, qh * hd:(qh + kvh) * hd].reshape(-1, hd), kw, 1e-6).reshape(T, 1, kvh, hd)
    qr, kr = mod.custom_rope(qn[..., :rd].contiguous(), kn[..., :rd].contiguous(), sin, cos)
    q = torch.cat([qr, qn[..., rd:]], -1).reshape(T, -1)
    k = torch.cat([kr, kn[..., rd:]], -1).reshape(T, -1)
    v = qkv[:, (qh + kvh) * hd:]
    cases.append({"name": "partial_rd64_hd256", "args": {
        "input": qkv, "sin": sin, "cos": cos, "q_weight": qw, "k_weight": kw,
        "q_hidden_size": qh * hd, "kv_hidden_size": kvh * hd, "head_dim": hd, "eps": 1e-6,
        "q_bias": None, "k_bias": None, "bias": False}, "out": {"q": q, "k": k, "v": v}})
    _save("split_rmsnorm_rope", cases)


def gen_conv(m):
    ref1 = m["test_causal_conv1d_update"].causal_conv1d_update_ref
    ref2 = m["test_causal_conv1d_update_v2"].causal_conv1d_update_ref_v2
    cases = []
    g = torch.Generator().manual_seed(7)
    # decode (seqlen 1) and short multi-token update, in place state
    for (B, dim, L, width, bias, dt) in [(4, 64, 1, 4, True, torch.float32),
                                         (3, 96, 1, 4, False, torch.float32),
                                         (5, 64, 1, 4, True, torch.bfloat16),
                                         (2, 32, 3, 4, True, torch.float32)]:
        x = torch.randn(B, dim, L, generator=g).to(dt)
        st = torch.randn(B, dim, width - 1, generator=g).to(dt)
        w = (0.5 * torch.randn(dim, width, generator=g)).to(dt)
        b = (0.5 * torch.randn(dim, generator=g)).to(dt) if bias else None
        st_out = st.clone()
        y = ref1(x.clone(), st_out, w, b, activation="silu")
        cases.append({"name": f"update_B{B}_d{dim}_L{L}_{dt}", "kind": "update",
                      "args": {"x": x, "conv_state": st, "weight": w, "bias": b},
                      "out": {"y": y, "conv_state": st_out}})
    # varlen prefill, one reference call per sequence (max_query_len = len)
    for (lens, dim, dt, zero_state) in [([5, 1, 17, 3], 64, torch.float32, False),
                                       ([64, 9, 130], 128, torch.float32, True),
                                       ([12, 40], 64, torch.bfloat16, False)]:
        width = 4
        T = sum(lens)
        x = torch.randn(T, dim, generator=g).to(dt)
        st = (torch.zeros(len(lens), dim, width - 1) if zero_state
              else torch.randn(len(lens), dim, width - 1, generator=g)).to(dt)
        w = (0.5 * torch.randn(dim, width, generator=g)).to(dt)
        b = (0.5 * torch.randn(dim, generator=g)).to(dt)
        qsl = torch.tensor([0] + list(torch.cumsum(torch.tensor(lens), 0).tolist()), dtype=torch.int32)
        st_out = st.clone()
        y = torch.empty_like(x)
        for i, L in enumerate(lens):
            s, e = int(qsl[i]), int(qsl[i + 1])
            y[s:e] = ref2(x[s:e].contiguous(), st_out[i:i + 1], w, b, activation=True,
                          conv_state_indices=torch.tensor([0], dtype=torch.int32),
                          query_start_loc=torch.tensor([0, L], dtype=torch.int32),
                          max_query_len=L)
        cases.append({"name": f"varlen_{lens}_d{dim}_{dt}", "kind": "varlen",
                      "args": {"x": x, "conv_state": st, "weight": w, "bias": b,
                               "query_start_loc": qsl},
                      "out": {"y": y, "conv_state": st_out}})
    _save("causal_conv1d", cases)


def gen_chunk(m):
    mod = m["test_chunk_gated_delta_rule"]
    cases = []
    # the reference's own pytest case (seed 1234, 31 tokens, 4 -> 8 heads)
    torch.manual_seed(1234)
    q = torch.randn(1, 31, 4, 128, dtype=torch.bfloat16)
    k = torch.randn(1, 31, 4, 128, dtype=torch.bfloat16)
    v = torch.randn(1, 31, 8, 128, dtype=torch.bfloat16)
    g = F.logsigmoid(torch.randn(1, 31, 8, dtype=torch.float32))
    beta = torch.sigmoid(torch.randn(1, 31, 8, dtype=torch.float32)).to(torch.bfloat16)
    h0 = torch.randn(1, 8, 128, 128, dtype=torch.bfloat16)
    cu = torch.tensor([0, 31], dtype=torch.int32)
    o, ht = mod.chunk_gated_delta_rule_ref(q, k, v, g, beta, initial_state=h0,
                                           output_final_state=True, cu_seqlens=cu,
                                           use_qk_l2norm_in_kernel=True)
    cases.append({"name": "ref_pytest_seed1234", "args": {
        "q": q, "k": k, "v": v, "g": g, "beta": beta, "initial_state": h0,
        "cu_seqlens": cu, "use_qk_l2norm_in_kernel": True},
        "out": {"o": o, "final_state": ht}})
    # varlen, grouped heads, ragged tails (65, 1, 130 tokens), GDN-style gates
    gen = torch.Generator().manual_seed(3)
    lens = [65, 1, 130]
    T = sum(lens)
    q = F.normalize(torch.randn(1, T, 1, 128, generator=gen), dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(1, T, 1, 128, generator=gen), dim=-1).to(torch.bfloat16)
    v = torch.randn(1, T, 2, 128, generator=gen).to(torch.bfloat16)
    a_log = torch.rand(2, generator=gen) * 2.7
    dt_b = torch.rand(2, generator=gen)
    g = -torch.exp(a_log) * F.softplus(torch.randn(1, T, 2, generator=gen) + dt_b)
    beta = torch.sigmoid(torch.randn(1, T, 2, generator=gen))
    h0 = 0.02 * torch.randn(3, 2, 128, 128, generator=gen)
    cu = torch.tensor([0, 65, 66, 196], dtype=torch.int32)
    o, ht = mod.chunk_gated_delta_rule_ref(q, k, v, g, beta, initial_state=h0,
                                           output_final_state=True, cu_seqlens=cu)
    cases.append({"name": "varlen_65_1_130_gqa", "args": {
        "q": q, "k": k, "v": v, "g": g, "beta": beta, "initial_state": h0,
        "cu_seqlens": cu, "use_qk_l2norm_in_kernel": False},
        "out": {"o": o, "final_state": ht}})
    # small head dim, no initial state (oracle-only pin)
    gen = torch.Generator().manual_seed(5)
    q = torch.randn(1, 100, 2, 32, generator=gen)
    k = torch.randn(1, 100, 2, 32, generator=gen)
    v = torch.randn(1, 100, 4, 16, generator=gen)
    g = F.logsigmoid(torch.randn(1, 100, 4, generator=gen))
    beta = torch.sigmoid(torch.randn(1, 100, 4, generator=gen))
    cu = torch.tensor([0, 37, 100], dtype=torch.int32)
    o, ht = mod.chunk_gated_delta_rule_ref(q, k, v, g, beta, output_final_state=True,
                                           cu_seqlens=cu, use_qk_l2norm_in_kernel=True)
    cases.append({"name": "small_dims_no_h0", "args": {
        "q": q, "k": k, "v": v, "g": g, "beta": beta, "initial_state": None,
        "cu_seqlens": cu, "use_qk_l2norm_in_kernel": True},
        "out": {"o": o, "final_state": ht}})
    _save("chunk_gated_delta_rule", cases)


def gen_recurrent(m):
    mod = m["test_fused_recurrent_gated_delta_rule"]
    from einops import repeat
    cases = []
    for (B, T, H, HV, D, scale, gln) in [(2, 1, 1, 2, 128, 0.5, 0.1), (3, 1, 2, 4, 64, 0.2, 1.0),
                                         (2, 3, 1, 2, 64, 0.3, 1.0)]:
        torch.manual_seed(42)
        q = torch.randn(B, T, H, D, dtype=torch.bfloat16)
        k = torch.randn(B, T, H, D, dtype=torch.bfloat16)
        v = torch.randn(B, T, HV, D, dtype=torch.bfloat16)
        beta = torch.rand(B, T, HV, dtype=torch.bfloat16).sigmoid()
        g = F.logsigmoid(torch.rand(B, T, HV, dtype=torch.float32)) / gln
        h0 = torch.randn(B, HV, D, D, dtype=torch.float32)
        outs, hts = [], []
        for i in range(B):
            qn = F.normalize(repeat(q[i:i + 1], "b t h d -> b t (h g) d", g=HV // H), p=2,
                             dim=-1, eps=1e-6).to(torch.bfloat16)
            kn = F.normalize(repeat(k[i:i + 1], "b t h d -> b t (h g) d", g=HV // H), p=2,
                             dim=-1, eps=1e-6).to(torch.bfloat16)
            o_i, ht_i = mod.recurrent_gated_delta_rule_ref(
                q=qn, k=kn, v=v[i:i + 1], beta=beta[i:i + 1], g=g[i:i + 1], scale=scale,
                initial_state=h0[i:i + 1].clone(), output_final_state=True)
            outs.append(o_i)
            hts.append(ht_i)
        cases.append({"name": f"B{B}_T{T}_H{H}_HV{HV}_D{D}", "args": {
            "q": q.reshape(1, B * T, H, D), "k": k.reshape(1, B * T, H, D),
            "v": v.reshape(1, B * T, HV, D), "g": g.reshape(1, B * T, HV),
            "beta": beta.reshape(1, B * T, HV), "scale": scale, "initial_state": h0,
            "cu_seqlens": torch.arange(B + 1, dtype=torch.int32) * T,
            "use_qk_l2norm_in_kernel": True},
            "out": {"o": torch.cat(outs, 1), "final_state": torch.cat(hts, 0)}})
    _save("fused_recurrent_gated_delta_rule", cases)


def gen_recurrent_spec(m):
    """Speculative decoding: initial state from the accepted token's slot,
    every token's state stored to its own slot.  Built the way the
    reference's spec tests build their expectation
    (test_fused_recurrent_gated_delta_rule.py:872-983): the reference's
    torch recurrence one token at a time from the accepted slot's state."""
    mod = m["test_fused_recurrent_gated_delta_rule"]
    from einops import repeat
    cases = []
    for name, (N, T, H, HV, D, slots, idx, acc) in {
        "accepted_offsets": (3, 4, 1, 2, 64, 27,
                             [[2, 4, 6, 8], [11, 13, 15, 17], [20, 22, 24, 26]], [1, 2, 3]),
        "all_first": (2, 3, 1, 2, 64, 6, [[0, 1, 2], [3, 4, 5]], [1, 1]),
    }.items():
        torch.manual_seed(44)
        q = torch.randn(N, T, H, D, dtype=torch.bfloat16)
        k = torch.randn(N, T, H, D, dtype=torch.bfloat16)
        v = torch.randn(N, T, HV, D, dtype=torch.bfloat16)
        beta = torch.rand(N, T, HV, dtype=torch.bfloat16).sigmoid()
        g = F.logsigmoid(torch.rand(N, T, HV, dtype=torch.float32))
        h0 = torch.randn(slots, HV, D, D, dtype=torch.float32)
        idx_t = torch.tensor(idx, dtype=torch.int32)
        acc_t = torch.tensor(acc, dtype=torch.int32)
        outs, states = [], []
        for n in range(N):
            h = h0[int(idx_t[n, acc[n] - 1])].unsqueeze(0)
            qn = F.normalize(repeat(q[n:n + 1], "b t h d -> b t (h g) d", g=HV // H), p=2,
                             dim=-1, eps=1e-6).to(torch.bfloat16)
            kn = F.normalize(repeat(k[n:n + 1], "b t h d -> b t (h g) d", g=HV // H), p=2,
                             dim=-1, eps=1e-6).to(torch.bfloat16)
            for t in range(T):
                o_t, h = mod.recurrent_gated_delta_rule_ref(
                    q=qn[:, t:t + 1], k=kn[:, t:t + 1], v=v[n:n + 1, t:t + 1],
                    beta=beta[n:n + 1, t:t + 1], g=g[n:n + 1, t:t + 1], scale=0.5,
                    initial_state=h, output_final_state=True)
                outs.append(o_t)
                states.append(h.squeeze(0))
        cases.append({"name": name, "args": {
            "q": q.reshape(1, N * T, H, D), "k": k.reshape(1, N * T, H, D),
            "v": v.reshape(1, N * T, HV, D), "g": g.reshape(1, N * T, HV),
            "beta": beta.reshape(1, N * T, HV), "scale": 0.5, "initial_state": h0,
            "cu_seqlens": torch.arange(N + 1, dtype=torch.int32) * T,
            "ssm_state_indices": idx_t, "num_accepted_tokens": acc_t,
            "use_qk_l2norm_in_kernel": True},
            "out": {"o": torch.cat(outs, 1), "token_states": torch.stack(states, 0)}})
    _save("fused_recurrent_spec", cases)


def gen_conv_slots(m):
    """Speculative decoding and prefix-cache block tables of the v2 conv,
    in the shapes of the reference's own tests
    (test_causal_conv1d_update_v2.py:502-750), with equal lengths per call so
    the reference function's max_query_len window is each sequence's own."""
    ref = m["test_causal_conv1d_update_v2"].causal_conv1d_update_ref_v2
    cases = []
    g0 = torch.Generator().manual_seed(712)
    # spec decoding, [B, D, T] rows (the reference test at :712)
    for name, (batch, dim, width, seqlen, acc) in {
            "spec_w4_t2": (2, 256, 4, 2, [1, 2]),
            "spec_w3_t3": (3, 128, 3, 3, [3, 1, 2])}.items():
        x = torch.randn(batch, dim, seqlen, generator=g0).to(torch.bfloat16)
        st = torch.randn(batch, dim, width - 1 + seqlen - 1, generator=g0).to(torch.bfloat16)
        w = torch.randn(dim, width, generator=g0).to(torch.bfloat16)
        idx = torch.arange(batch, dtype=torch.int32)
        acc_t = torch.tensor(acc, dtype=torch.int32)
        st_ref = st.clone()
        out = ref(x, st_ref, w, activation="silu", conv_state_indices=idx,
                  num_accepted_tokens=acc_t)
        cases.append({"name": name, "args": {
            "x": x, "conv_state": st, "weight": w, "bias": None, "activation": True,
            "conv_state_indices": idx, "num_accepted_tokens": acc_t, "query_start_loc": None,
            "max_query_len": -1, "pad_slot_id": -1, "initial_state_idx": None,
            "block_idx_last_scheduled_token": None},
            "out": {"out": out, "conv_state": st_ref}})
    # prefix-cache block tables: read one line, write another; a padded row
    # (the reference tests at :502 and :602, equal lengths)
    for name, (dim, width, lens, idx, last, pad) in {
            "apc_decode": (256, 4, [1, 1, 1], [[0, 0], [1, 1], [2, 2]], [0, 0, 0], -1),
            "apc_move_pad_w5": (128, 5, [2, 0, 2], [[0, 1], [-7, -7], [2, 3]], [1, 0, 1], -7)}.items():
        total = sum(lens)
        x = torch.randn(total, dim, generator=g0).to(torch.bfloat16)
        st = torch.randn(4, dim, width - 1, generator=g0).to(torch.bfloat16)
        w = torch.randn(dim, width, generator=g0).to(torch.bfloat16)
        b = torch.zeros(dim).to(torch.bfloat16)
        qsl = torch.tensor([0] + list(torch.tensor(lens).cumsum(0)), dtype=torch.int32)
        idx_t = torch.tensor(idx, dtype=torch.int32)
        ini = torch.zeros(len(lens), dtype=torch.int32)
        last_t = torch.tensor(last, dtype=torch.int32)
        st_ref = st.clone()
        out = ref(x, st_ref, w, bias=b, activation="silu", conv_state_indices=idx_t,
                  query_start_loc=qsl, max_query_len=max(lens), pad_slot_id=pad,
                  block_idx_last_scheduled_token=last_t, initial_state_idx=ini)
        cases.append({"name": name, "args": {
            "x": x, "conv_state": st, "weight": w, "bias": b, "activation": True,
            "conv_state_indices": idx_t, "num_accepted_tokens": None, "query_start_loc": qsl,
            "max_query_len": max(lens), "pad_slot_id": pad, "initial_state_idx": ini,
            "block_idx_last_scheduled_token": last_t},
            "out": {"out": out, "conv_state": st_ref}})
    _save("causal_conv1d_slots", cases)


def gen_rope_inplace(m):
    ref = m["test_rope_inplace"].rope_ref
    cases = []
    # the reference test's (batch, head) list with hidden 512, rope_dim 64
    # (test_rope_inplace.py:100-112), plus 2D x and a 128-wide tail
    g0 = torch.Generator().manual_seed(100)
    for batch, head, hidden, rd in [(1, 8, 512, 64), (4, 8, 512, 64), (8, 1, 512, 64),
                                    (4, 0, 512, 64), (3, 4, 576, 128)]:
        shape = (batch, hidden) if head == 0 else (batch, head, hidden)
        x = torch.randn(*shape, generator=g0).to(torch.bfloat16)
        sin = torch.randn(batch, rd, generator=g0).to(torch.bfloat16)
        cos = torch.randn(batch, rd, generator=g0).to(torch.bfloat16)
        out = ref(x if head else x.unsqueeze(1), sin, cos, rd)
        cases.append({"name": f"b{batch}_h{head}_d{hidden}_r{rd}", "args": {
            "x": x, "sin": sin, "cos": cos, "rope_dim": rd},
            "out": {"x": out if head else out.squeeze(1)}})
    _save("rope_inplace", cases)


def gen_gating(m):
    ref = m["test_fused_gdn_gating"].torch_fused_gdn_gating
    cases = []
    # the reference test's head counts and token counts (test_fused_gdn_gating.py:95-97),
    # plus a prefill-sized row count and a saturated-softplus case
    for T, HV, dt in [(1, 1, torch.bfloat16), (4, 3, torch.bfloat16), (16, 32, torch.bfloat16),
                      (8, 48, torch.bfloat16), (1000, 32, torch.bfloat16),
                      (64, 16, torch.float32)]:
        g0 = torch.Generator().manual_seed(T * 100 + HV)
        A_log = torch.randn(HV, generator=g0)
        a = torch.randn(T, HV, generator=g0).to(dt)
        if dt == torch.float32:
            a = a * 15  # a + dt_bias crosses the softplus threshold (20)
        b = torch.randn(T, HV, generator=g0).to(dt)
        dt_bias = torch.ones(HV) if T < 1000 else torch.rand(HV, generator=g0)
        g, beta = ref(A_log, a, b, dt_bias)
        cases.append({"name": f"T{T}_HV{HV}_{str(dt)[6:]}", "args": {
            "A_log": A_log, "a": a, "b": b, "dt_bias": dt_bias, "beta": 1.0, "threshold": 20.0},
            "out": {"g": g[None], "beta": beta[None]}})
    _save("fused_gdn_gating", cases)


def gen_sigmoid_gating(m):
    ref = m["test_fused_sigmoid_gating_delta_rule_update"].torch_sigmoid_gating_delta_rule_update
    cases = []
    # (batch, T, H, HV, K, indices) -- small versions of the reference test's
    # head ratios (test_fused_sigmoid_gating_delta_rule_update.py:225-247; the
    # fp32 states keep fixtures small only at few heads), multi-token rows and
    # a negative slot (starts from zero, writes nothing back)
    for B, T, H, HV, K, idx in [(2, 1, 2, 4, 128, None), (2, 1, 1, 8, 64, None),
                                (3, 1, 2, 6, 64, None), (3, 3, 2, 4, 64, [2, -1, 0])]:
        torch.manual_seed(47 + B + H + HV)
        q = torch.randn(B, T, H, K, dtype=torch.bfloat16)
        k = torch.randn(B, T, H, K, dtype=torch.bfloat16)
        v = torch.randn(B, T, HV, K, dtype=torch.bfloat16)
        a = torch.randn(B, T, HV, dtype=torch.bfloat16)
        b = torch.randn(B, T, HV, dtype=torch.bfloat16)
        A_log = torch.randn(HV, dtype=torch.float32)
        dt_bias = torch.randn(HV, dtype=torch.float32)
        h0 = torch.randn(B, HV, K, K, dtype=torch.float32)
        indices = (torch.arange(B, dtype=torch.int32) if idx is None
                   else torch.tensor(idx, dtype=torch.int32))
        cu = torch.arange(B + 1, dtype=torch.int32) * T
        o, state = ref(A_log, a, dt_bias, q, k, v, b, h0.clone(), indices, cu, K ** -0.5, True)
        cases.append({"name": f"B{B}_T{T}_H{H}_HV{HV}_K{K}" + ("_neg" if idx else ""), "args": {
            "A_log": A_log, "a": a, "dt_bias": dt_bias, "q": q, "k": k, "v": v, "b": b,
            "initial_state_source": h0, "initial_state_indices": indices, "cu_seqlens": cu,
            "scale": K ** -0.5, "use_qk_l2norm_in_kernel": True},
            "out": {"o": o, "state": state}})
    _save("fused_sigmoid_gating_delta_rule_update", cases)


def gen_qkvzba(m):
    ref = m["test_fused_qkvzba_split_reshape"].fused_qkvzba_split_reshape_cat_ref
    cases = []
    # ratios 1..4 of the reference test (test_fused_qkvzba_split_reshape.py:518-555),
    # at small batch, plus an fp16 projection with fp32 b/a
    for rows, nqk, nv, hqk, hv, dt, dba in [(4, 8, 16, 128, 128, torch.bfloat16, torch.bfloat16),
                                           (3, 4, 4, 128, 128, torch.bfloat16, torch.bfloat16),
                                           (2, 2, 6, 128, 128, torch.bfloat16, torch.bfloat16),
                                           (5, 2, 8, 128, 128, torch.bfloat16, torch.bfloat16),
                                           (7, 3, 6, 64, 32, torch.float16, torch.float32)]:
        r = nv // nqk
        g0 = torch.Generator().manual_seed(rows * 1000 + nqk * 10 + nv)
        mixed_qkvz = torch.randn(rows, nqk * (2 * hqk + 2 * r * hv), generator=g0).to(dt)
        mixed_ba = torch.randn(rows, nqk * 2 * r, generator=g0).to(dba)
        qkv, z, b, a = ref(mixed_qkvz, mixed_ba, nqk, nv, hqk, hv)
        cases.append({"name": f"rows{rows}_qk{nqk}_v{nv}_h{hqk}x{hv}", "args": {
            "mixed_qkvz": mixed_qkvz, "mixed_ba": mixed_ba, "num_heads_qk": nqk,
            "num_heads_v": nv, "head_qk": hqk, "head_v": hv},
            "out": {"mixed_qkv": qkv, "z": z, "b": b, "a": a}})
    _save("fused_qkvzba_split_reshape_cat", cases)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref-root", required=True,
                    help="root of the reference checkout (the directory holding triton_npu/)")
    ap.add_argument("--only", default="",
                    help="comma-separated subset of: layernorm,l2norm,rope,conv,chunk,"
                         "recurrent,gating,sigmoid_gating,qkvzba,recurrent_spec,conv_slots,"
                         "rope_inplace")
    args = ap.parse_args()
    torch.set_num_threads(max(1, os.cpu_count() or 1))
    m = _import_reference(args.ref_root)
    gens = {"layernorm": gen_layernorm, "l2norm": gen_l2norm, "rope": gen_rope,
            "conv": gen_conv, "chunk": gen_chunk, "recurrent": gen_recurrent,
            "gating": gen_gating, "sigmoid_gating": gen_sigmoid_gating, "qkvzba": gen_qkvzba,
            "recurrent_spec": gen_recurrent_spec, "conv_slots": gen_conv_slots,
            "rope_inplace": gen_rope_inplace}
    for name, fn in gens.items():
        if not args.only or name in args.only.split(","):
            fn(m)


if __name__ == "__main__":
    main()
