"""Gated delta rule oracles (test infrastructure only).

Layouts follow the reference: token-major ``[B, T, H, D]``; varlen batches
are ``B == 1`` plus ``cu_seqlens`` (int32/int64, ``[N+1]``).  Grouped-query
heads: value head ``h`` reads key/query head ``h // (H // Hg)``
(triton_npu/triton_src/test_chunk_gated_delta_rule.py:24-31).  Everything is
computed in fp32.
"""

import torch

from . import _out

CHUNK = 64


def _spans(batch, total, cu_seqlens):
    """(batch row, start, end) for every sequence."""
    if cu_seqlens is None:
        return [(b, 0, total) for b in range(batch)]
    cu = [int(v) for v in cu_seqlens.reshape(-1).tolist()]
    return [(0, cu[i], cu[i + 1]) for i in range(len(cu) - 1)]


def prepare_chunk_offsets(cu_seqlens, chunk_size=CHUNK):
    """Chunk offset of every sequence: ``[0, c0, c0+c1, ...]`` with
    ``c_i = ceil(len_i / chunk)`` (prepare_chunk_offsets_like_python,
    triton_npu/torch_api/npu_triton_chunk_gated_delta_rule.cpp:77-113)."""
    cu = cu_seqlens.reshape(-1).to(torch.int64)
    lens = cu[1:] - cu[:-1]
    n = (lens + chunk_size - 1) // chunk_size
    return torch.cat([torch.zeros(1, dtype=torch.int64), torch.cumsum(n, 0)])


def _expand(x, h):
    hq = x.shape[-2]
    return x if hq == h else x.repeat_interleave(h // hq, dim=-2)


def chunk_local_cumsum(g, chunk_size=CHUNK, cu_seqlens=None):
    """Inclusive cumsum of g [B, T, H] inside every chunk of every sequence
    (chunk_local_cumsum_scalar_kernel,
    triton_npu/triton_src/chunk_gated_delta_rule/cumsum.py:25-73)."""
    g = g.to(torch.float32)
    out = torch.empty_like(g)
    for b, s, e in _spans(g.shape[0], g.shape[1], cu_seqlens):
        for c in range(s, e, chunk_size):
            ce = min(c + chunk_size, e)
            out[b, c:ce] = torch.cumsum(g[b, c:ce], dim=0)
    return out


def chunk_scaled_dot_kkt_fwd(k, beta, g_cumsum, chunk_size=CHUNK, cu_seqlens=None):
    """A[t, h, j] = beta_t * exp(g_t - g_{c+j}) * <k_t, k_{c+j}> for j < t-c
    inside the chunk starting at c, else 0; fp32 [B, T, H, BT]
    (chunk_scaled_dot_kkt_fwd_kernel,
    triton_npu/triton_src/chunk_gated_delta_rule/chunk_scaled_dot_kkt.py:25-84)."""
    bsz, t_all, _, _ = k.shape
    h = beta.shape[-1]
    kf = _expand(k.to(torch.float32), h)
    bf = beta.to(torch.float32)
    gf = g_cumsum.to(torch.float32)
    A = torch.zeros(bsz, t_all, h, chunk_size, dtype=torch.float32)
    for b, s, e in _spans(bsz, t_all, cu_seqlens):
        for c in range(s, e, chunk_size):
            ce = min(c + chunk_size, e)
            L = ce - c
            kc = kf[b, c:ce].transpose(0, 1)                     # [H, L, K]
            gram = kc @ kc.transpose(-1, -2)                     # [H, L, L]
            gcs = gf[b, c:ce].t()                                # [H, L]
            dec = torch.exp((gcs[:, :, None] - gcs[:, None, :]).clamp(max=0.0))
            strict = torch.ones(L, L, dtype=torch.bool).tril(-1)
            a = torch.where(strict, gram * dec * bf[b, c:ce].t()[:, :, None], torch.zeros(()))
            A[b, c:ce, :, :L] = a.transpose(0, 1)
    return A


def solve_tril(A, chunk_size=CHUNK, cu_seqlens=None, output_dtype=torch.float32):
    """Per chunk, (I + A_c)^-1 of the valid L x L block (solve_tril_16x16 +
    merge_16x16_to_64x64_inverse kernels,
    triton_npu/triton_src/chunk_gated_delta_rule/solve_tril.py:32-330);
    entries outside the block are zero."""
    bsz, t_all, h, bt = A.shape
    out = torch.zeros(bsz, t_all, h, bt, dtype=torch.float32)
    for b, s, e in _spans(bsz, t_all, cu_seqlens):
        for c in range(s, e, chunk_size):
            ce = min(c + chunk_size, e)
            L = ce - c
            a = A[b, c:ce, :, :L].to(torch.float32).transpose(0, 1)   # [H, L, L]
            eye = torch.eye(L, dtype=torch.float32).expand(h, L, L)
            inv = torch.linalg.solve_triangular(eye + a.tril(-1), eye, upper=False)
            out[b, c:ce, :, :L] = inv.transpose(0, 1)
    return out.to(output_dtype)


def recompute_w_u_fwd(k, v, beta, g_cumsum, A, cu_seqlens=None, chunk_size=CHUNK):
    """WY transform per chunk: ``u = Ai (beta v)``, ``w = Ai (beta e^g k)``
    (recompute_w_u_fwd_kernel,
    triton_npu/triton_src/chunk_gated_delta_rule/wy_fast.py:23-85)."""
    bsz, t_all, h, vd = v.shape
    kf = _expand(k.to(torch.float32), h)
    vf = v.to(torch.float32)
    bf = beta.to(torch.float32)
    gf = g_cumsum.to(torch.float32)
    w = torch.zeros(bsz, t_all, h, kf.shape[-1], dtype=torch.float32)
    u = torch.zeros(bsz, t_all, h, vd, dtype=torch.float32)
    for b, s, e in _spans(bsz, t_all, cu_seqlens):
        for c in range(s, e, chunk_size):
            ce = min(c + chunk_size, e)
            L = ce - c
            ai = A[b, c:ce, :, :L].to(torch.float32).transpose(0, 1)  # [H, L, L]
            bb = bf[b, c:ce].t()[:, :, None]
            eg = torch.exp(gf[b, c:ce]).t()[:, :, None]
            u[b, c:ce] = (ai @ (vf[b, c:ce].transpose(0, 1) * bb)).transpose(0, 1)
            w[b, c:ce] = (ai @ (kf[b, c:ce].transpose(0, 1) * bb * eg)).transpose(0, 1)
    return w, u


def chunk_gated_delta_rule_fwd_h(k, w, u, g=None, initial_state=None,
                                 output_final_state=False, chunk_size=CHUNK,
                                 save_new_value=True, cu_seqlens=None):
    """Chunk-serial state pass
    (chunk_gated_delta_rule_fwd_kernel_h_blockdim64,
    triton_npu/triton_src/chunk_gated_delta_rule/chunk_delta_h.py:30-199):

        h_c stored (state at the start of chunk c)
        v_new   = u_c - w_c h_c
        h_{c+1} = e^{g_last} h_c + (k_c * e^{g_last - g})^T v_new

    Returns ``(h [B, NT, H, K, V], v_new [B, T, H, V], final [N, H, K, V])``
    in fp32 (the reference kernel stores h and v_new in bf16).
    """
    bsz, t_all, h, vd = u.shape
    kd = k.shape[-1]
    kf = _expand(k.to(torch.float32), h)
    wf = w.to(torch.float32)
    uf = u.to(torch.float32)
    gf = g.to(torch.float32) if g is not None else None
    spans = _spans(bsz, t_all, cu_seqlens)
    nts = [(e - s + chunk_size - 1) // chunk_size for _, s, e in spans]
    if cu_seqlens is None:
        hs = torch.zeros(bsz, nts[0] if nts else 0, h, kd, vd, dtype=torch.float32)
    else:
        hs = torch.zeros(1, sum(nts), h, kd, vd, dtype=torch.float32)
    v_new = torch.zeros(bsz, t_all, h, vd, dtype=torch.float32)
    final = torch.zeros(len(spans), h, kd, vd, dtype=torch.float32)
    off = 0
    for n, (b, s, e) in enumerate(spans):
        st = (initial_state[n].to(torch.float32).clone() if initial_state is not None
              else torch.zeros(h, kd, vd, dtype=torch.float32))
        for ci, c in enumerate(range(s, e, chunk_size)):
            ce = min(c + chunk_size, e)
            slot = (b, ci) if cu_seqlens is None else (0, off + ci)
            hs[slot[0], slot[1]] = st
            vn = uf[b, c:ce].transpose(0, 1) - wf[b, c:ce].transpose(0, 1) @ st   # [H, L, V]
            v_new[b, c:ce] = vn.transpose(0, 1)
            kc = kf[b, c:ce].transpose(0, 1)                                     # [H, L, K]
            if gf is not None:
                gl = gf[b, ce - 1]                                               # [H]
                fac = torch.exp((gl[None, :] - gf[b, c:ce]).clamp(max=0.0)).t()  # [H, L]
                st = st * torch.exp(gl)[:, None, None] + (kc * fac[:, :, None]).transpose(-1, -2) @ vn
            else:
                st = st + kc.transpose(-1, -2) @ vn
        final[n] = st
        off += nts[n]
    return hs, (v_new if save_new_value else None), (final if output_final_state else None)


def chunk_fwd_o(q, k, v_new, h_states, g=None, scale=None, chunk_size=CHUNK, cu_seqlens=None):
    """Output pass (chunk_fwd_kernel_o,
    triton_npu/triton_src/chunk_gated_delta_rule/chunk_o.py:26-116):
    ``o = scale * (q h_c e^g + tril(q k^T e^{g_i - g_j}) v_new)``."""
    bsz, t_all, h, vd = v_new.shape
    kd = q.shape[-1]
    if scale is None:
        scale = kd ** -0.5
    qf = _expand(q.to(torch.float32), h)
    kf = _expand(k.to(torch.float32), h)
    vf = v_new.to(torch.float32)
    gf = g.to(torch.float32) if g is not None else None
    o = torch.zeros(bsz, t_all, h, vd, dtype=torch.float32)
    off = 0
    for b, s, e in _spans(bsz, t_all, cu_seqlens):
        for ci, c in enumerate(range(s, e, chunk_size)):
            ce = min(c + chunk_size, e)
            L = ce - c
            hb = h_states[b, ci] if cu_seqlens is None else h_states[0, off + ci]
            hb = hb.to(torch.float32)
            qc = qf[b, c:ce].transpose(0, 1)
            kc = kf[b, c:ce].transpose(0, 1)
            inter = qc @ hb
            att = qc @ kc.transpose(-1, -2)
            if gf is not None:
                gcs = gf[b, c:ce].t()
                inter = inter * torch.exp(gcs)[:, :, None]
                att = att * torch.exp((gcs[:, :, None] - gcs[:, None, :]).clamp(max=0.0))
            att = att * torch.ones(L, L).tril()
            o[b, c:ce] = (scale * (inter + att @ vf[b, c:ce].transpose(0, 1))).transpose(0, 1)
        if cu_seqlens is not None:
            off += (e - s + chunk_size - 1) // chunk_size
    return o


def _l2n(x, eps=1e-6):
    # _l2norm, triton_npu/triton_src/test_chunk_gated_delta_rule.py:20-21
    return x * torch.rsqrt((x * x).sum(dim=-1, keepdim=True) + eps)


def chunk_gated_delta_rule(q, k, v, g, beta, scale=None, initial_state=None,
                           output_final_state=False, cu_seqlens=None,
                           use_qk_l2norm_in_kernel=False):
    """Chunked gated delta rule prefill.

    Restates ``chunk_gated_delta_rule_ref`` and its per-sequence engine
    ``_torch_chunk_gated_delta_rule_chunked``
    (triton_npu/triton_src/test_chunk_gated_delta_rule.py:134-197 and :34-131):
    per sequence and head, chunks of 64 tokens,

        gc   = cumsum(g) in the chunk,  D_ij = e^{gc_i - gc_j} (i >= j)
        T    = (I + strict_tril(beta_i D_ij k_i.k_j))^-1
        u    = T (beta v),  w = T (beta e^{gc} k)
        v'   = u - w S,  o = s (q e^{gc}) S + s tril(q k^T * D) v'
        S   <- e^{gc_last} S + (k e^{gc_last - gc})^T v'

    ``scale`` defaults to K^-0.5 (the reference path always uses that;
    npu_triton_chunk_gated_delta_rule.cpp:615 also accepts an explicit one).
    Batches without ``cu_seqlens`` treat every batch row as one sequence.
    Returns ``(o in v's dtype, final fp32 [N, H, K, V] or None)``.
    """
    bsz, t_all, hq, kd = q.shape
    h, vd = v.shape[2], v.shape[3]
    if scale is None:
        scale = kd ** -0.5
    qf = q.to(torch.float32)
    kf = k.to(torch.float32)
    if use_qk_l2norm_in_kernel:
        # the reference normalises in the input dtype before the chunked pass
        # (npu_l2norm_last_dim, npu_triton_chunk_gated_delta_rule.cpp:608-609,
        # returns q's dtype): normalise in fp32, round once to that dtype
        qf = _l2n(qf).to(q.dtype).to(torch.float32)
        kf = _l2n(kf).to(k.dtype).to(torch.float32)
    qf, kf = _expand(qf, h), _expand(kf, h)
    vf, gf, bf = v.to(torch.float32), g.to(torch.float32), beta.to(torch.float32)
    spans = _spans(bsz, t_all, cu_seqlens)
    o = torch.zeros(bsz, t_all, h, vd, dtype=torch.float32)
    final = torch.zeros(len(spans), h, kd, vd, dtype=torch.float32)
    for n, (b, s, e) in enumerate(spans):
        st = (initial_state[n].to(torch.float32).clone() if initial_state is not None
              else torch.zeros(h, kd, vd, dtype=torch.float32))
        for c in range(s, e, CHUNK):
            ce = min(c + CHUNK, e)
            L = ce - c
            qc, kc, vc = (x[b, c:ce].transpose(0, 1) for x in (qf, kf, vf))   # [H, L, D]
            bc = bf[b, c:ce].t()[:, :, None]                                   # [H, L, 1]
            gc = torch.cumsum(gf[b, c:ce].t(), dim=-1)                         # [H, L]
            dd = gc[:, :, None] - gc[:, None, :]
            low = torch.ones(L, L, dtype=torch.bool).tril()
            D = torch.where(low, torch.exp(dd.clamp(max=0.0)), torch.zeros(()))
            a = (kc @ kc.transpose(-1, -2)) * D * bc
            a = a * torch.ones(L, L).tril(-1)
            eye = torch.eye(L).expand(h, L, L)
            T = torch.linalg.solve_triangular(eye + a, eye, upper=False)
            u = T @ (vc * bc)
            w = T @ (kc * bc * torch.exp(gc)[:, :, None])
            vn = u - w @ st
            att = (qc @ kc.transpose(-1, -2)) * D
            oc = scale * ((qc * torch.exp(gc)[:, :, None]) @ st + att @ vn)
            o[b, c:ce] = oc.transpose(0, 1)
            gl = gc[:, -1]
            kt = kc * torch.exp((gl[:, None] - gc).clamp(max=0.0))[:, :, None]
            st = st * torch.exp(gl)[:, None, None] + kt.transpose(-1, -2) @ vn
        final[n] = st
    return _out.out(o, v.dtype), (final if output_final_state else None)


def fused_recurrent_gated_delta_rule(q, k, v, g, beta=None, scale=None,
                                     initial_state=None, inplace_final_state=True,
                                     cu_seqlens=None, ssm_state_indices=None,
                                     use_qk_l2norm_in_kernel=False, num_accepted_tokens=None):
    """Token-serial gated delta rule (decode), plain and speculative.

    Restates ``recurrent_gated_delta_rule_ref``
    (triton_npu/triton_src/test_fused_recurrent_gated_delta_rule.py:584-617)
    with the state addressing of ``fused_recurrent_gated_delta_rule_fwd_kernel``
    (same file :31-178) and ``..._spec_fwd_kernel`` (:193-307): per token
    ``S *= e^g; v' = beta (v - S^T k); S += k v'^T; o = scale * S^T q``; the
    in-kernel L2 norm is ``x / sqrt(sum(x^2) + 1e-6)`` (:125-127).

    State slots: ``ssm_state_indices`` None (slot n), ``[N]`` (one slot per
    sequence) or ``[N, T]`` (one per token).  The initial state is the slot
    of token 0, or of token ``num_accepted_tokens[n] - 1`` under speculative
    decoding (where a ``[N]`` table is read as the flat table the reference
    kernel addresses with token stride 1).  Under speculative decoding, or
    in place with a ``[N, T]`` table, the state after every token t is
    written to slot (n, t); otherwise the final state goes back to the
    initial slot (in place) or to row n of a new ``[N, HV, K, V]`` tensor.
    A negative slot reads as zeros and is never written.  Returns
    ``(o [B, T, HV, V] in v's dtype, final_state)``.
    """
    bsz, t_all, hq, kd = q.shape
    hv, vd = v.shape[2], v.shape[3]
    if scale is None:
        scale = kd ** -0.5
    qf, kf = q.to(torch.float32), k.to(torch.float32)
    if use_qk_l2norm_in_kernel:
        qf = qf / torch.sqrt((qf * qf).sum(-1, keepdim=True) + 1e-6)
        kf = kf / torch.sqrt((kf * kf).sum(-1, keepdim=True) + 1e-6)
    qf, kf = _expand(qf, hv) * scale, _expand(kf, hv)
    vf, gf = v.to(torch.float32), g.to(torch.float32)
    bf = beta.to(torch.float32) if beta is not None else torch.ones_like(gf)
    spans = _spans(bsz, t_all, cu_seqlens)
    spec = num_accepted_tokens is not None
    idx = None if ssm_state_indices is None else ssm_state_indices.to(torch.int64)
    flat = None if idx is None else idx.reshape(-1)
    if idx is not None:
        s_seq = idx.shape[1] if idx.dim() == 2 else 1
        s_tok = 1 if (idx.dim() == 2 or spec) else 0
    per_token = spec or (idx is not None and idx.dim() == 2 and inplace_final_state)
    o = torch.zeros(bsz, t_all, hv, vd, dtype=torch.float32)
    target = initial_state if inplace_final_state else torch.zeros(
        len(spans), hv, kd, vd, dtype=initial_state.dtype)
    for n, (b, s, e) in enumerate(spans):
        if per_token and e == s:
            continue
        i0 = int(num_accepted_tokens.reshape(-1)[n]) - 1 if spec else 0
        slot = n if idx is None else int(flat[n * s_seq + i0 * s_tok])
        st = (initial_state[slot].to(torch.float32).clone() if slot >= 0
              else torch.zeros(hv, kd, vd))
        for t in range(s, e):
            st = st * torch.exp(gf[b, t])[:, None, None]
            vn = (vf[b, t] - torch.einsum("hk,hkv->hv", kf[b, t], st)) * bf[b, t][:, None]
            st = st + kf[b, t][:, :, None] * vn[:, None, :]
            o[b, t] = torch.einsum("hk,hkv->hv", qf[b, t], st)
            if per_token:
                ts = int(flat[n * s_seq + (t - s) * s_tok])
                if ts >= 0:
                    target[ts] = st.to(target.dtype)
        if per_token:
            continue
        if inplace_final_state:
            if slot >= 0:
                initial_state[slot].copy_(st.to(initial_state.dtype))
        else:
            target[n] = st.to(target.dtype)
    return _out.out(o, v.dtype), target


def _softplus(x, beta=1.0, threshold=20.0):
    """torch Softplus semantics: log(1 + e^{beta x}) / beta, or x where
    beta x > threshold."""
    bx = beta * x
    return torch.where(bx <= threshold, torch.log1p(torch.exp(bx)) / beta, x)


def fused_gdn_gating(A_log, a, b, dt_bias, beta=1.0, threshold=20.0):
    """GDN gates from the projections: ``g = -exp(A_log) * softplus(a +
    dt_bias)`` (fp32) and ``beta_out = sigmoid(b)`` (b's dtype).

    Restates ``torch_fused_gdn_gating``
    (triton_npu/triton_src/test_fused_gdn_gating.py:45-57) with the output
    shapes of ``npu_fused_gdn_gating``
    (triton_npu/torch_api/npu_triton_fused_gdn_gating.cpp:55-63):
    a, b are ``[batch, heads]``; both outputs are ``[1, batch, heads]``.
    """
    g = -torch.exp(A_log.to(torch.float32)) * _softplus(
        a.to(torch.float32) + dt_bias.to(torch.float32), beta, threshold)
    beta_out = _out.out(torch.sigmoid(b.to(torch.float32)), b.dtype)
    return g[None], beta_out[None]


def fused_sigmoid_gating_delta_rule_update(A_log, a, dt_bias, q, k, v, b,
                                           initial_state_source, initial_state_indices,
                                           cu_seqlens, scale=None,
                                           use_qk_l2norm_in_kernel=False,
                                           softplus_beta=1.0, softplus_threshold=20.0):
    """Recurrent gated delta rule with the gates computed from the
    projections inside the step.

    Restates ``torch_sigmoid_gating_delta_rule_update``
    (triton_npu/triton_src/test_fused_sigmoid_gating_delta_rule_update.py:
    178-222) with the slot rules of
    ``fused_sigmoid_gating_delta_rule_update_kernel`` (same file :11-117):
    per token ``g = -exp(A_log) softplus(a + dt_bias)``, ``beta =
    sigmoid(b)`` (fp32), then the delta-rule step of
    ``fused_recurrent_gated_delta_rule``.  Sequence n starts from slot
    ``initial_state_indices[n]`` of ``initial_state_source`` and writes its
    final state back there (in place); a negative index starts from zeros
    and writes nothing.  Returns ``o [B, T, HV, V]`` in q's dtype.
    """
    bsz, t_all, hq, kd = k.shape
    hv, vd = v.shape[2], v.shape[3]
    if scale is None:
        scale = kd ** -0.5
    qf, kf = q.to(torch.float32), k.to(torch.float32)
    if use_qk_l2norm_in_kernel:
        qf = qf / torch.sqrt((qf * qf).sum(-1, keepdim=True) + 1e-6)
        kf = kf / torch.sqrt((kf * kf).sum(-1, keepdim=True) + 1e-6)
    qf, kf = _expand(qf, hv) * scale, _expand(kf, hv)
    vf = v.to(torch.float32)
    g = -torch.exp(A_log.to(torch.float32)) * _softplus(
        a.to(torch.float32) + dt_bias.to(torch.float32), softplus_beta, softplus_threshold)
    bt = torch.sigmoid(b.to(torch.float32))
    qf, kf, vf = (x.reshape(bsz * t_all, hv, -1) for x in (qf, kf, vf))
    g, bt = g.reshape(bsz * t_all, hv), bt.reshape(bsz * t_all, hv)
    o = torch.zeros(bsz * t_all, hv, vd, dtype=torch.float32)
    for n in range(cu_seqlens.numel() - 1):
        s, e = int(cu_seqlens[n]), int(cu_seqlens[n + 1])
        if e == s:
            continue
        slot = int(initial_state_indices[n])
        st = (torch.zeros(hv, kd, vd) if slot < 0
              else initial_state_source[slot].to(torch.float32).clone())
        for t in range(s, e):
            st = st * torch.exp(g[t])[:, None, None]
            vn = (vf[t] - torch.einsum("hk,hkv->hv", kf[t], st)) * bt[t][:, None]
            st = st + kf[t][:, :, None] * vn[:, None, :]
            o[t] = torch.einsum("hk,hkv->hv", qf[t], st)
        if slot >= 0:
            initial_state_source[slot].copy_(st.to(initial_state_source.dtype))
    return _out.out(o.reshape(bsz, t_all, hv, vd), q.dtype)


def fused_qkvzba_split_reshape_cat(mixed_qkvz, mixed_ba, num_heads_qk, num_heads_v, head_qk,
                                   head_v):
    """De-interleave the GDN input projections.

    Restates ``fused_qkvzba_split_reshape_cat_ref``
    (triton_npu/triton_src/test_fused_qkvzba_split_reshape.py:463-507):
    ``mixed_qkvz [rows, nqk * (2 hqk + 2 r hv)]`` holds, per key head,
    ``q | k | v (r heads) | z (r heads)`` and ``mixed_ba [rows, nqk * 2r]``
    holds ``b (r) | a (r)``, r = num_heads_v / num_heads_qk.  Returns
    ``mixed_qkv [rows, 2 nqk hqk + nv hv]`` (all q, then all k, then all v),
    ``z [rows, nv, hv]``, ``b`` and ``a [rows, nv]``.  A pure permutation:
    every output value is an input value.
    """
    rows = mixed_qkvz.shape[0]
    r = num_heads_v // num_heads_qk
    qkvz = mixed_qkvz.reshape(rows, num_heads_qk, 2 * head_qk + 2 * r * head_v)
    ba = mixed_ba.reshape(rows, num_heads_qk, 2 * r)
    q = qkvz[..., :head_qk].reshape(rows, num_heads_qk * head_qk)
    k = qkvz[..., head_qk:2 * head_qk].reshape(rows, num_heads_qk * head_qk)
    v = qkvz[..., 2 * head_qk:2 * head_qk + r * head_v].reshape(rows, num_heads_v * head_v)
    z = qkvz[..., 2 * head_qk + r * head_v:].reshape(rows, num_heads_v, head_v)
    b = ba[..., :r].reshape(rows, num_heads_v)
    a = ba[..., r:].reshape(rows, num_heads_v)
    return torch.cat([q, k, v], dim=-1).contiguous(), z.contiguous(), b.contiguous(), a.contiguous()
