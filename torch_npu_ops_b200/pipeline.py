"""The GDN layer's prefill core as one call: causal conv1d -> chunked gated
delta rule -> gated RMSNorm.

This is the sequence the xLLM Qwen3-Next / Qwen3.5 GDN layer runs between
its input and output projections.  A caller of the reference makes the calls
``npu_causal_conv1d_update_v2`` -> ``npu_chunk_gated_delta_rule(...,
use_qk_l2norm_in_kernel=True)`` -> ``layer_norm_fwd``; here the q/k L2
normalisation moves out of the chunked rule into the conv kernel's output
(``causal_conv1d_varlen_qk_l2norm``), which saves one read and one write of
q and k, and the gated RMSNorm moves into the chunked rule's output
epilogue (``chunk_gated_delta_rule_out_norm``), which saves one write and
one read of o.  ``bench.py`` times this function and the bench-configuration
parity test checks it, so both exercise exactly one code path.
"""

import torch

from . import ops


def gdn_prefill(x, conv_state, conv_weight, conv_bias, g, beta, initial_state, z, norm_weight,
                num_k_heads, num_v_heads, head_dim=128, eps=1e-6, query_start_loc=None,
                events=None, gating=None, return_o=False, fuse_norm=True):
    """Runs one prefill of a GDN layer on the current CUDA stream.

    x: [T, (2 num_k_heads + num_v_heads) head_dim] conv input (q | k | v
    channel blocks), bf16.  conv_state: [N, channels, width - 1], updated in
    place (a fresh prefill passes zeros).  g, beta: [1, T, num_v_heads] fp32;
    or, with ``gating=(A_log, a, b, dt_bias)`` (the inputs of
    ``npu_fused_gdn_gating``, a and b [T, num_v_heads]), g and beta are None
    and the gates are computed inside the chunked rule's kernels.
    initial_state: [N, num_v_heads, head_dim, head_dim] fp32 or None.
    z: [T, num_v_heads, head_dim] gate of the output norm.  query_start_loc:
    [N + 1] int32 on the device (None: one sequence of T tokens).
    ``events``: optional list of 4 CUDA events recorded before the conv,
    after it, after the chunked rule and after the norm.  With g and beta
    given and ``fuse_norm`` (the default), the norm runs inside the chunked
    rule's chain kernel (``chunk_gated_delta_rule_out_norm``), so the last
    two events bracket nothing and o is written only with ``return_o``;
    ``fuse_norm=False`` runs the rule and ``layer_norm_fwd`` as two
    operators (the reference's sequence).

    Returns (conv output [T, channels] with its q and k blocks
    L2-normalised per head, o [1, T, num_v_heads, head_dim] or None, final
    state [N, num_v_heads, head_dim, head_dim] fp32, normed output
    [T * num_v_heads, head_dim]).
    """
    T = x.shape[0]
    hk, hv, d = num_k_heads, num_v_heads, head_dim
    if query_start_loc is None:
        query_start_loc = torch.tensor([0, T], dtype=torch.int32, device=x.device)
    if events:
        events[0].record()
    y = ops.causal_conv1d_varlen_qk_l2norm(x, conv_state, conv_weight, conv_bias, query_start_loc,
                                           2 * hk * d)
    if events:
        events[1].record()
    q = y[:, : hk * d].view(1, T, hk, d)
    k = y[:, hk * d: 2 * hk * d].view(1, T, hk, d)
    v = y[:, 2 * hk * d:].view(1, T, hv, d)
    cu = None if query_start_loc.numel() == 2 else query_start_loc
    if gating is None and fuse_norm:
        out, ht, o = ops.chunk_gated_delta_rule_out_norm(q, k, v, g, beta, z, norm_weight, None,
                                                         initial_state, True, cu, False, eps,
                                                         return_o)
        for e in (events or [])[2:]:
            e.record()
        return y, o, ht, out.view(-1, d)
    if gating is None:
        o, ht = ops.npu_chunk_gated_delta_rule(q, k, v, g, beta, None, initial_state, True, cu,
                                               False, False)
    else:
        A_log, a, b, dt_bias = gating
        o, ht = ops.chunk_gated_delta_rule_gated(q, k, v, A_log, a, b, dt_bias, None,
                                                 initial_state, True, cu, False)
    if events:
        events[2].record()
    out = ops.layer_norm_fwd(o.view(-1, d), norm_weight, None, eps, z.view(-1, d), d, True, True)
    if events:
        events[3].record()
    return y, o, ht, out


def gdn_layer_prefill(mixed_qkvz, mixed_ba, conv_state, conv_weight, conv_bias, A_log, dt_bias,
                      initial_state, norm_weight, num_k_heads, num_v_heads, head_dim=128,
                      eps=1e-6, query_start_loc=None, events=None, return_o=False,
                      fuse_norm=True):
    """One prefill of a GDN layer from its input projections.

    A caller of the reference runs ``npu_fused_qkvzba_split_reshape_cat`` ->
    conv -> ``npu_fused_gdn_gating`` -> ``npu_chunk_gated_delta_rule`` ->
    gated ``layer_norm_fwd``.  Here nothing is de-interleaved: the conv
    reads q, k, v from ``mixed_qkvz [T, Hk * (2 + 2r) * 128]`` in place
    (``causal_conv1d_varlen_qkvz``), the chunked rule computes its gates
    from ``mixed_ba [T, Hk * 2r]`` in place, and the gated norm reads z from
    ``mixed_qkvz`` as a strided view (r = num_v_heads / num_k_heads) inside
    the rule's chain kernel (``chunk_gated_delta_rule_gated_out_norm``;
    ``fuse_norm=False`` runs ``layer_norm_fwd`` after the rule instead).
    The results equal the five-call sequence bit for bit.

    Returns (conv output [T, (2 Hk + Hv) 128] with q/k L2-normalised, o
    [1, T, Hv, 128] (None when the norm is fused and ``return_o`` is not
    set), final state [N, Hv, 128, 128] fp32, normed output [T * Hv, 128]).
    ``events``: optional list of 4 CUDA events recorded before the conv and
    after each stage (with the fused norm the last two bracket nothing).
    """
    T = mixed_qkvz.shape[0]
    hk, hv, d = num_k_heads, num_v_heads, head_dim
    r = hv // hk
    gw = (2 + 2 * r) * d
    if query_start_loc is None:
        query_start_loc = torch.tensor([0, T], dtype=torch.int32, device=mixed_qkvz.device)
    if events:
        events[0].record()
    y = ops.causal_conv1d_varlen_qkvz(mixed_qkvz, conv_state, conv_weight, conv_bias,
                                      query_start_loc, hk, hv, True, True, eps)
    if events:
        events[1].record()
    q = y[:, : hk * d].view(1, T, hk, d)
    k = y[:, hk * d: 2 * hk * d].view(1, T, hk, d)
    v = y[:, 2 * hk * d:].view(1, T, hv, d)
    cu = None if query_start_loc.numel() == 2 else query_start_loc
    if fuse_norm:
        # z head h of token t: in key head h // r's group of the projection
        # row, after its q, k and r v heads
        zv = mixed_qkvz[:, (2 + r) * d:]
        out, ht, o = ops.chunk_gated_delta_rule_gated_out_norm(
            q, k, v, A_log, None, None, dt_bias, zv, norm_weight, None, initial_state, True, cu,
            False, eps, mixed_ba=mixed_ba, z_heads_per_group=r, z_group_stride=gw,
            return_o=return_o)
        for e in (events or [])[2:]:
            e.record()
        return y, o, ht, out.view(T * hv, d)
    o, ht = ops.chunk_gated_delta_rule_gated(q, k, v, A_log, None, None, dt_bias, None,
                                             initial_state, True, cu, False, mixed_ba=mixed_ba)
    if events:
        events[2].record()
    # rows of r value heads: o's r heads of (token, key head) are adjacent, and
    # so are their z heads in the projection, a row of gw elements further on
    z = mixed_qkvz.view(T * hk, gw)[:, (2 + r) * d:]
    out = ops.layer_norm_fwd(o.view(T * hk, r * d), norm_weight.repeat(r), None, eps, z, d, True,
                             True)
    if events:
        events[3].record()
    return y, o, ht, out.view(T * hv, d)
