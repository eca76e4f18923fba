"""Host-side mirror of the reference's operator API for the GDN / norm hot
path, on top of the C ABI (``include/xops_b200.h``).

Names, argument meaning, defaults, output allocation and error behaviour
follow ``xllm::kernel::npu`` (triton_npu/torch_api/triton_ops_api.h:29-198),
``npu_ops`` (ascendc_npu/ascendc_ops_api.h:24-39) and the pybind schemas of
``npu_python_extension_lib`` (npu_python_extension/op_register.cpp:52-63).
Validation failures raise ``RuntimeError`` (what the reference's
``TORCH_CHECK`` raises in Python).  Every op launches on the current CUDA
stream of the input's device and never synchronises; there is no CPU path.
"""

import math

import torch

from . import _lib

_DT = {torch.float32: _lib.F32, torch.bfloat16: _lib.BF16, torch.float16: _lib.F16}


def _check(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _dt(t, what):
    _check(t.dtype in _DT, f"{what}: unsupported dtype {t.dtype}")
    return _DT[t.dtype]


def _cuda(*ts):
    for t in ts:
        if t is not None:
            _check(t.is_cuda, "tensors must be on a CUDA device")


def _stream(t):
    return torch.cuda.current_stream(t.device).cuda_stream


def _ptr(t):
    return None if t is None else t.data_ptr()


def _i32(t):
    return None if t is None else t.to(torch.int32).contiguous()


# --------------------------------------------------------------------- norms
def npu_l2norm_last_dim(x, eps=1e-6):
    """``x * rsqrt(sum(x^2) + eps)`` over the last axis, bf16
    (npu_triton_l2norm.cpp:52-108 requires bf16; fp32 is also accepted)."""
    _cuda(x)
    _check(x.dim() >= 1, "npu_l2norm_last_dim expects x.dim() >= 1")
    _check(x.dtype in (torch.bfloat16, torch.float32), "x tensor must be bfloat16")
    xc = x.contiguous()
    y = torch.empty_like(xc)
    cols = x.shape[-1]
    _check(cols > 0, "npu_l2norm_last_dim expects hidden dim > 0")
    rows = xc.numel() // cols
    _check(rows > 0, "npu_l2norm_last_dim expects non-empty input")
    _lib.call("xops_l2norm_last_dim", xc.data_ptr(), y.data_ptr(), rows, cols, float(eps),
              _dt(x, "npu_l2norm_last_dim"), _stream(x))
    return y.view(x.shape)


def _layer_norm(x, weight, bias, eps, z, group_size, norm_before_gate, is_rms_norm):
    _cuda(x, weight, bias, z)
    n = x.shape[-1]
    x2 = x.reshape(-1, n)
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    m = x2.shape[0]
    gs = n if group_size is None or group_size < 0 else int(group_size)
    _check(gs > 0 and n % gs == 0, f"layer_norm_fwd: N={n} not divisible by group_size={gs}")
    _check(weight.shape == (n,), "layer_norm_fwd: weight must have shape (N,)")
    if bias is not None:
        _check(bias.shape == (n,), "layer_norm_fwd: bias must have shape (N,)")
        _check(bias.dtype == weight.dtype, "layer_norm_fwd: bias dtype must match weight")
    z2 = None
    if z is not None:
        z2 = z.reshape(-1, n)
        if z2.stride(-1) != 1:
            z2 = z2.contiguous()
        _check(z2.shape == (m, n), "layer_norm_fwd: z must have the shape of x")
        _check(z2.dtype == x.dtype, "layer_norm_fwd: z dtype must match x")
    w = weight.contiguous()
    b = bias.contiguous() if bias is not None else None
    ng = n // gs
    y = torch.empty((m, n), dtype=x.dtype, device=x.device)
    rstd = torch.empty(ng * m, dtype=torch.float32, device=x.device)
    mean = None if is_rms_norm else torch.empty(ng * m, dtype=torch.float32, device=x.device)
    _lib.call("xops_layer_norm_fwd", x2.data_ptr(), w.data_ptr(), _ptr(b), _ptr(z2), y.data_ptr(),
              _ptr(mean), rstd.data_ptr(), m, n, gs, x2.stride(0),
              z2.stride(0) if z2 is not None else 0, y.stride(0), float(eps),
              int(bool(norm_before_gate)), int(bool(is_rms_norm)), _dt(x, "layer_norm_fwd"),
              _dt(w, "layer_norm_fwd"), _stream(x))
    return y.view(x.shape), mean, rstd


def layer_norm_fwd(x, weight, bias=None, eps=1e-6, z=None, group_size=-1, norm_before_gate=True,
                   is_rms_norm=False):
    """Grouped LayerNorm / RMSNorm with optional bias and SiLU gate z; returns
    y with x's shape and dtype (npu_triton_layernorm_fwd.cpp:48-333; group
    sizes beyond 128 take the same kernel family, with bias)."""
    return _layer_norm(x, weight, bias, eps, z, group_size, norm_before_gate, is_rms_norm)[0]


def layer_norm_fwd_with_stats(x, weight, bias=None, eps=1e-6, z=None, group_size=-1,
                              norm_before_gate=True, is_rms_norm=False):
    """``layer_norm_fwd`` that also returns the fp32 ``mean`` (None for RMS)
    and ``rstd`` vectors, indexed ``group * M + row`` like the reference
    kernels (test_layernorm_fwd.py:1163-1165)."""
    return _layer_norm(x, weight, bias, eps, z, group_size, norm_before_gate, is_rms_norm)


def npu_gemma_rms_norm(x, gamma, epsilon=1e-6):
    """Gemma RMSNorm; returns ``(rstd, y)`` with rstd fp32 of shape
    ``x.shape[:-gamma.dim()] + (1,)*gamma.dim()`` (ascendc_npu/gemma_rms_norm.cpp:28-57)."""
    _cuda(x, gamma)
    gd = gamma.dim()
    _check(gd >= 1 and x.dim() >= gd and tuple(x.shape[x.dim() - gd:]) == tuple(gamma.shape),
           "gemma_rms_norm: gamma must match the trailing dims of x")
    n = gamma.numel()
    xc = x.contiguous()
    g = gamma.contiguous()
    rows = xc.numel() // n if n else 0
    y = torch.empty_like(xc)
    lead = tuple(x.shape[: x.dim() - gd])
    rstd = torch.empty(lead + (1,) * gd if x.dim() > gd else (1,) * x.dim(),
                       dtype=torch.float32, device=x.device)
    _lib.call("xops_gemma_rms_norm", xc.data_ptr(), g.data_ptr(), y.data_ptr(), rstd.data_ptr(),
              rows, n, float(epsilon), _dt(x, "gemma_rms_norm"), _dt(g, "gemma_rms_norm"),
              _stream(x))
    return rstd, y


# ---------------------------------------------------------------------- rope
def rope_inplace(x, sin, cos, rope_dim=64):
    """Interleaved RoPE on the last ``rope_dim`` dims of x ([bsz, hidden] or
    [bsz, heads, hidden]) in place, sin / cos [bsz, rope_dim] shared by a
    row's heads (npu_triton_rope_inplace.cpp:22-66).  Returns x."""
    _cuda(x, sin, cos)
    _check(x.dim() in (2, 3), "rope_inplace expects x of shape [bsz, hidden] or "
                              "[bsz, heads, hidden]")
    _check(x.stride(-1) == 1, "rope_inplace expects x's last dimension to be contiguous")
    x3 = x if x.dim() == 3 else x.unsqueeze(1)
    bsz, heads, hidden = x3.shape
    _check(sin.dim() == 2 and cos.dim() == 2 and sin.shape == cos.shape
           and sin.shape[0] == bsz and sin.shape[1] >= rope_dim,
           "rope_inplace expects sin and cos of shape [bsz, rope_dim]")
    _check(sin.stride(-1) == 1 and cos.stride(-1) == 1 and sin.stride(0) == cos.stride(0),
           "rope_inplace expects sin and cos rows with the same stride")
    _lib.call("xops_rope_inplace", x.data_ptr(), sin.data_ptr(), cos.data_ptr(), bsz, heads,
              hidden, int(rope_dim), x3.stride(0), x3.stride(1), sin.stride(0),
              _dt(x, "rope_inplace"), _dt(sin, "rope_inplace"), _stream(x))
    return x


def npu_split_rmsnorm_rope(input, sin, cos, q_weight, k_weight, q_hidden_size, kv_hidden_size,
                           head_dim, eps, q_bias=None, k_bias=None, bias=False):
    """Split packed qkv, per-head RMSNorm on q/k, NeoX RoPE, copy v; returns
    ``(q, k, v)`` (npu_triton_split_rmsnorm_rope.cpp:57-143).  ``sin``/``cos``
    may be narrower than ``head_dim`` (partial rotary: the first
    ``sin.size(1)`` dims rotate)."""
    _check(input.dim() == 2, "split_rmsnorm_rope input must be a 2D tensor")
    _check(sin.dim() == 2 and cos.dim() == 2, "split_rmsnorm_rope sin and cos must be 2D tensors")
    _check(q_weight.dim() == 1 and k_weight.dim() == 1,
           "split_rmsnorm_rope q_weight and k_weight must be 1D tensors")
    _check(head_dim > 0 and (head_dim & (head_dim - 1)) == 0,
           "split_rmsnorm_rope head_dim must be a power of two")
    _check(kv_hidden_size > 0 and q_hidden_size % kv_hidden_size == 0,
           "split_rmsnorm_rope q_hidden_size must be divisible by kv_hidden_size")
    _check(kv_hidden_size % head_dim == 0,
           "split_rmsnorm_rope kv_hidden_size must be divisible by head_dim")
    _check(input.size(1) == q_hidden_size + 2 * kv_hidden_size,
           "split_rmsnorm_rope input hidden size mismatch")
    rd = sin.size(1)
    _check(sin.size(0) == input.size(0) and cos.size(0) == input.size(0) and cos.size(1) == rd
           and 0 < rd <= head_dim, "split_rmsnorm_rope sin/cos shape mismatch")
    _check(q_weight.size(0) == head_dim and k_weight.size(0) == head_dim,
           "split_rmsnorm_rope q/k weight shape mismatch")
    _check(q_weight.dtype == k_weight.dtype, "split_rmsnorm_rope q/k weight dtype mismatch")
    _check(sin.dtype == cos.dtype, "split_rmsnorm_rope sin/cos dtype mismatch")
    _cuda(input, sin, cos, q_weight, k_weight, q_bias, k_bias)
    t = input.size(0)
    inp = input.contiguous()
    s, c = sin.contiguous(), cos.contiguous()
    qw, kw = q_weight.contiguous(), k_weight.contiguous()
    use_b = bool(bias) and q_bias is not None and k_bias is not None
    qb = q_bias.to(qw.dtype).contiguous() if use_b else None
    kb = k_bias.to(qw.dtype).contiguous() if use_b else None
    q = torch.empty((t, q_hidden_size), dtype=input.dtype, device=input.device)
    k = torch.empty((t, kv_hidden_size), dtype=input.dtype, device=input.device)
    v = torch.empty((t, kv_hidden_size), dtype=input.dtype, device=input.device)
    _lib.call("xops_split_rmsnorm_rope", inp.data_ptr(), s.data_ptr(), c.data_ptr(), q.data_ptr(),
              k.data_ptr(), v.data_ptr(), qw.data_ptr(), _ptr(qb), kw.data_ptr(), _ptr(kb), t,
              q_hidden_size, kv_hidden_size, head_dim, rd, float(eps),
              _dt(input, "split_rmsnorm_rope"), _dt(qw, "split_rmsnorm_rope"),
              _dt(s, "split_rmsnorm_rope"), _stream(input))
    return q, k, v


# -------------------------------------------------------------------- conv1d
def npu_causal_conv1d_update(x, conv_state, weight, activation=True, bias=None,
                             cache_seqlens=None, conv_state_indices=None, num_accepted_tokens=None,
                             query_start_loc=None, max_query_len=-1, intermediate_conv_window=None,
                             pad_slot_id=-1, validate_data=False):
    """Decode conv update (npu_triton_causal_conv1d_update.cpp:22-137).
    x: [batch, dim] or [batch, dim, seqlen]; conv_state [lines, dim,
    state_len] is updated IN PLACE; returns out shaped like x.  Like the
    reference, ``query_start_loc``, ``cache_seqlens`` and
    ``num_accepted_tokens`` are rejected here (use
    ``npu_causal_conv1d_update_v2`` for varlen batches)."""
    _check(query_start_loc is None,
           "Current op does not support non-empty values for query_start_loc.")
    _check(cache_seqlens is None and num_accepted_tokens is None,
           "currently causal_conv1d_update don't support input cache_len and mtp scenerios.")
    _cuda(x, conv_state, weight, bias, conv_state_indices)
    squeeze = x.dim() == 2
    x3 = x.unsqueeze(-1) if squeeze else x
    _check(x3.dim() == 3 and conv_state.dim() == 3 and weight.dim() == 2,
           "causal_conv1d_update: bad tensor ranks")
    batch, dim, seqlen = x3.shape
    width = weight.size(1)
    _check(weight.size(0) == dim and conv_state.size(1) == dim, "causal_conv1d_update: dim mismatch")
    _check(conv_state.is_contiguous(), "causal_conv1d_update: conv_state must be contiguous")
    _check(conv_state.dtype == x.dtype and weight.dtype == x.dtype,
           "causal_conv1d_update: x, conv_state and weight must share a dtype")
    w = weight.contiguous()
    b = bias.to(x.dtype).contiguous() if bias is not None else None
    idx = _i32(conv_state_indices)
    if idx is not None:
        _check(idx.numel() == batch, "causal_conv1d_update: conv_state_indices batch mismatch")
    out = torch.empty((batch, dim, seqlen), dtype=x.dtype, device=x.device)
    _lib.call("xops_causal_conv1d_update", x3.data_ptr(), conv_state.data_ptr(), w.data_ptr(),
              _ptr(b), _ptr(idx), out.data_ptr(), batch, dim, seqlen, width, conv_state.size(2),
              conv_state.size(0), x3.stride(0), x3.stride(1), x3.stride(2), int(bool(activation)),
              int(pad_slot_id), _dt(x, "causal_conv1d_update"), _stream(x))
    return out.squeeze(-1) if squeeze else out


def npu_causal_conv1d_update_v2(x, conv_state, weight, activation=True, bias=None,
                                conv_state_indices=None, query_start_loc=None, max_query_len=-1,
                                pad_slot_id=-1, block_idx_last_scheduled_token=None,
                                initial_state_idx=None, validate_data=False,
                                num_accepted_tokens=None):
    """Varlen conv (npu_triton_causal_conv1d_update_v2.cpp:99-239).  With
    ``query_start_loc`` x is [num_tokens, dim] token-major and every
    sequence convolves over cat(conv_state history, its tokens); without it
    x is [B, D] or [B, D, T] (each row one sequence of T tokens).
    conv_state [lines, dim, state_len] is updated IN PLACE.  Speculative
    decoding (``num_accepted_tokens``: history from column accepted - 1,
    width - 1 + len - 1 columns rewritten) and prefix-cache block tables
    (a [B, blocks] ``conv_state_indices`` with ``initial_state_idx`` /
    ``block_idx_last_scheduled_token`` choosing the read and the written
    line) run on the slot-table kernel."""
    _check(weight.dim() == 2, "causal_conv1d_update_v2 expects weight shape [dim, width].")
    _check((block_idx_last_scheduled_token is None) == (initial_state_idx is None),
           "causal_conv1d_update_v2 expects both APC tensors or neither.")
    _check(conv_state.dim() == 3,
           "causal_conv1d_update_v2 expects conv_state shape [num_cache_lines, dim, state_len].")
    _cuda(x, conv_state, weight, bias, conv_state_indices, query_start_loc,
          block_idx_last_scheduled_token, initial_state_idx, num_accepted_tokens)
    width = weight.size(1)
    _check(1 <= width <= 6, f"causal_conv1d_update_v2 expects width in [1, 6], got {width}")
    unsq = False
    if query_start_loc is not None:
        _check(x.dim() == 2, "causal_conv1d_update_v2 expects x to be 2D [num_tokens, dim] "
                             "when query_start_loc is provided.")
        qsl = _i32(query_start_loc)
        _check(qsl.dim() == 1 and qsl.numel() >= 2,
               "query_start_loc must be 1D with shape [batch + 1].")
        xv = x.contiguous()
        batch = qsl.numel() - 1
    else:
        unsq = x.dim() == 2
        xw = x.unsqueeze(-1) if unsq else x
        _check(xw.dim() == 3, "causal_conv1d_update_v2 expects x to have shape [B, D] or [B, D, T] "
                              "when query_start_loc is not provided.")
        batch, _, seqlen = xw.shape
        xv = xw.transpose(1, 2).contiguous().view(batch * seqlen, xw.size(1))
        qsl = torch.arange(0, (batch + 1) * seqlen, seqlen, dtype=torch.int32, device=x.device)
    dim = xv.size(1)
    _check(weight.size(0) == dim, f"weight dim mismatch. Expected {dim}, got {weight.size(0)}")
    _check(conv_state.size(1) == dim,
           f"conv_state dim mismatch. Expected {dim}, got {conv_state.size(1)}")
    _check(conv_state.size(2) >= width - 1,
           "causal_conv1d_update_v2: conv_state must hold at least width - 1 history columns")
    _check(conv_state.is_contiguous(), "causal_conv1d_update_v2: conv_state must be contiguous")
    _check(conv_state.dtype == xv.dtype and weight.dtype == xv.dtype,
           "causal_conv1d_update_v2: x, conv_state and weight must share a dtype")
    if bias is not None:
        _check(bias.dim() == 1 and bias.size(0) == dim,
               "bias must have shape [dim] for causal_conv1d_update_v2.")
    b = bias.to(xv.dtype).contiguous() if bias is not None else None
    idx = _i32(conv_state_indices)
    slots = (num_accepted_tokens is not None or initial_state_idx is not None
             or (idx is not None and idx.dim() == 2 and idx.size(1) > 1)
             or conv_state.size(2) != width - 1)
    if slots:
        if idx is not None:
            _check(idx.dim() in (1, 2) and idx.size(0) == batch,
                   f"conv_state_indices batch mismatch. Expected {batch}, got {idx.size(0)}")
        acc, ini, last = (_i32(num_accepted_tokens), _i32(initial_state_idx),
                          _i32(block_idx_last_scheduled_token))
        for t, name in ((acc, "num_accepted_tokens"), (ini, "initial_state_idx"),
                        (last, "block_idx_last_scheduled_token")):
            _check(t is None or t.numel() == batch, f"{name} must have one entry per sequence")
        out = torch.empty_like(xv)
        _lib.call("xops_causal_conv1d_update_v2_slots", xv.data_ptr(), conv_state.data_ptr(),
                  weight.contiguous().data_ptr(), _ptr(b), _ptr(idx),
                  idx.stride(0) if idx is not None else 0, _ptr(acc), _ptr(ini), _ptr(last),
                  qsl.data_ptr(), out.data_ptr(), batch, dim, width, conv_state.size(2),
                  conv_state.size(0), int(bool(activation)), int(pad_slot_id),
                  _dt(xv, "causal_conv1d_update_v2"), _stream(x))
        if query_start_loc is not None:
            return out
        out = out.view(batch, -1, dim).transpose(1, 2)
        return out.squeeze(-1) if unsq else out
    if idx is not None:
        if idx.dim() == 2:
            idx = idx[:, 0].contiguous()
        _check(idx.numel() == batch,
               f"conv_state_indices batch mismatch. Expected {batch}, got {idx.numel()}")
    out = torch.empty_like(xv)
    if width == 1:  # no history: pointwise scale + bias
        y = xv.float() * weight[:, 0].float() + (b.float() if b is not None else 0.0)
        out = (torch.nn.functional.silu(y) if activation else y).to(xv.dtype)
    else:
        _lib.call("xops_causal_conv1d_varlen", xv.data_ptr(), conv_state.data_ptr(),
                  weight.contiguous().data_ptr(), _ptr(b), qsl.data_ptr(), _ptr(idx),
                  out.data_ptr(), batch, xv.size(0), dim, width, conv_state.size(0),
                  int(bool(activation)), int(pad_slot_id), _dt(xv, "causal_conv1d_update_v2"),
                  _stream(x))
    if query_start_loc is not None:
        return out
    out = out.view(batch, -1, dim).transpose(1, 2)
    return out.squeeze(-1) if unsq else out


def causal_conv1d_varlen_qk_l2norm(x, conv_state, weight, bias, query_start_loc, qk_channels,
                                   activation=True, eps=1e-6, conv_state_indices=None,
                                   pad_slot_id=-1):
    """The GDN layer's prefill conv with its q/k L2 normalisation fused in.

    Computes ``npu_causal_conv1d_update_v2(x, conv_state, weight, activation,
    bias, conv_state_indices, query_start_loc)`` (x [num_tokens, dim]
    token-major, conv_state updated IN PLACE) and, in the same kernel,
    L2-normalises the first ``qk_channels`` output channels per 128-channel
    head, as ``npu_l2norm_last_dim`` would on the q and k blocks
    (npu_triton_chunk_gated_delta_rule.cpp:608-609).  Feed views of the
    result to ``npu_chunk_gated_delta_rule`` with
    ``use_qk_l2norm_in_kernel=False``.  bf16 / fp16 only."""
    _cuda(x, conv_state, weight, bias, query_start_loc, conv_state_indices)
    _check(x.dim() == 2 and weight.dim() == 2 and conv_state.dim() == 3,
           "causal_conv1d_varlen_qk_l2norm expects x [tokens, dim], weight [dim, width], "
           "conv_state [lines, dim, width - 1]")
    _check(x.dtype in (torch.bfloat16, torch.float16),
           "causal_conv1d_varlen_qk_l2norm expects bf16 or fp16 activations")
    dim, width = x.size(1), weight.size(1)
    _check(weight.size(0) == dim and conv_state.size(1) == dim and conv_state.size(2) >= width - 1,
           "causal_conv1d_varlen_qk_l2norm: shape mismatch")
    _check(conv_state.is_contiguous() and conv_state.dtype == x.dtype,
           "causal_conv1d_varlen_qk_l2norm: conv_state must be contiguous in x's dtype")
    xv = x.contiguous()
    qsl = _i32(query_start_loc)
    idx = _i32(conv_state_indices)
    batch = qsl.numel() - 1
    b = bias.to(x.dtype).contiguous() if bias is not None else None
    out = torch.empty_like(xv)
    _lib.call("xops_causal_conv1d_varlen_qk_l2norm", xv.data_ptr(), conv_state.data_ptr(),
              weight.to(x.dtype).contiguous().data_ptr(), _ptr(b), qsl.data_ptr(), _ptr(idx),
              out.data_ptr(), batch, xv.size(0), dim, width, conv_state.size(0),
              int(bool(activation)), int(pad_slot_id), _dt(xv, "causal_conv1d_varlen_qk_l2norm"),
              int(qk_channels), float(eps), _stream(x))
    return out


def causal_conv1d_varlen_qkvz(mixed_qkvz, conv_state, weight, bias, query_start_loc,
                              num_k_heads, num_v_heads, activation=True, qk_l2norm=True, eps=1e-6,
                              conv_state_indices=None, pad_slot_id=-1):
    """The GDN layer's prefill conv fed straight from its input projection.

    ``mixed_qkvz [num_tokens, num_k_heads * (2 + 2r) * 128]`` holds, per key
    head, q | k | v (r value heads) | z (r heads), r = num_v_heads /
    num_k_heads (the input of ``npu_fused_qkvzba_split_reshape_cat``).  The
    result equals that split's ``mixed_qkv`` through
    ``causal_conv1d_varlen_qk_l2norm`` (q/k L2-normalised when
    ``qk_l2norm``), computed without materialising ``mixed_qkv``.  Returns
    the conv output ``[num_tokens, (2 num_k_heads + num_v_heads) * 128]``;
    conv_state (``[lines, dim, width - 1]``) is updated in place."""
    _cuda(mixed_qkvz, conv_state, weight, bias, query_start_loc, conv_state_indices)
    _check(mixed_qkvz.dim() == 2 and mixed_qkvz.stride(1) == 1,
           "causal_conv1d_varlen_qkvz expects mixed_qkvz [tokens, cols] with contiguous rows")
    _check(mixed_qkvz.dtype in (torch.bfloat16, torch.float16),
           "causal_conv1d_varlen_qkvz expects bf16 or fp16 activations")
    _check(num_v_heads % num_k_heads == 0, "num_v_heads must be a multiple of num_k_heads")
    r = num_v_heads // num_k_heads
    _check(mixed_qkvz.size(1) == num_k_heads * (2 + 2 * r) * 128,
           "mixed_qkvz must hold num_k_heads * (2 + 2r) * 128 columns")
    dim, width = (2 * num_k_heads + num_v_heads) * 128, weight.size(1)
    _check(weight.size(0) == dim and conv_state.size(1) == dim and conv_state.size(2) >= width - 1,
           "causal_conv1d_varlen_qkvz: shape mismatch")
    _check(conv_state.is_contiguous() and conv_state.dtype == mixed_qkvz.dtype,
           "causal_conv1d_varlen_qkvz: conv_state must be contiguous in x's dtype")
    qsl = _i32(query_start_loc)
    idx = _i32(conv_state_indices)
    batch = qsl.numel() - 1
    b = bias.to(mixed_qkvz.dtype).contiguous() if bias is not None else None
    T = mixed_qkvz.size(0)
    out = torch.empty((T, dim), dtype=mixed_qkvz.dtype, device=mixed_qkvz.device)
    _lib.call("xops_causal_conv1d_varlen_qkvz", mixed_qkvz.data_ptr(), mixed_qkvz.stride(0),
              num_k_heads, num_v_heads, conv_state.data_ptr(),
              weight.to(mixed_qkvz.dtype).contiguous().data_ptr(), _ptr(b), qsl.data_ptr(),
              _ptr(idx), out.data_ptr(), batch, T, width, conv_state.size(0),
              int(bool(activation)), int(pad_slot_id), _dt(mixed_qkvz, "causal_conv1d_varlen_qkvz"),
              int(bool(qk_l2norm)), float(eps), _stream(mixed_qkvz))
    return out


# ---------------------------------------------------------- gated delta rule
def _seq_info(q, cu_seqlens):
    b, t = q.shape[0], q.shape[1]
    if cu_seqlens is None:
        return None, b, t, b
    _check(b == 1, "variable-length mode expects batch size B=1")
    cu = _i32(cu_seqlens)
    return cu, b, t, cu.numel() - 1


def npu_fused_recurrent_gated_delta_rule(q, k, v, g, beta=None, scale=None, initial_state=None,
                                         inplace_final_state=True, cu_seqlens=None,
                                         ssm_state_indices=None, num_accepted_tokens=None,
                                         use_qk_l2norm_in_kernel=False):
    """Token-serial gated delta rule; returns ``(o, final_state)``
    (npu_triton_recurrent_gated_delta_rule.cpp:54-246).  ``initial_state``
    is required.  ``ssm_state_indices`` is ``[N]`` (one slot per sequence)
    or ``[N, T]`` (one slot per token).  With ``inplace_final_state`` the
    states go back into ``initial_state``: per token for a ``[N, T]`` table
    or under speculative decoding (``num_accepted_tokens`` given: the initial
    state is token ``num_accepted_tokens[n] - 1``'s slot), else the final
    state to the sequence's slot."""
    spec = num_accepted_tokens is not None
    if cu_seqlens is None:
        _check(q.shape[0] == 1, "batch size is not 1 when cu_seqlens is not provided")
    _check(initial_state is not None,
           "initial_state must be provided when inplace_final_state is "
           + ("true" if inplace_final_state else "false"))
    if spec:
        _check(cu_seqlens is not None, "cu_seqlens must be provided for spec decoding")
        _check(ssm_state_indices is not None,
               "ssm_state_indices must be provided for spec decoding")
    _cuda(q, k, v, g, beta, initial_state, cu_seqlens, ssm_state_indices, num_accepted_tokens)
    _check(q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16,
           "npu_fused_recurrent_gated_delta_rule expects q/k/v to be bfloat16")
    _check(initial_state.dtype == torch.float32, "initial_state must be float32")
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    _check(q.shape == k.shape and v.shape[:2] == (B, T), "q/k/v shape mismatch")
    scale = float(scale) if scale is not None else 1.0 / math.sqrt(K)
    cu = _i32(cu_seqlens)
    N = cu.numel() - 1 if cu is not None else B
    gg = g.to(torch.float32).contiguous()
    bb = beta.to(torch.float32).contiguous() if beta is not None else None
    idx = ssm_state_indices
    ss = st = 0
    if idx is not None:
        _check(idx.dim() in (1, 2), "ssm_state_indices must be 1D or 2D")
        idx = idx if idx.dtype == torch.int32 else idx.to(torch.int32)
        _check(idx.shape[0] == N, "ssm_state_indices must have one row per sequence")
        ss = idx.stride(0)
        # a [N] table under speculative decoding is addressed like the
        # reference's (token stride 1); otherwise one slot per sequence
        st = idx.stride(1) if idx.dim() == 2 else (1 if spec else 0)
    acc = _i32(num_accepted_tokens)
    if acc is not None:
        _check(acc.numel() == N, "num_accepted_tokens must have one entry per sequence")
    _check(initial_state.is_contiguous() or initial_state.stride(0) >= HV * K * V,
           "initial_state slots must be contiguous")
    _check(initial_state.shape[1:] == (HV, K, V), "initial_state must be [slots, HV, K, V]")
    if inplace_final_state:
        final = initial_state
    else:
        final = torch.empty((N, HV, K, V), dtype=torch.float32, device=q.device)
    o = torch.empty((B, T, HV, V), dtype=q.dtype, device=q.device)
    qc, kc, vc = q.contiguous(), k.contiguous(), v.contiguous()
    _lib.call("xops_fused_recurrent_gated_delta_rule", qc.data_ptr(), kc.data_ptr(), vc.data_ptr(),
              gg.data_ptr(), _ptr(bb), o.data_ptr(), initial_state.data_ptr(), final.data_ptr(),
              _ptr(cu), _ptr(idx), ss, st, _ptr(acc),
              B, T, N, H, HV, K, V, initial_state.stride(0), final.stride(0), scale,
              int(bool(use_qk_l2norm_in_kernel)), _stream(q))
    return o, final


def npu_fused_qkvzba_split_reshape_cat(mixed_qkvz, mixed_ba, num_heads_qk, num_heads_v,
                                       head_qk, head_v):
    """De-interleave the GDN input projections into ``(mixed_qkv [rows,
    2 nqk hqk + nv hv], z [rows, nv, hv], b [rows, nv], a [rows, nv])``
    (npu_triton_fused_qkvzba_split_reshape.cpp:105-206)."""
    _cuda(mixed_qkvz, mixed_ba)
    rows = mixed_qkvz.shape[0]
    r = num_heads_v // num_heads_qk
    _check(1 <= r <= 4, "npu_fused_qkvzba_split_reshape_cat only supports v_heads_per_qk in "
           f"[1, 4], but got {r} for num_heads_qk={num_heads_qk} num_heads_v={num_heads_v}")
    qkvz = mixed_qkvz.contiguous()
    ba = mixed_ba.contiguous()
    _check(qkvz.numel() == rows * num_heads_qk * (2 * head_qk + 2 * r * head_v)
           and ba.numel() == rows * num_heads_qk * 2 * r,
           "npu_fused_qkvzba_split_reshape_cat: projection widths do not match the head counts")
    qkv = torch.empty((rows, 2 * num_heads_qk * head_qk + num_heads_v * head_v),
                      dtype=qkvz.dtype, device=qkvz.device)
    z = torch.empty((rows, num_heads_v, head_v), dtype=qkvz.dtype, device=qkvz.device)
    b = torch.empty((rows, num_heads_v), dtype=ba.dtype, device=ba.device)
    a = torch.empty((rows, num_heads_v), dtype=ba.dtype, device=ba.device)
    _lib.call("xops_fused_qkvzba_split_reshape_cat", qkvz.data_ptr(), ba.data_ptr(),
              qkv.data_ptr(), z.data_ptr(), b.data_ptr(), a.data_ptr(), rows, num_heads_qk,
              num_heads_v, head_qk, head_v, _dt(qkvz, "npu_fused_qkvzba_split_reshape_cat"),
              _dt(ba, "npu_fused_qkvzba_split_reshape_cat"), _stream(qkvz))
    return qkv, z, b, a


def npu_fused_gdn_gating(A_log, a, b, dt_bias, beta=1.0, threshold=20.0):
    """GDN gates from the projections: ``g = -exp(A_log) * softplus(a +
    dt_bias)`` (fp32) and ``beta_output = sigmoid(b)`` (b's dtype), both
    ``[1, batch, heads]`` (npu_triton_fused_gdn_gating.cpp:33-93)."""
    for t, name in ((A_log, "A_log"), (a, "a"), (b, "b"), (dt_bias, "dt_bias")):
        _check(t is not None, f"{name} tensor is not defined")
        _check(t.is_contiguous(), f"{name} tensor must be contiguous")
    _cuda(A_log, a, b, dt_bias)
    _check(A_log.dtype == torch.float32, "A_log must be float32")
    _check(dt_bias.dtype == torch.float32, "dt_bias must be float32")
    _check(A_log.dim() == 1, "A_log must be 1D tensor")
    _check(a.dim() == 2, "a must be 2D tensor (batch, num_heads)")
    _check(b.dim() == 2, "b must be 2D tensor (batch, num_heads)")
    _check(dt_bias.dim() == 1, "dt_bias must be 1D tensor")
    batch, heads = a.shape
    _check(b.shape == a.shape, "a and b must have the same shape")
    _check(A_log.numel() == heads and dt_bias.numel() == heads,
           "A_log and dt_bias must have num_heads elements")
    g = torch.empty((1, batch, heads), dtype=torch.float32, device=a.device)
    beta_output = torch.empty((1, batch, heads), dtype=b.dtype, device=b.device)
    _lib.call("xops_fused_gdn_gating", A_log.data_ptr(), a.data_ptr(), b.data_ptr(),
              dt_bias.data_ptr(), g.data_ptr(), beta_output.data_ptr(), batch, heads,
              _dt(a, "npu_fused_gdn_gating"), _dt(b, "npu_fused_gdn_gating"), float(beta),
              float(threshold), _stream(a))
    return g, beta_output


def npu_fused_sigmoid_gating_delta_rule_update(A_log, a, dt_bias, q, k, v, b,
                                               initial_state_source, initial_state_indices,
                                               cu_seqlens, scale=None,
                                               use_qk_l2norm_in_kernel=False, softplus_beta=1.0,
                                               softplus_threshold=20.0):
    """Recurrent gated delta rule with the gates computed from the
    projections in the step; updates ``initial_state_source`` in place (slot
    ``initial_state_indices[n]``; a negative index starts from zeros and
    writes nothing) and returns ``o [B, T, HV, V]``
    (npu_triton_fused_sigmoid_gating_delta_rule_update.cpp:54-179)."""
    named = (("A_log", A_log), ("a", a), ("dt_bias", dt_bias), ("q", q), ("k", k), ("v", v),
             ("b", b), ("initial_state_source", initial_state_source),
             ("initial_state_indices", initial_state_indices), ("cu_seqlens", cu_seqlens))
    for name, t in named:
        _check(t is not None, f"{name} must be defined")
        _check(t.is_contiguous(), f"{name} must be contiguous")
    _cuda(*[t for _, t in named])
    _check(q.dim() == 4, "q must be 4D [B, T, H, K]")
    _check(k.dim() == 4, "k must be 4D [B, T, H, K]")
    _check(v.dim() == 4, "v must be 4D [B, T, HV, V]")
    _check(a.dim() == 3, "a must be 3D [B, T, HV]")
    _check(b.dim() == 3, "b must be 3D [B, T, HV]")
    _check(A_log.dim() == 1, "A_log must be 1D [HV]")
    _check(dt_bias.dim() == 1, "dt_bias must be 1D [HV]")
    _check(initial_state_source.dim() == 4,
           "initial_state_source must be 4D [slots, HV, K, V]")
    _check(initial_state_indices.dim() == 1, "initial_state_indices must be 1D [N]")
    _check(cu_seqlens.dim() == 1, "cu_seqlens must be 1D [N + 1]")
    B, T, H, K = k.shape
    HV, V = v.shape[2], v.shape[3]
    N = cu_seqlens.numel() - 1
    _check(q.shape == k.shape, "q/k shape mismatch")
    _check(v.shape[0] == B and v.shape[1] == T, "v B/T mismatch")
    _check(a.shape == (B, T, HV), "a shape mismatch")
    _check(b.shape == a.shape, "a/b shape mismatch")
    _check(A_log.numel() == HV, "A_log HV mismatch")
    _check(dt_bias.numel() == HV, "dt_bias HV mismatch")
    _check(initial_state_source.shape[1:] == (HV, K, V), "initial_state_source shape mismatch")
    _check(initial_state_indices.numel() == N,
           "initial_state_indices size must equal cu_seqlens size - 1")
    _check(HV % H == 0, "HV must be divisible by H")
    _check(A_log.dtype == torch.float32, "A_log must be float32")
    _check(dt_bias.dtype == torch.float32, "dt_bias must be float32")
    _check(initial_state_source.dtype == torch.float32, "initial_state_source must be float32")
    _check(initial_state_indices.dtype == torch.int32, "initial_state_indices must be int32")
    _check(cu_seqlens.dtype == torch.int32, "cu_seqlens must be int32")
    _check(q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16,
           "npu_fused_sigmoid_gating_delta_rule_update expects q/k/v to be bfloat16")
    _check(a.dtype == b.dtype, "a and b must have the same dtype")
    scale = float(scale) if scale is not None else 1.0 / math.sqrt(K)
    o = torch.empty((B, T, HV, V), dtype=q.dtype, device=q.device)
    _lib.call("xops_fused_sigmoid_gating_delta_rule_update", A_log.data_ptr(), a.data_ptr(),
              dt_bias.data_ptr(), float(softplus_beta), float(softplus_threshold), q.data_ptr(),
              k.data_ptr(), v.data_ptr(), b.data_ptr(), o.data_ptr(),
              initial_state_source.data_ptr(), initial_state_indices.data_ptr(),
              cu_seqlens.data_ptr(), scale, B, T, N, H, HV, K, V,
              _dt(a, "npu_fused_sigmoid_gating_delta_rule_update"),
              int(bool(use_qk_l2norm_in_kernel)), _stream(q))
    return o


def _token_rows(x, B):
    """x [B, T, H, D] as rows of tokens: heads and dims contiguous inside a
    token, any 16-byte aligned token stride (slices of a packed projection
    need no copy); otherwise a contiguous copy."""
    ok = (x.stride(3) == 1 and x.stride(2) == x.shape[3] and x.stride(1) % 8 == 0
          and (B == 1 or x.stride(0) == x.shape[1] * x.stride(1)) and x.data_ptr() % 16 == 0)
    return x if ok else x.contiguous()


def npu_chunk_gated_delta_rule(q, k, v, g, beta, scale=None, initial_state=None,
                               output_final_state=False, cu_seqlens=None, head_first=False,
                               use_qk_l2norm_in_kernel=False):
    """Chunked gated delta rule prefill, fused into one kernel; returns
    ``(o, final_state or None)`` (npu_triton_chunk_gated_delta_rule.cpp:556-642).
    ``initial_state`` (bf16 or fp32) is read, never modified."""
    _check(not head_first, "chunk_gated_delta_rule torch_api only supports head_first=false.")
    _check(q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16,
           "chunk_gated_delta_rule expects q/k/v to be bfloat16.")
    if initial_state is not None:
        _check(initial_state.dtype in (torch.bfloat16, torch.float32),
               "chunk_gated_delta_rule expects initial_state to be bfloat16 or float32, got "
               f"{initial_state.dtype}")
    _cuda(q, k, v, g, beta, initial_state, cu_seqlens)
    B, T, Hg, K = q.shape
    H, V = v.shape[2], v.shape[3]
    _check(q.shape == k.shape, "q and k must have the same shape.")
    _check(H % Hg == 0, "chunk_gated_delta_rule expects num_heads_v to be divisible by "
                        f"num_heads_qk, got {H} and {Hg}")
    _check(beta.dim() == 3 and tuple(beta.shape) == (B, T, H), "beta must have shape [B, T, H].")
    _check(g.dim() == 3 and tuple(g.shape) == (B, T, H), "g must have shape [B, T, H].")
    cu, _, _, N = _seq_info(q, cu_seqlens)
    scale_v = float(scale) if scale is not None else K ** -0.5
    h0 = initial_state.to(torch.float32).contiguous() if initial_state is not None else None
    if h0 is not None:
        _check(tuple(h0.shape) == (N, H, K, V), "initial_state must have shape [N, H, K, V]")
    o = torch.empty((B, T, H, V), dtype=v.dtype, device=v.device)
    ht = torch.empty((N, H, K, V), dtype=torch.float32, device=v.device) if output_final_state else None
    qc, kc, vc = _token_rows(q, B), _token_rows(k, B), _token_rows(v, B)
    gg, bb = g.to(torch.float32).contiguous(), beta.to(torch.float32).contiguous()
    l2 = int(bool(use_qk_l2norm_in_kernel))
    wsb = _lib.load().xops_chunk_gated_delta_rule_workspace_size(B, T, N, Hg, H, K, l2,
                                                                 int(cu is not None))
    ws = torch.empty(max(int(wsb), 16), dtype=torch.uint8, device=q.device)
    _lib.call("xops_chunk_gated_delta_rule", qc.data_ptr(), kc.data_ptr(), vc.data_ptr(),
              gg.data_ptr(), bb.data_ptr(), _ptr(h0), o.data_ptr(), _ptr(ht), _ptr(cu), B, T, N,
              Hg, H, K, V, qc.stride(1), kc.stride(1), vc.stride(1), scale_v, l2, ws.data_ptr(),
              ws.numel(), _stream(q))
    return o, ht


def chunk_gated_delta_rule_out_norm(q, k, v, g, beta, z, norm_weight, scale=None,
                                    initial_state=None, output_final_state=False,
                                    cu_seqlens=None, use_qk_l2norm_in_kernel=False, eps=1e-6,
                                    return_o=False):
    """``npu_chunk_gated_delta_rule`` followed by the GDN layer's output norm
    ``layer_norm_fwd(o, norm_weight, None, eps, z, V, norm_before_gate=True,
    is_rms_norm=True)`` (npu_triton_layernorm_fwd.cpp:48-333) as one call:
    the chain kernel normalises each (token, head) row of its bf16 output as
    it writes it, so o makes no round trip through HBM.  z: ``[B, T, H, V]``
    (or any shape of those elements with V contiguous and a token stride),
    bf16; norm_weight ``[V]`` fp32 or bf16.  Returns ``(y [B, T, H, V],
    final_state or None, o or None)``; o (the rule's own output) is written
    only with ``return_o``."""
    _check(q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16
           and z.dtype == torch.bfloat16,
           "chunk_gated_delta_rule_out_norm expects q/k/v/z to be bfloat16.")
    _check(norm_weight.dtype in (torch.float32, torch.bfloat16),
           "chunk_gated_delta_rule_out_norm: norm weight must be fp32 or bf16")
    if initial_state is not None:
        _check(initial_state.dtype in (torch.bfloat16, torch.float32),
               "chunk_gated_delta_rule expects initial_state to be bfloat16 or float32, got "
               f"{initial_state.dtype}")
    _cuda(q, k, v, g, beta, z, norm_weight, initial_state, cu_seqlens)
    B, T, Hg, K = q.shape
    H, V = v.shape[2], v.shape[3]
    _check(q.shape == k.shape, "q and k must have the same shape.")
    _check(H % Hg == 0, "chunk_gated_delta_rule expects num_heads_v to be divisible by "
                        f"num_heads_qk, got {H} and {Hg}")
    _check(beta.dim() == 3 and tuple(beta.shape) == (B, T, H), "beta must have shape [B, T, H].")
    _check(g.dim() == 3 and tuple(g.shape) == (B, T, H), "g must have shape [B, T, H].")
    _check(z.numel() == B * T * H * V and norm_weight.numel() == V,
           "chunk_gated_delta_rule_out_norm: z must hold [B, T, H, V] and the weight [V]")
    cu, _, _, N = _seq_info(q, cu_seqlens)
    scale_v = float(scale) if scale is not None else K ** -0.5
    h0 = initial_state.to(torch.float32).contiguous() if initial_state is not None else None
    if h0 is not None:
        _check(tuple(h0.shape) == (N, H, K, V), "initial_state must have shape [N, H, K, V]")
    zr = z.reshape(B * T, H * V)
    if zr.stride(1) != 1 or zr.stride(0) % 8 or zr.data_ptr() % 16:
        zr = zr.contiguous()
    w = norm_weight.contiguous()
    y = torch.empty((B, T, H, V), dtype=v.dtype, device=v.device)
    o = torch.empty((B, T, H, V), dtype=v.dtype, device=v.device) if return_o else None
    ht = torch.empty((N, H, K, V), dtype=torch.float32, device=v.device) if output_final_state else None
    qc, kc, vc = _token_rows(q, B), _token_rows(k, B), _token_rows(v, B)
    gg, bb = g.to(torch.float32).contiguous(), beta.to(torch.float32).contiguous()
    l2 = int(bool(use_qk_l2norm_in_kernel))
    wsb = _lib.load().xops_chunk_gated_delta_rule_workspace_size(B, T, N, Hg, H, K, l2,
                                                                 int(cu is not None))
    ws = torch.empty(max(int(wsb), 16), dtype=torch.uint8, device=q.device)
    _lib.call("xops_chunk_gated_delta_rule_out_norm", qc.data_ptr(), kc.data_ptr(), vc.data_ptr(),
              gg.data_ptr(), bb.data_ptr(), _ptr(h0), _ptr(o), _ptr(ht), _ptr(cu), B, T, N, Hg, H,
              K, V, qc.stride(1), kc.stride(1), vc.stride(1), scale_v, l2, zr.data_ptr(),
              zr.stride(0), w.data_ptr(), _dt(w, "chunk_gated_delta_rule_out_norm"), float(eps),
              y.data_ptr(), ws.data_ptr(), ws.numel(), _stream(q))
    return y, ht, o


def chunk_gated_delta_rule_gated(q, k, v, A_log, a, b, dt_bias, scale=None, initial_state=None,
                                 output_final_state=False, cu_seqlens=None,
                                 use_qk_l2norm_in_kernel=False, softplus_beta=1.0,
                                 softplus_threshold=20.0, mixed_ba=None):
    """``npu_fused_gdn_gating`` followed by ``npu_chunk_gated_delta_rule`` as
    one call: the gates ``g = -exp(A_log) * softplus(a + dt_bias)`` and
    ``beta = sigmoid(b)`` (rounded to b's dtype) are computed inside the
    chunked rule's kernels from a, b ``[B, T, H]`` (or ``[T, H]`` with B = 1)
    and A_log, dt_bias ``[H]`` fp32, with the same arithmetic as the gating
    operator (npu_triton_fused_gdn_gating.cpp:33-93), so the result equals
    the two-call sequence bit for bit.  With ``mixed_ba [T, Hg * 2r]`` (the
    un-split projection: per key head b (r heads) | a (r heads)) a and b are
    None and the gates are read from it in place.  Returns
    ``(o, final_state or None)``."""
    o, ht, _ = _chunk_gated_call(q, k, v, A_log, a, b, dt_bias, scale, initial_state,
                                 output_final_state, cu_seqlens, use_qk_l2norm_in_kernel,
                                 softplus_beta, softplus_threshold, mixed_ba, None)
    return o, ht


def chunk_gated_delta_rule_gated_out_norm(q, k, v, A_log, a, b, dt_bias, z, norm_weight,
                                          scale=None, initial_state=None,
                                          output_final_state=False, cu_seqlens=None,
                                          use_qk_l2norm_in_kernel=False, eps=1e-6,
                                          softplus_beta=1.0, softplus_threshold=20.0,
                                          mixed_ba=None, z_heads_per_group=1,
                                          z_group_stride=None, return_o=False):
    """``chunk_gated_delta_rule_gated`` followed by the layer's gated RMSNorm
    ``layer_norm_fwd(o, norm_weight, None, eps, z, V, True, True)`` as one
    call (the norm inside the chain kernel, as in
    ``chunk_gated_delta_rule_out_norm``).  z: a bf16 view whose first
    element is the gate of token 0, head 0; head h of token t starts
    ``t * z.stride(0) + (h // z_heads_per_group) * z_group_stride +
    (h % z_heads_per_group) * V`` elements further on (z_group_stride
    defaults to z_heads_per_group * V), so it can be read in place from the
    layer's projection.  Returns ``(y [B, T, H, V], final_state or None, o
    or None)``."""
    _check(z.dtype == torch.bfloat16 and z.stride(-1) == 1,
           "chunk_gated_delta_rule_gated_out_norm: z must be bf16 with unit inner stride")
    _check(norm_weight.dtype in (torch.float32, torch.bfloat16),
           "chunk_gated_delta_rule_out_norm: norm weight must be fp32 or bf16")
    _cuda(z, norm_weight)
    V = v.shape[3]
    zr = int(z_heads_per_group)
    zgs = int(z_group_stride) if z_group_stride is not None else zr * V
    w = norm_weight.contiguous()
    _check(w.numel() == V, "chunk_gated_delta_rule_out_norm: the weight must have V elements")
    norm = (z, z.stride(0), zr, zgs, w, float(eps), bool(return_o))
    o, ht, y = _chunk_gated_call(q, k, v, A_log, a, b, dt_bias, scale, initial_state,
                                 output_final_state, cu_seqlens, use_qk_l2norm_in_kernel,
                                 softplus_beta, softplus_threshold, mixed_ba, norm)
    return y, ht, o


def _chunk_gated_call(q, k, v, A_log, a, b, dt_bias, scale, initial_state, output_final_state,
                      cu_seqlens, use_qk_l2norm_in_kernel, softplus_beta, softplus_threshold,
                      mixed_ba, norm):
    _check(q.dtype == torch.bfloat16 and k.dtype == torch.bfloat16 and v.dtype == torch.bfloat16,
           "chunk_gated_delta_rule expects q/k/v to be bfloat16.")
    _cuda(q, k, v, A_log, a, b, dt_bias, initial_state, cu_seqlens)
    B, T, Hg, K = q.shape
    H, V = v.shape[2], v.shape[3]
    _check(q.shape == k.shape, "q and k must have the same shape.")
    _check(H % Hg == 0, "chunk_gated_delta_rule expects num_heads_v to be divisible by "
                        f"num_heads_qk, got {H} and {Hg}")
    if mixed_ba is not None:
        _check(a is None and b is None, "pass either a and b or mixed_ba")
        _check(B == 1 and mixed_ba.dim() == 2 and tuple(mixed_ba.shape) == (T, 2 * H)
               and mixed_ba.stride(1) == 1, "mixed_ba must have shape [T, 2 H] with contiguous rows")
        _cuda(mixed_ba)
        a3 = b3 = mixed_ba
    else:
        a3 = a if a.dim() == 3 else a.unsqueeze(0)
        b3 = b if b.dim() == 3 else b.unsqueeze(0)
        _check(tuple(a3.shape) == (B, T, H) and tuple(b3.shape) == (B, T, H),
               "a and b must have shape [B, T, H] (or [T, H] with B == 1)")
    _check(A_log.dtype == torch.float32 and dt_bias.dtype == torch.float32,
           "A_log and dt_bias must be float32")
    _check(A_log.numel() == H and dt_bias.numel() == H, "A_log and dt_bias must have H elements")
    if initial_state is not None:
        _check(initial_state.dtype in (torch.bfloat16, torch.float32),
               "chunk_gated_delta_rule expects initial_state to be bfloat16 or float32, got "
               f"{initial_state.dtype}")
    cu, _, _, N = _seq_info(q, cu_seqlens)
    scale_v = float(scale) if scale is not None else K ** -0.5
    h0 = initial_state.to(torch.float32).contiguous() if initial_state is not None else None
    if h0 is not None:
        _check(tuple(h0.shape) == (N, H, K, V), "initial_state must have shape [N, H, K, V]")
    want_o = norm is None or norm[6]
    o = torch.empty((B, T, H, V), dtype=v.dtype, device=v.device) if want_o else None
    ht = torch.empty((N, H, K, V), dtype=torch.float32, device=v.device) if output_final_state else None
    qc, kc, vc = _token_rows(q, B), _token_rows(k, B), _token_rows(v, B)
    if mixed_ba is not None:
        ac = bc = mixed_ba
        ab_ld, inter = mixed_ba.stride(0), 1
    else:
        ac, bc = a3.contiguous(), b3.contiguous()
        ab_ld, inter = H, 0
    Al, dtb = A_log.contiguous(), dt_bias.contiguous()
    l2 = int(bool(use_qk_l2norm_in_kernel))
    wsb = _lib.load().xops_chunk_gated_delta_rule_workspace_size(B, T, N, Hg, H, K, l2,
                                                                 int(cu is not None))
    ws = torch.empty(max(int(wsb), 16), dtype=torch.uint8, device=q.device)
    head = (qc.data_ptr(), kc.data_ptr(), vc.data_ptr(), Al.data_ptr(), ac.data_ptr(),
            bc.data_ptr(), dtb.data_ptr(), _dt(ac, "chunk_gated_delta_rule_gated"),
            _dt(bc, "chunk_gated_delta_rule_gated"), ab_ld, inter, float(softplus_beta),
            float(softplus_threshold), _ptr(h0), _ptr(o), _ptr(ht), _ptr(cu), B, T, N, Hg, H, K, V,
            qc.stride(1), kc.stride(1), vc.stride(1), scale_v, l2)
    if norm is None:
        _lib.call("xops_chunk_gated_delta_rule_gated", *head, ws.data_ptr(), ws.numel(),
                  _stream(q))
        return o, ht, None
    z, zld, zr, zgs, w, eps, _ = norm
    y = torch.empty((B, T, H, V), dtype=v.dtype, device=v.device)
    _lib.call("xops_chunk_gated_delta_rule_gated_out_norm", *head, z.data_ptr(), zld, zr, zgs,
              w.data_ptr(), _dt(w, "chunk_gated_delta_rule_out_norm"), eps, y.data_ptr(),
              ws.data_ptr(), ws.numel(), _stream(q))
    return o, ht, y


# ---- chunk pipeline sub-operators (reference decomposition, chunk.py:31-73)
def _ncu(q_like, cu_seqlens):
    cu, b, t, n = _seq_info(q_like, cu_seqlens)
    return cu, b, t, n


def npu_chunk_local_cumsum(g, chunk_size, cu_seqlens=None):
    """Per-chunk inclusive cumsum of g [B, T, H] (fp32 out)
    (npu_triton_chunk_gated_delta_rule.cpp:151-227)."""
    gf = g.to(torch.float32).contiguous()
    _check(gf.dim() == 3, "chunk_local_cumsum expects g to have shape [B, T, H].")
    _check(chunk_size > 0 and (chunk_size & (chunk_size - 1)) == 0,
           f"chunk_local_cumsum expects chunk_size to be a power of two, got {chunk_size}")
    _cuda(gf, cu_seqlens)
    cu, B, T, N = _ncu(gf, cu_seqlens)
    out = torch.empty_like(gf)
    _lib.call("xops_chunk_local_cumsum", gf.data_ptr(), out.data_ptr(), _ptr(cu), B, T, N,
              gf.shape[2], chunk_size, _stream(gf))
    return out


def npu_chunk_scaled_dot_kkt_fwd(k, beta, g_cumsum, chunk_size, cu_seqlens=None):
    """A [B, T, H, 64] fp32 = strict_tril(beta_i e^{g_i-g_j} k_i.k_j)
    (npu_triton_chunk_gated_delta_rule.cpp:229-297)."""
    _cuda(k, beta, g_cumsum, cu_seqlens)
    _check(k.dtype == torch.bfloat16, "chunk_scaled_dot_kkt_fwd expects bf16 k")
    B, T, Hg, K = k.shape
    H = beta.shape[-1]
    cu, _, _, N = _ncu(k, cu_seqlens)
    A = torch.zeros((B, T, H, chunk_size), dtype=torch.float32, device=k.device)
    bb = beta.to(torch.float32).contiguous()
    gc = g_cumsum.to(torch.float32).contiguous() if g_cumsum is not None else None
    _lib.call("xops_chunk_scaled_dot_kkt_fwd", k.contiguous().data_ptr(), bb.data_ptr(), _ptr(gc),
              A.data_ptr(), _ptr(cu), B, T, N, Hg, H, K, chunk_size, _stream(k))
    return A


def npu_solve_tril(A, chunk_size, cu_seqlens=None, output_dtype=torch.bfloat16):
    """(I + A_c)^-1 per chunk, [B, T, H, 64] in ``output_dtype``
    (npu_triton_chunk_gated_delta_rule.cpp:299-395)."""
    _cuda(A, cu_seqlens)
    Af = A.to(torch.float32).contiguous()
    B, T, H, BT = Af.shape
    cu, _, _, N = _ncu(Af, cu_seqlens)
    Ai = torch.zeros((B, T, H, BT), dtype=output_dtype, device=A.device)
    _lib.call("xops_solve_tril", Af.data_ptr(), Ai.data_ptr(), _ptr(cu), B, T, N, H, chunk_size,
              _dt(Ai, "solve_tril"), _stream(A))
    return Ai


def npu_recompute_w_u_fwd(k, v, beta, g_cumsum, A, cu_seqlens=None):
    """WY transform: ``w = Ai (beta e^g k)``, ``u = Ai (beta v)`` (bf16)
    (npu_triton_chunk_gated_delta_rule.cpp:397-475)."""
    _cuda(k, v, beta, g_cumsum, A, cu_seqlens)
    B, T, Hg, K = k.shape
    H, V = v.shape[2], v.shape[3]
    cu, _, _, N = _ncu(k, cu_seqlens)
    w = torch.empty((B, T, H, K), dtype=k.dtype, device=k.device)
    u = torch.empty_like(v)
    Ac = A.contiguous()
    _lib.call("xops_recompute_w_u_fwd", k.contiguous().data_ptr(), v.contiguous().data_ptr(),
              beta.to(torch.float32).contiguous().data_ptr(),
              g_cumsum.to(torch.float32).contiguous().data_ptr(), Ac.data_ptr(),
              _dt(Ac, "recompute_w_u_fwd"), w.data_ptr(), u.data_ptr(), _ptr(cu), B, T, N, Hg, H,
              K, V, _stream(k))
    return w, u


def npu_chunk_gated_delta_rule_fwd_h(k, w, u, g=None, initial_state=None,
                                     output_final_state=False, chunk_size=64, save_new_value=True,
                                     cu_seqlens=None, chunk_offsets=None):
    """Chunk-state pass; returns ``(h [B, NT, H, K, V] bf16, v_new bf16 or
    None, final_state fp32 or None)``
    (npu_triton_chunk_gated_delta_rule.cpp:644-802)."""
    _check(chunk_size == 64, "chunk_gated_delta_rule_fwd_h only supports chunk_size=64 in "
                             "the current compiled binary.")
    for t, nm in ((k, "k"), (w, "w"), (u, "u")):
        _check(t.dtype == torch.bfloat16,
               f"chunk_gated_delta_rule_fwd_h expects {nm} to be bfloat16, got {t.dtype}")
    _cuda(k, w, u, g, initial_state, cu_seqlens)
    B, T, Hg, K = k.shape
    H, V = u.shape[2], u.shape[3]
    cu, _, _, N = _ncu(k, cu_seqlens)
    if cu is not None:
        if chunk_offsets is not None:
            NT = int(chunk_offsets.reshape(-1)[-1].item())
        else:  # host copy of the offsets, as the reference does (cpp:77-113)
            cu_host = cu.cpu()
            NT = int(_lib.load().xops_total_chunks(cu_host.data_ptr(), B, T, N, 64))
    else:
        NT = (T + 63) // 64
    h = torch.empty((B, NT, H, K, V), dtype=k.dtype, device=k.device)
    v_new = torch.empty_like(u) if save_new_value else None
    ht = torch.empty((N, H, K, V), dtype=torch.float32, device=k.device) if output_final_state else None
    h0 = initial_state.to(torch.float32).contiguous() if initial_state is not None else None
    gc = g.to(torch.float32).contiguous() if g is not None else None
    _lib.call("xops_chunk_gated_delta_rule_fwd_h", k.contiguous().data_ptr(),
              w.contiguous().data_ptr(), u.contiguous().data_ptr(), _ptr(gc), _ptr(h0),
              h.data_ptr(), _ptr(v_new), _ptr(ht), _ptr(cu), B, T, N, Hg, H, K, V,
              B * NT if cu is None else NT, _stream(k))
    return h, v_new, ht


def npu_chunk_fwd_o(q, k, v, h, g_cumsum, scale, chunk_size=64, cu_seqlens=None):
    """``o = scale (q h e^g + tril(q k^T e^{g_i-g_j}) v)`` per chunk, bf16
    (npu_triton_chunk_gated_delta_rule.cpp:477-554); ``v`` is v_new and
    ``h`` the per-chunk states from ``npu_chunk_gated_delta_rule_fwd_h``."""
    _check(chunk_size == 64, "chunk_fwd_o only supports chunk_size=64")
    _cuda(q, k, v, h, g_cumsum, cu_seqlens)
    B, T, Hg, K = q.shape
    H, V = v.shape[2], v.shape[3]
    cu, _, _, N = _ncu(q, cu_seqlens)
    o = torch.empty_like(v)
    gc = g_cumsum.to(torch.float32).contiguous() if g_cumsum is not None else None
    hh = h.to(torch.bfloat16).contiguous()
    _lib.call("xops_chunk_fwd_o", q.contiguous().data_ptr(), k.contiguous().data_ptr(),
              v.contiguous().data_ptr(), hh.data_ptr(), _ptr(gc), o.data_ptr(), _ptr(cu), B, T, N,
              Hg, H, K, V, hh.shape[1], float(scale), _stream(q))
    return o
