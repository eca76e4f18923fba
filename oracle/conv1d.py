"""Depthwise causal conv1d oracles (test infrastructure only)."""

import torch
import torch.nn.functional as F

from . import _out


def _taps(hist, xs, weight, bias):
    """Depthwise causal conv of ``xs`` [dim, L] preceded by ``hist``
    [dim, width-1]; returns fp32 [dim, L]:
    ``out[:, t] = bias + sum_j weight[:, j] * cat(hist, xs)[:, t + j]`` (the
    valid cross-correlation the reference's ``F.conv1d(..., groups=dim)``
    computes, written as width shifted multiply-adds)."""
    width = weight.shape[1]
    cat = torch.cat([hist.to(torch.float32), xs.to(torch.float32)], dim=-1)
    L = xs.shape[-1]
    w = weight.to(torch.float32)
    out = (torch.zeros(cat.shape[0], L) if bias is None
           else bias.to(torch.float32)[:, None].expand(-1, L).clone())
    for j in range(width):
        out += w[:, j:j + 1] * cat[:, j:j + L]
    return out


def causal_conv1d_update(x, conv_state, weight, bias=None, activation=True,
                         conv_state_indices=None, pad_slot_id=-1):
    """Decode-style update (``causal_conv1d_update_ref``,
    triton_npu/triton_src/test_causal_conv1d_update.py:1158-1210, non-circular
    branch) with the continuous-batching slot lookup and pad-slot skip of the
    decode kernels (test_causal_conv1d_update.py:783-792, :904-912).

    x: [B, dim] or [B, dim, L]; conv_state: [lines, dim, state_len] updated IN
    PLACE (state <- last state_len columns of cat(state, x)); weight:
    [dim, width]; out = SiLU(conv + bias) in x's dtype.  Rows whose slot is
    ``pad_slot_id`` are skipped: their state is untouched and their output
    row is returned as zeros here (the kernels leave it unwritten).
    """
    squeeze = x.dim() == 2
    xs = x.unsqueeze(-1) if squeeze else x
    bsz, dim, seqlen = xs.shape
    width = weight.shape[1]
    state_len = conv_state.shape[-1]
    out = torch.zeros(xs.shape, dtype=torch.float32)
    for b in range(bsz):
        line = b if conv_state_indices is None else int(conv_state_indices[b])
        if conv_state_indices is not None and line == pad_slot_id:
            continue
        cat = torch.cat([conv_state[line].to(torch.float32), xs[b].to(torch.float32)], dim=-1)
        y = _taps(cat[:, : state_len][:, state_len - (width - 1):] if width > 1
                  else cat[:, :0], xs[b], weight, bias)
        if activation:
            y = F.silu(y)
        out[b] = y
        conv_state[line].copy_(cat[:, -state_len:].to(conv_state.dtype))
    out = _out.out(out, x.dtype)
    return out.squeeze(-1) if squeeze else out


def causal_conv1d_varlen(x, conv_state, weight, bias=None, activation=True,
                         query_start_loc=None, conv_state_indices=None,
                         pad_slot_id=-1):
    """Varlen prefill: ``causal_conv1d_update_ref_v2``
    (triton_npu/triton_src/test_causal_conv1d_update_v2.py:260-339) called
    once per sequence with ``max_query_len`` equal to that sequence's length
    (the reference function itself breaks when the lengths differ).

    x: [T, dim] token-major; query_start_loc: [B+1]; conv_state:
    [lines, dim, width-1] holding each sequence's history (zeros for a fresh
    prefill) and updated IN PLACE to the last width-1 inputs of
    cat(history, x_seq).  Returns [T, dim] in x's dtype (rows of skipped
    sequences are zeros here).
    """
    width = weight.shape[1]
    hist_len = width - 1
    out = torch.zeros(x.shape, dtype=torch.float32)
    nseq = query_start_loc.numel() - 1
    for b in range(nseq):
        s, e = int(query_start_loc[b]), int(query_start_loc[b + 1])
        line = b if conv_state_indices is None else int(conv_state_indices[b])
        if conv_state_indices is not None and line == pad_slot_id:
            continue
        if e <= s:
            continue
        xs = x[s:e].t()
        hist = conv_state[line, :, :hist_len]
        y = _taps(hist, xs, weight, bias)
        if activation:
            y = F.silu(y)
        out[s:e] = y.t()
        cat = torch.cat([hist.to(torch.float32), xs.to(torch.float32)], dim=-1)
        conv_state[line, :, :hist_len].copy_(cat[:, cat.shape[1] - hist_len:].to(conv_state.dtype))
    return _out.out(out, x.dtype)


def causal_conv1d_update_v2_slots(x, conv_state, weight, bias=None, activation=True,
                                  query_start_loc=None, conv_state_indices=None,
                                  num_accepted_tokens=None, initial_state_idx=None,
                                  block_idx_last_scheduled_token=None, pad_slot_id=-1):
    """Slot-table conv (speculative decoding, prefix-cache block tables):
    ``causal_conv1d_update_ref_v2``
    (triton_npu/triton_src/test_causal_conv1d_update_v2.py:260-345) with each
    sequence's window length taken from its own length (the reference takes
    it from ``max_query_len``, which breaks for shorter sequences).

    Sequence b reads line ``idx[b, initial_state_idx[b]]`` (``idx[b]`` for a
    [B] table, b without one) and writes line ``idx[b, last[b]]``; a read
    line equal to ``pad_slot_id`` skips it.  History = state columns
    ``[off, off + width - 1)`` with ``off = num_accepted_tokens[b] - 1`` (0
    without).  ``L = width - 1 + (len - 1 if speculative else 0)`` state
    columns are rewritten: the last L columns of cat(state[off + shift :],
    x_seq), shift = 1 (speculative) or len.  x: [T, dim] token-major;
    conv_state [lines, dim, state_len] updated IN PLACE.
    """
    width = weight.shape[1]
    out = torch.zeros(x.shape, dtype=torch.float32)
    spec = num_accepted_tokens is not None
    for b in range(query_start_loc.numel() - 1):
        if conv_state_indices is None:
            in_line = out_line = b
        elif conv_state_indices.dim() == 1:
            in_line = out_line = int(conv_state_indices[b])
        else:
            i0 = int(initial_state_idx[b]) if initial_state_idx is not None else 0
            i1 = int(block_idx_last_scheduled_token[b]) if initial_state_idx is not None else 0
            in_line, out_line = int(conv_state_indices[b, i0]), int(conv_state_indices[b, i1])
        if in_line == pad_slot_id:
            continue
        s, e = int(query_start_loc[b]), int(query_start_loc[b + 1])
        n = e - s
        if n <= 0:
            continue
        off = int(num_accepted_tokens[b]) - 1 if spec else 0
        L = width - 1 + (n - 1 if spec else 0)
        xs = x[s:e].t()
        src = conv_state[in_line].to(torch.float32)
        y = _taps(src[:, off:off + width - 1], xs, weight, bias)
        if activation:
            y = F.silu(y)
        out[s:e] = y.t()
        if n >= L:
            new = xs.to(torch.float32)[:, n - L:]
        else:
            shift = 1 if spec else n
            new = torch.cat([src[:, off + shift:off + shift + L - n], xs.to(torch.float32)], -1)
        conv_state[out_line, :, :L].copy_(new.to(conv_state.dtype))
    return _out.out(out, x.dtype)
