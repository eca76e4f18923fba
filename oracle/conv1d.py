"""Depthwise causal conv1d oracles (test infrastructure only)."""

import torch
import torch.nn.functional as F


def _taps(hist, xs, weight, bias):
    """Depthwise causal conv of ``xs`` [dim, L] preceded by ``hist``
    [dim, width-1]; returns fp32 [dim, L]."""
    width = weight.shape[1]
    cat = torch.cat([hist.to(torch.float32), xs.to(torch.float32)], dim=-1)
    out = F.conv1d(cat.unsqueeze(0), weight.to(torch.float32).unsqueeze(1),
                   None if bias is None else bias.to(torch.float32),
                   groups=weight.shape[0])[0]
    return out[:, -xs.shape[-1]:] if width > 1 else out


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
    out = out.to(x.dtype)
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
    return out.to(x.dtype)
