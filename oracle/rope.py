"""q/k RMSNorm + NeoX RoPE oracle (test infrastructure only)."""

import torch


def _rms(x, w, eps, b=None):
    # rms_norm, triton_npu/triton_src/test_split_rmsnorm_rope.py:342-355
    xf = x.to(torch.float32)
    r = 1.0 / torch.sqrt((xf * xf).mean(dim=-1, keepdim=True) + eps)
    y = xf * r * w.to(torch.float32)
    if b is not None:
        y = y + b.to(torch.float32)
    return y


def _neox(x, sin, cos):
    """NeoX rotate-half on the first ``rd = sin.shape[-1]`` dims of each head.

    ``custom_rope`` (test_split_rmsnorm_rope.py:277-299) rotates the whole head
    (``rd == head_dim``): ``x*cos + cat(-x2, x1)*sin`` with x1/x2 the two
    halves.  With ``rd < head_dim`` the same rotation is applied to
    ``x[..., :rd]`` and dims ``[rd, head_dim)`` pass through unchanged.
    x: [T, heads, hd]; sin/cos: [T, rd].
    """
    rd = sin.shape[-1]
    s = sin.to(torch.float32)[:, None, :]
    c = cos.to(torch.float32)[:, None, :]
    xr = x[..., :rd]
    x1, x2 = xr[..., : rd // 2], xr[..., rd // 2:]
    rot = torch.cat([-x2, x1], dim=-1)
    out = x.clone()
    out[..., :rd] = xr * c + rot * s
    return out


def split_rmsnorm_rope(inp, sin, cos, q_weight, k_weight, q_hidden_size,
                       kv_hidden_size, head_dim, eps, q_bias=None, k_bias=None,
                       bias=False):
    """Split packed qkv, per-head RMSNorm on q and k, NeoX RoPE, copy v.

    Follows ``split_rmsnorm_rope_ref``
    (triton_npu/triton_src/test_split_rmsnorm_rope.py:302-339).  With
    ``sin.shape[-1] == head_dim`` this is the reference exactly; with a
    narrower sin/cos (partial rotary, e.g. 64 of 256) only the first
    ``rotary_dim`` dims rotate -- parity unpinned for that case (the
    reference API requires ``sin.size(1) == head_dim``,
    torch_api/npu_triton_split_rmsnorm_rope.cpp:85-87).
    Returns fp32 q [T, q_hidden], k [T, kv_hidden] and v in the input dtype.
    """
    t = inp.shape[0]
    q, k, v = inp.split([q_hidden_size, kv_hidden_size, kv_hidden_size], dim=-1)
    qb = q_bias if (bias and q_bias is not None and k_bias is not None) else None
    kb = k_bias if (bias and q_bias is not None and k_bias is not None) else None
    qn = _rms(q.reshape(t, -1, head_dim), q_weight, eps, qb)
    kn = _rms(k.reshape(t, -1, head_dim), k_weight, eps, kb)
    qo = _neox(qn, sin, cos).reshape(t, -1)
    ko = _neox(kn, sin, cos).reshape(t, -1)
    return qo, ko, v.clone()



def rope_inplace(x, sin, cos, rope_dim=64):
    """Interleaved (GPT-J style) RoPE on the last ``rope_dim`` dims, in place.

    Restates ``rope_ref`` (triton_npu/triton_src/test_rope_inplace.py:73-98):
    for each pair (2i, 2i+1) of the rotated tail,
    ``out[2i] = x[2i] cos[2i] - x[2i+1] sin[2i]`` and
    ``out[2i+1] = x[2i+1] cos[2i+1] + x[2i] sin[2i+1]``, computed in fp32 and
    rounded to x's dtype.  x is [bsz, hidden] or [bsz, heads, hidden]; sin
    and cos are [bsz, >= rope_dim] (one row per batch entry, shared by its
    heads).  Modifies x and returns it.
    """
    x3 = x if x.dim() == 3 else x.unsqueeze(1)
    tail = x3[..., x3.shape[-1] - rope_dim:].to(torch.float32)
    s = sin[:, :rope_dim].to(torch.float32).unsqueeze(1)
    c = cos[:, :rope_dim].to(torch.float32).unsqueeze(1)
    rot = torch.empty_like(tail)
    rot[..., 0::2] = -tail[..., 1::2]
    rot[..., 1::2] = tail[..., 0::2]
    x3[..., x3.shape[-1] - rope_dim:] = (tail * c + rot * s).to(x.dtype)
    return x
