"""White-box GPU check of the chunked rule's preparation stage.

The fused chunk operator leaves, per (64-token chunk, value head), the
images its preparation kernel computed in the caller's workspace:
T' = (I + A)^-1 diag(beta), -w = -(I + A)^-1 diag(beta e^gc) k and
Aqk = tril(q k^T * e^{gc_i - gc_j}), stored as 128-byte-swizzled bf16 tiles
(chunk c of row r at c ^ (r & 7)).  These tests decode them and compare
with the same quantities computed in float64 from their definition
(npu_triton_chunk_gated_delta_rule.cpp:556-642: chunk_scaled_dot_kkt ->
solve_tril -> recompute_w_u; chunk_fwd_o's q k^T term).

The inputs are chosen so that the triangular inverse matters: weak gates
(slow decay inside a chunk) and keys sharing a common direction give
|A_ij| up to ~0.5 across the whole chunk, where the synthetic cfg3 gates
make A nearly bidiagonal."""

import ctypes as C

import pytest
import torch
import torch.nn.functional as F

from torch_npu_ops_b200 import _lib

pytestmark = pytest.mark.gpu
WS_CHUNK, WS_W, WS_TP, WS_AQK, WS_GB = 33280, 0, 16384, 24576, 32768


def _swz(rows, cols, base, half_stride):
    """bf16 element index of (r, c) in a swizzled [rows x cols] image."""
    r = torch.arange(rows)[:, None]
    c = torch.arange(cols)[None, :]
    byte = base + (c >> 6) * half_stride + r * 128 + ((((c & 63) >> 3) ^ (r & 7)) << 4) + (c & 7) * 2
    return byte // 2


def _inputs(T, hk, hv, corr, gscale, seed):
    g = torch.Generator().manual_seed(seed)
    base = torch.randn(1, 1, hk, 128, generator=g)
    k = F.normalize(torch.randn(1, T, hk, 128, generator=g) + corr * base, dim=-1)
    q = F.normalize(torch.randn(1, T, hk, 128, generator=g), dim=-1)
    v = torch.randn(1, T, hv, 128, generator=g)
    gate = -gscale * torch.rand(1, T, hv, generator=g)
    beta = torch.sigmoid(torch.randn(1, T, hv, generator=g))
    return (q.to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16), gate, beta)


def _reference(q, k, gate, beta, c, h, r, L):
    kc = k[0, c * 64:c * 64 + L, h // r].double()
    qc = q[0, c * 64:c * 64 + L, h // r].double()
    gc = torch.cumsum(gate[0, c * 64:c * 64 + L, h].double(), 0)
    b = beta[0, c * 64:c * 64 + L, h].double()
    dec = torch.exp((gc[:, None] - gc[None, :]).clamp(max=0))
    A = torch.tril(b[:, None] * dec * (kc @ kc.T), -1)
    Tm = torch.linalg.inv(torch.eye(L, dtype=torch.float64) + A)
    tp = Tm * b[None, :]
    w = (Tm * (b * torch.exp(gc))[None, :]) @ kc
    aqk = torch.tril((qc @ kc.T) * dec)
    return tp, w, aqk


def _rel(a, b):
    return ((a - b).norm() / b.norm().clamp(min=1e-30)).item()


@pytest.mark.parametrize("T,hk,hv,corr,gscale", [
    (256, 2, 4, 1.5, 0.02),   # two value heads per key head (the paired preparation)
    (200, 2, 4, 3.0, 0.01),   # strongly correlated keys, a partial last chunk
    (192, 2, 6, 1.5, 0.02),   # three value heads per key head (the per-head preparation)
])
def test_preparation_images_match_definition(T, hk, hv, corr, gscale):
    lib = _lib.load()
    q, k, v, gate, beta = _inputs(T, hk, hv, corr, gscale, seed=T + hv)
    cu = torch.tensor([0, T], dtype=torch.int32)
    d = [x.cuda() for x in (q, k, v, gate, beta)]
    o = torch.empty_like(d[2])
    ht = torch.empty(1, hv, 128, 128, device="cuda")
    need = lib.xops_chunk_gated_delta_rule_workspace_size(1, T, 1, hk, hv, 128, 0, 1)
    ws = torch.zeros(need, dtype=torch.uint8, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    cud = cu.cuda()
    rc = lib.xops_chunk_gated_delta_rule(
        d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), d[3].data_ptr(), d[4].data_ptr(), None,
        o.data_ptr(), ht.data_ptr(), cud.data_ptr(), 1, T, 1, hk, hv, 128, 128, 0, 0, 0,
        128 ** -0.5, 0, ws.data_ptr(), need, stream)
    assert rc == 0, lib.xops_last_error()
    torch.cuda.synchronize()
    img = ws.cpu().view(torch.bfloat16)
    r = hv // hk
    i_tp, i_aqk = _swz(64, 64, WS_TP, 0), _swz(64, 64, WS_AQK, 0)
    i_w = _swz(64, 128, WS_W, 8192)
    worst = {"T'": 0.0, "-w": 0.0, "Aqk": 0.0}
    for c in range((T + 63) // 64):
        L = min(64, T - 64 * c)
        for h in range(hv):
            off = (c * hv + h) * WS_CHUNK // 2
            tp = img[off + i_tp].double()[:L, :L]
            w = -img[off + i_w].double()[:L]
            aqk = img[off + i_aqk].double()[:L, :L]
            rtp, rw, raqk = _reference(q, k, gate, beta, c, h, r, L)
            # the diagonal of T' is bf16(beta); the chain adds beta - bf16(beta)
            dg = torch.diagonal(tp)
            assert torch.equal(dg, torch.diagonal(rtp).to(torch.bfloat16).double()), (c, h)
            off_d = ~torch.eye(L, dtype=torch.bool)
            e = {"T'": _rel(tp[off_d], rtp[off_d]), "-w": _rel(w, rw), "Aqk": _rel(aqk, raqk)}
            for n, x in e.items():
                worst[n] = max(worst[n], x)
    # bf16 rounding of each stored value alone gives ~1e-3 relative; -w is a
    # bf16 product of the rounded T'' with k, whose cancellations (keys
    # sharing a direction) amplify that rounding
    assert worst["T'"] < 5e-3 and worst["Aqk"] < 5e-3 and worst["-w"] < 1.5e-2, worst
