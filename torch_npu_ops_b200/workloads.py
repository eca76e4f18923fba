"""Seeded synthetic inputs for the benchmark configurations of this path.

No dataset is involved anywhere: every config is synthetic, with the shapes
and value distributions of the benchmark definition.  Inputs are generated
on the CPU in fp32 from ``torch.Generator().manual_seed(<config #>)`` and
then cast, so the same tensors feed the CUDA path, the CPU baseline and the
parity tests.

Configs:
  1  q/k RMSNorm + partial NeoX RoPE, fp32, T=128, 16 q / 2 kv heads,
     head_dim 256, rotary 64, theta 1e7, positions 0..127, eps 1e-6.
  2  causal_conv1d, 8192 channels, width 4, bias, SiLU; prefill = 8 seqs of
     seeded lengths in [256, 4096] summing to 16384; decode = batch 256.
  3  chunked gated delta rule, 8 seqs summing to 16384, Hk 16 -> Hv 32,
     dk = dv = 128.
  4  decode batch 256: recurrent GDN, gated RMSNorm on [256*32, 128],
     layer_norm / gemma on [256, 2048].
  5  single 65536-token sequence: conv -> chunk GDN (initial state
     ~N(0, 0.02), final state returned) -> gated RMSNorm, heads sharded over
     ranks.
"""

import math

import torch
import torch.nn.functional as F

QK_HEADS, V_HEADS, HEAD_DIM = 16, 32, 128
CONV_DIM = 2 * QK_HEADS * HEAD_DIM + V_HEADS * HEAD_DIM  # 8192


def seeded_lengths(total, n, lo, hi, gen):
    """n lengths in [lo, hi] summing to total, drawn from ``gen``."""
    assert n * lo <= total <= n * hi
    lens = [lo] * n
    rem = total - n * lo
    while rem > 0:
        w = torch.rand(n, generator=gen)
        room = torch.tensor([hi - l for l in lens], dtype=torch.float64)
        w = w.double() * (room > 0)
        if w.sum() == 0:
            break
        add = torch.floor(w / w.sum() * rem).long()
        add = torch.minimum(add, room.long())
        if add.sum() == 0:  # place the last few tokens one by one
            i = int(torch.argmax(w))
            add[i] = 1
        for i in range(n):
            lens[i] += int(add[i])
        rem = total - sum(lens)
    return lens


def cu_from_lengths(lens):
    return torch.tensor([0] + torch.cumsum(torch.tensor(lens), 0).tolist(), dtype=torch.int32)


def neox_sin_cos(positions, rotary_dim, theta):
    inv = 1.0 / (theta ** (torch.arange(0, rotary_dim, 2, dtype=torch.float64) / rotary_dim))
    ang = positions.to(torch.float64)[:, None] * inv[None, :]
    ang = torch.cat([ang, ang], dim=-1)
    return torch.sin(ang).float(), torch.cos(ang).float()


def rope_config1(T=128, seed=1):
    g = torch.Generator().manual_seed(seed)
    qh, kvh, hd, rd = 16, 2, 256, 64
    inp = torch.randn(T, (qh + 2 * kvh) * hd, generator=g)
    qw = 1 + 0.1 * torch.randn(hd, generator=g)
    kw = 1 + 0.1 * torch.randn(hd, generator=g)
    sin, cos = neox_sin_cos(torch.arange(T), rd, 1e7)
    return {"tensors": (inp, sin, cos, qw, kw),
            "kwargs": dict(q_hidden_size=qh * hd, kv_hidden_size=kvh * hd, head_dim=hd, eps=1e-6)}


def conv_prefill_config2(total=16384, nseq=8, dim=CONV_DIM, seed=2):
    g = torch.Generator().manual_seed(seed)
    lens = seeded_lengths(total, nseq, 256, 4096, g)
    x = torch.randn(total, dim, generator=g).to(torch.bfloat16)
    w = (0.5 * torch.randn(dim, 4, generator=g)).to(torch.bfloat16)
    b = (0.5 * torch.randn(dim, generator=g)).to(torch.bfloat16)
    st = torch.zeros(nseq, dim, 3, dtype=torch.bfloat16)
    return {"x": x, "conv_state": st, "weight": w, "bias": b,
            "query_start_loc": cu_from_lengths(lens), "lengths": lens}


def conv_decode_config2(batch=256, dim=CONV_DIM, seed=2):
    g = torch.Generator().manual_seed(seed + 100)
    x = torch.randn(batch, dim, generator=g).to(torch.bfloat16)
    st = torch.randn(batch, dim, 3, generator=g).to(torch.bfloat16)
    w = (0.5 * torch.randn(dim, 4, generator=g)).to(torch.bfloat16)
    b = (0.5 * torch.randn(dim, generator=g)).to(torch.bfloat16)
    return {"x": x, "conv_state": st, "weight": w, "bias": b}


def gdn_gates(T, H, g):
    """g = -exp(A_log) * softplus(a + dt_bias), beta = sigmoid(N(0,1))."""
    a_log = torch.rand(H, generator=g) * 2.7
    a = torch.randn(T, H, generator=g)
    dt_bias = torch.rand(H, generator=g)
    gate = -torch.exp(a_log) * F.softplus(a + dt_bias)
    beta = torch.sigmoid(torch.randn(T, H, generator=g))
    return gate, beta


def chunk_config3(total=16384, nseq=8, hk=QK_HEADS, hv=V_HEADS, d=HEAD_DIM, seed=3,
                  lengths=None):
    g = torch.Generator().manual_seed(seed)
    lens = lengths if lengths is not None else seeded_lengths(total, nseq, 256, 4096, g)
    T = sum(lens)
    q = F.normalize(torch.randn(1, T, hk, d, generator=g), dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(1, T, hk, d, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(1, T, hv, d, generator=g).to(torch.bfloat16)
    gate, beta = gdn_gates(T, hv, g)
    h0 = 0.02 * torch.randn(len(lens), hv, d, d, generator=g)
    return {"q": q, "k": k, "v": v, "g": gate[None], "beta": beta[None], "initial_state": h0,
            "cu_seqlens": cu_from_lengths(lens), "lengths": lens}


def decode_config4(batch=256, hk=QK_HEADS, hv=V_HEADS, d=HEAD_DIM, hidden=2048, seed=4):
    g = torch.Generator().manual_seed(seed)
    q = F.normalize(torch.randn(1, batch, hk, d, generator=g), dim=-1).to(torch.bfloat16)
    k = F.normalize(torch.randn(1, batch, hk, d, generator=g), dim=-1).to(torch.bfloat16)
    v = torch.randn(1, batch, hv, d, generator=g).to(torch.bfloat16)
    gate, beta = gdn_gates(batch, hv, g)
    state = 0.02 * torch.randn(batch, hv, d, d, generator=g)
    o = torch.randn(batch * hv, d, generator=g).to(torch.bfloat16)
    z = torch.randn(batch * hv, d, generator=g).to(torch.bfloat16)
    nw = (1 + 0.1 * torch.randn(d, generator=g)).to(torch.bfloat16)
    hid = torch.randn(batch, hidden, generator=g).to(torch.bfloat16)
    lw = (1 + 0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    lb = (0.1 * torch.randn(hidden, generator=g)).to(torch.bfloat16)
    return {"q": q, "k": k, "v": v, "g": gate[None], "beta": beta[None], "state": state,
            "cu_seqlens": torch.arange(batch + 1, dtype=torch.int32),
            "ssm_state_indices": torch.arange(batch, dtype=torch.int32),
            "norm_x": o, "norm_z": z, "norm_w": nw, "hidden": hid, "ln_w": lw, "ln_b": lb}


def head_shard(rank, world, hv=V_HEADS, hk=QK_HEADS):
    """Value heads and key heads owned by ``rank`` of ``world`` (contiguous
    blocks; value head h reads key head h // (hv // hk))."""
    assert hv % world == 0 and hk % world == 0
    v0, v1 = hv * rank // world, hv * (rank + 1) // world
    k0, k1 = hk * rank // world, hk * (rank + 1) // world
    return (v0, v1), (k0, k1)


def conv_channels(rank, world, hv=V_HEADS, hk=QK_HEADS, d=HEAD_DIM):
    """Conv channel indices of the q | k | v blocks that feed ``rank``'s heads."""
    (v0, v1), (k0, k1) = head_shard(rank, world, hv, hk)
    qb = torch.arange(k0 * d, k1 * d)
    kb = hk * d + torch.arange(k0 * d, k1 * d)
    vb = 2 * hk * d + torch.arange(v0 * d, v1 * d)
    return torch.cat([qb, kb, vb])


def long_config5_shard(rank, world, T=65536, seed=5):
    """Config 5 inputs for one rank's head shard (the same full-size draw for
    every world size, sliced, so results do not depend on the sharding).

    The conv input is generated per channel block of this rank only, from a
    per-block seed, so a rank never materialises the whole 1 GB tensor."""
    d = HEAD_DIM
    (v0, v1), (k0, k1) = head_shard(rank, world)
    blocks = []  # conv input columns for q, k, v heads of this shard
    for kind, lo, hi in (("q", k0, k1), ("k", k0, k1), ("v", v0, v1)):
        for hh in range(lo, hi):
            gb = torch.Generator().manual_seed(seed * 1000 + {"q": 0, "k": 1, "v": 2}[kind] * 100 + hh)
            blocks.append(torch.randn(T, d, generator=gb).to(torch.bfloat16))
    x = torch.cat(blocks, dim=1)
    gw = torch.Generator().manual_seed(seed)
    w_full = (0.5 * torch.randn(CONV_DIM, 4, generator=gw)).to(torch.bfloat16)
    b_full = (0.5 * torch.randn(CONV_DIM, generator=gw)).to(torch.bfloat16)
    gate_full, beta_full = gdn_gates(T, V_HEADS, gw)
    nw = (1 + 0.1 * torch.randn(d, generator=gw)).to(torch.bfloat16)
    ch = conv_channels(rank, world)
    zs = []
    for hh in range(v0, v1):
        gz = torch.Generator().manual_seed(seed * 1000 + 300 + hh)
        zs.append(torch.randn(T, d, generator=gz).to(torch.bfloat16))
    # initial recurrent state of the one sequence, fp32 ~N(0, 0.02) as in
    # config 3, drawn per value head so a shard never draws the others
    h0 = torch.stack([0.02 * torch.randn(d, d, generator=torch.Generator().manual_seed(
        seed * 1000 + 400 + hh)) for hh in range(v0, v1)])[None]
    return {"x": x, "weight": w_full[ch].contiguous(), "bias": b_full[ch].contiguous(),
            "g": gate_full[:, v0:v1].contiguous()[None], "beta": beta_full[:, v0:v1].contiguous()[None],
            "z": torch.stack(zs, dim=1), "norm_w": nw, "initial_state": h0, "heads": (v0, v1),
            "k_heads": (k0, k1), "T": T}


def chunk_flops(lengths, hv):
    """Algorithmic tensor FLOPs of the chunked rule: per (value head, 64-token
    chunk) 5*(2*64*64*128) + 3*(2*64*128*128) = 11,534,336."""
    per = 5 * (2 * 64 * 64 * 128) + 3 * (2 * 64 * 128 * 128)
    return per * hv * sum(math.ceil(l / 64) for l in lengths)
