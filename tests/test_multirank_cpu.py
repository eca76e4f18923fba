"""The N > 1 path on CPU: head sharding of the long-context workload (cfg 5)
and its independence across ranks, checked with world-size-2 gloo ranks
that run the oracle pipeline on their shards (the GPU bench runs the same
shards through the CUDA kernels)."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from torch_npu_ops_b200 import workloads


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_head_shards_partition_heads_and_channels(world):
    hv, hk, d = workloads.V_HEADS, workloads.QK_HEADS, workloads.HEAD_DIM
    vs, ks, chans = [], [], []
    for r in range(world):
        (v0, v1), (k0, k1) = workloads.head_shard(r, world)
        vs += list(range(v0, v1))
        ks += list(range(k0, k1))
        # every value head's key head (GQA: h // (hv / hk)) lives on the same rank
        assert all(k0 <= h // (hv // hk) < k1 for h in range(v0, v1))
        chans.append(workloads.conv_channels(r, world))
    assert sorted(vs) == list(range(hv)) and sorted(ks) == list(range(hk))
    allc = torch.cat(chans)
    assert allc.numel() == workloads.CONV_DIM
    assert torch.equal(torch.sort(allc).values, torch.arange(workloads.CONV_DIM))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shard_inputs_are_slices_of_the_full_draw(world):
    """Every rank's cfg-5 inputs are exactly its slice of the world-1 draw, so
    one oracle run over all heads checks every shard (the GPU parity test of
    the bench configuration relies on this)."""
    T = 128
    full = workloads.long_config5_shard(0, 1, T=T)
    for r in range(world):
        w = workloads.long_config5_shard(r, world, T=T)
        v0, v1 = w["heads"]
        ch = workloads.conv_channels(r, world)
        assert torch.equal(w["x"], full["x"][:, ch])
        assert torch.equal(w["weight"], full["weight"][ch])
        assert torch.equal(w["bias"], full["bias"][ch])
        assert torch.equal(w["g"], full["g"][:, :, v0:v1])
        assert torch.equal(w["beta"], full["beta"][:, :, v0:v1])
        assert torch.equal(w["z"], full["z"][:, v0:v1])
        assert torch.equal(w["initial_state"], full["initial_state"][:, v0:v1])
        assert torch.equal(w["norm_w"], full["norm_w"])


def _pipeline(w, T):
    """conv1d -> chunk GDN (q/k L2 in the op) -> gated RMSNorm on one shard."""
    (v0, v1), (k0, k1) = w["heads"], w["k_heads"]
    hv, hk, d = v1 - v0, k1 - k0, workloads.HEAD_DIM
    st = torch.zeros(1, w["x"].shape[1], 3, dtype=torch.bfloat16)
    y = oracle.causal_conv1d_varlen(w["x"], st, w["weight"], w["bias"], True,
                                    torch.tensor([0, T], dtype=torch.int32))
    q = y[:, : hk * d].reshape(1, T, hk, d)
    k = y[:, hk * d: 2 * hk * d].reshape(1, T, hk, d)
    v = y[:, 2 * hk * d:].reshape(1, T, hv, d)
    o, _ = oracle.chunk_gated_delta_rule(q, k, v, w["g"], w["beta"], None, w["initial_state"], True,
                                         None, True)
    out, _, _ = oracle.layer_norm_fwd(o.reshape(-1, d), w["norm_w"], None, 1e-6,
                                      w["z"].reshape(-1, d), d, True, True)
    return out.reshape(T, hv, d)


def _rank_main(rank, world, port, T, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = workloads.long_config5_shard(rank, world, T=T)
        out = _pipeline(w, T)
        parts = [torch.empty_like(out) for _ in range(world)]
        dist.all_gather(parts, out)  # verification only, outside any timed path
        if rank == 0:
            torch.save(torch.cat(parts, dim=1), result_path)
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_two_rank_shards_reproduce_the_single_rank_result(tmp_path):
    T = 192
    path = str(tmp_path / "sharded.pt")
    mp.spawn(_rank_main, args=(2, _free_port(), T, path), nprocs=2, join=True)
    sharded = torch.load(path)
    full = _pipeline(workloads.long_config5_shard(0, 1, T=T), T)
    assert sharded.shape == full.shape == (T, workloads.V_HEADS, workloads.HEAD_DIM)
    torch.testing.assert_close(sharded.float(), full.float(), rtol=0, atol=1e-2)
    # heads are independent, so most elements agree exactly
    assert (sharded == full).float().mean() > 0.99
