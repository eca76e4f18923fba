"""xops_chunk_gated_delta_rule_noalloc: the chunked gated delta rule with its
scratch in the library's fixed device array instead of a caller workspace.
Called through the C ABI; it must give exactly the results of
xops_chunk_gated_delta_rule, call after call.  (Named to be collected last,
so it also runs after every other test has used the library.)"""

import ctypes as C

import pytest
import torch

from torch_npu_ops_b200 import _lib, workloads


def _args(d, o, ht, T, N, hk, hv):
    return [d["q"].data_ptr(), d["k"].data_ptr(), d["v"].data_ptr(), d["g"].data_ptr(),
            d["beta"].data_ptr(), d["initial_state"].data_ptr(), o.data_ptr(), ht.data_ptr(),
            d["cu_seqlens"].data_ptr(), 1, T, N, hk, hv, 128, 128, 0, 0, 0, 128 ** -0.5, 1]


@pytest.mark.gpu
@pytest.mark.parametrize("lens,hk,hv", [
    ([600, 401], 2, 4),   # short sequences: one chain pass per (sequence, head)
    ([4096], 2, 4),       # one long sequence on few heads: the segment-parallel
                          # chain, whose segment states sit at the scratch's tail
])
def test_noalloc_matches_workspace_entry_on_consecutive_calls(lens, hk, hv):
    lib = _lib.load()
    w = workloads.chunk_config3(hk=hk, hv=hv, lengths=lens, seed=77)
    g = torch.Generator().manual_seed(78)  # raw q/k: the in-kernel L2 norm is exercised
    w["q"] = torch.randn(w["q"].shape, generator=g).to(torch.bfloat16)
    w["k"] = torch.randn(w["k"].shape, generator=g).to(torch.bfloat16)
    d = {n: (t.cuda() if torch.is_tensor(t) else t) for n, t in w.items()}
    T, N = sum(lens), len(lens)
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)

    need = lib.xops_chunk_gated_delta_rule_workspace_size(1, T, N, hk, hv, 128, 1, 1)
    assert need <= 64 << 20
    if len(lens) == 1:  # the plan is segmented: segment states follow the per-chunk part
        assert need > (T // 64 + N) * hv * 33280 + 2 * T * hk * 128 * 2
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    o_ref = torch.empty_like(d["v"])
    ht_ref = torch.empty(N, hv, 128, 128, device="cuda")
    rc = lib.xops_chunk_gated_delta_rule(*_args(d, o_ref, ht_ref, T, N, hk, hv), ws.data_ptr(),
                                         need, stream)
    assert rc == 0, lib.xops_last_error()

    for _ in range(2):  # the second call reuses the scratch the first one left behind
        o = torch.full_like(d["v"], float("nan"))
        ht = torch.full((N, hv, 128, 128), float("nan"), device="cuda")
        rc = lib.xops_chunk_gated_delta_rule_noalloc(*_args(d, o, ht, T, N, hk, hv), stream)
        assert rc == 0, lib.xops_last_error()
        torch.cuda.synchronize()
        assert torch.equal(o, o_ref)
        assert torch.equal(ht, ht_ref)
    assert lib.xops_device_error_count() == 0


def test_noalloc_rejects_problems_beyond_the_fixed_scratch():
    """A workspace above 64 MiB is refused with XOPS_ERR_WORKSPACE before
    any device work (so this runs without a GPU too)."""
    lib = _lib.load()
    T, N, hk, hv = 65536, 1, 16, 32
    assert lib.xops_chunk_gated_delta_rule_workspace_size(1, T, N, hk, hv, 128, 1, 1) > 64 << 20
    dummy = C.c_void_p(16)
    rc = lib.xops_chunk_gated_delta_rule_noalloc(dummy, dummy, dummy, dummy, dummy, None, dummy,
                                                 None, dummy, 1, T, N, hk, hv, 128, 128, 0, 0, 0,
                                                 0.1, 1, None)
    assert rc == _lib.ERR_WORKSPACE
    assert b"fixed scratch" in lib.xops_last_error()
