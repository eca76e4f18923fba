"""C-ABI checks that need no GPU: the library loads, exports every symbol
declared in include/*.h, and rejects bad arguments on the host (before any
CUDA call) with the documented status codes."""

import ctypes as C
import glob
import os
import re

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in glob.glob(os.path.join(ROOT, "include", "*.h")):
        text = open(h).read()
        names |= set(re.findall(r"XOPS_API\s+[\w\s\*]+?\b(xops_\w+)\s*\(", text))
    return names


@pytest.fixture(scope="module")
def lib():
    from torch_npu_ops_b200 import _lib
    return _lib.load()


def test_header_declares_entry_points():
    names = _declared()
    assert "xops_chunk_gated_delta_rule" in names
    assert len(names) >= 18


def test_library_exports_every_declared_symbol(lib):
    for name in sorted(_declared()):
        assert hasattr(lib, name), f"{name} declared in include/ but not exported"


def test_binding_covers_header():
    from torch_npu_ops_b200 import _lib
    assert _declared() == set(_lib.SIGNATURES), "ctypes signature table out of sync with header"


def test_version(lib):
    assert b"sm_100a" in lib.xops_version()


def _call(lib, name, *args):
    return getattr(lib, name)(*args), lib.xops_last_error().decode()


def test_host_validation_layer_norm(lib):
    rc, msg = _call(lib, "xops_layer_norm_fwd", None, None, None, None, None, None, None,
                    4, 100, 30, 100, 0, 100, 1e-6, 1, 1, 1, 1, None)
    assert rc == 1 and "divisible" in msg


def test_host_validation_chunk_unsupported_dims(lib):
    rc, msg = _call(lib, "xops_chunk_gated_delta_rule", None, None, None, None, None, None, None,
                    None, None, 1, 64, 1, 1, 1, 64, 64, 0, 0, 0, 0.1, 0, None, 0, None)
    assert rc == 2 and "128" in msg


def test_host_validation_gqa(lib):
    rc, msg = _call(lib, "xops_chunk_gated_delta_rule", None, None, None, None, None, None, None,
                    None, None, 1, 64, 1, 3, 4, 128, 128, 0, 0, 0, 0.1, 0, None, 0, None)
    assert rc == 1 and "divisible" in msg


def _out_norm(lib, z, zld, w_dtype, y, T=64, H=4):
    # q k v g beta h0 o ht cu | B T N Hg H K V | strides | scale l2 | z zld w wdt eps y | ws
    return _call(lib, "xops_chunk_gated_delta_rule_out_norm", None, None, None, None, None, None,
                 None, None, None, 1, T, 1, 2, H, 128, 128, 0, 0, 0, 0.1, 0, z, zld, 16, w_dtype,
                 1e-6, y, None, 0, None)


def test_host_validation_out_norm(lib):
    # the norm weight is fp32 or bf16 only
    rc, msg = _out_norm(lib, 16, 0, 2, 16)
    assert rc == 1 and "fp32 or bf16" in msg
    # z token stride below the heads, or not a multiple of 8
    rc, msg = _out_norm(lib, 16, 4 * 128 - 8, 1, 16)
    assert rc == 1 and "stride" in msg
    rc, msg = _out_norm(lib, 16, 4 * 128 + 4, 1, 16)
    assert rc == 1 and "stride" in msg
    # z and y are required (o is optional)
    rc, msg = _out_norm(lib, None, 0, 1, 16)
    assert rc == 1 and "must be given" in msg
    # nothing to do: OK without touching the device
    assert _out_norm(lib, None, 0, 1, None, T=0)[0] == 0


def test_host_validation_gated_out_norm(lib):
    # z heads grouped per key head: the group size must divide H
    rc, msg = _call(lib, "xops_chunk_gated_delta_rule_gated_out_norm", None, None, None, None,
                    None, None, None, 1, 1, 0, 1, 1.0, 20.0, None, None, None, None, 1, 64, 1, 2,
                    4, 128, 128, 0, 0, 0, 0.1, 0, 16, 0, 3, 0, 16, 1, 1e-6, 16, None, 0, None)
    assert rc == 1 and "stride" in msg


def test_host_validation_conv_width(lib):
    rc, msg = _call(lib, "xops_causal_conv1d_varlen", None, None, None, None, None, None, None,
                    2, 10, 64, 9, 2, 1, -1, 1, None)
    assert rc == 1 and "width" in msg


def test_empty_inputs_are_noops(lib):
    # zero sequences / rows: nothing to launch, OK without touching the device
    assert lib.xops_chunk_gated_delta_rule(None, None, None, None, None, None, None, None, None,
                                           1, 0, 1, 1, 1, 128, 128, 0, 0, 0, 0.1, 0, None, 0, None) == 0
    assert lib.xops_layer_norm_fwd(None, None, None, None, None, None, None, 0, 128, 128, 128, 0,
                                   128, 1e-6, 1, 1, 1, 1, None) == 0


def test_chunk_workspace_rules(lib):
    assert lib.xops_chunk_gated_delta_rule_workspace_size(1, 16384, 8, 16, 32, 128, 0, 1) == \
        (16384 // 64 + 8) * 32 * 33280
    with_l2 = lib.xops_chunk_gated_delta_rule_workspace_size(2, 100, 2, 2, 4, 128, 1, 0)
    assert with_l2 == 2 * 2 * 4 * 33280 + 2 * 2 * 100 * 2 * 128 * 2
    # one long sequence over few heads: the chain is cut into 205-chunk
    # segments and three fp32 states per (segment slot, head) are added
    long_seq = lib.xops_chunk_gated_delta_rule_workspace_size(1, 65536, 1, 16, 32, 128, 0, 1)
    slots = (1024 + 1 + 204) // 205 + 1
    assert long_seq == (1024 + 1) * 32 * 33280 + slots * 32 * 3 * 128 * 128 * 4
    rc, msg = _call(lib, "xops_chunk_gated_delta_rule", 16, 16, 16, 16, 16, None, 16, None, None,
                    1, 64, 1, 1, 1, 128, 128, 0, 0, 0, 0.1, 0, None, 0, None)
    assert rc == 4 and "workspace" in msg


def test_total_chunks_host(lib):
    cu = (C.c_int32 * 4)(0, 65, 66, 196)
    assert lib.xops_total_chunks(cu, 1, 196, 3, 64) == 2 + 1 + 3
    assert lib.xops_total_chunks(None, 2, 100, 2, 64) == 4


def test_ops_fail_loudly_off_gpu():
    """The host API has no CPU path: CPU tensors raise instead of computing."""
    import torch_npu_ops_b200 as ops
    x = torch.randn(4, 128, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.npu_l2norm_last_dim(x)
    q = torch.randn(1, 8, 2, 128, dtype=torch.bfloat16)
    v = torch.randn(1, 8, 4, 128, dtype=torch.bfloat16)
    g = torch.zeros(1, 8, 4)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.npu_chunk_gated_delta_rule(q, q, v, g, g)
    z = torch.randn(1, 8, 4, 128, dtype=torch.bfloat16)
    w = torch.ones(128)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.chunk_gated_delta_rule_out_norm(q, q, v, g, g, z, w)
    A_log, dt = torch.zeros(4), torch.zeros(4)
    with pytest.raises(RuntimeError, match="CUDA"):
        ops.chunk_gated_delta_rule_gated_out_norm(q, q, v, A_log, g[0], g[0], dt, z, w)


def test_ops_reject_like_reference():
    import torch_npu_ops_b200 as ops
    q = torch.randn(1, 8, 2, 128)
    v = torch.randn(1, 8, 4, 128)
    g = torch.zeros(1, 8, 4)
    with pytest.raises(RuntimeError, match="bfloat16"):
        ops.npu_chunk_gated_delta_rule(q, q, v, g, g)
    with pytest.raises(RuntimeError, match="head_first"):
        ops.npu_chunk_gated_delta_rule(q, q, v, g, g, head_first=True)
    with pytest.raises(RuntimeError, match="query_start_loc"):
        ops.npu_causal_conv1d_update(torch.randn(2, 8), torch.randn(2, 8, 3), torch.randn(8, 4),
                                     query_start_loc=torch.tensor([0, 1, 2]))
    with pytest.raises(RuntimeError, match="power of two"):
        ops.npu_split_rmsnorm_rope(torch.randn(2, 30 * 5), torch.randn(2, 30), torch.randn(2, 30),
                                   torch.randn(30), torch.randn(30), 90, 30, 30, 1e-6)
