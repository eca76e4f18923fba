"""The reference runtime's launch path on CPU: OperationBase::execute packs
the reference's argument buffer and either launches through a decoder or
returns an error without launching (so these cases need no GPU)."""

import pytest

C = pytest.importorskip("torch_npu_ops_b200._C")


def test_unknown_kernel_name_is_refused():
    rc, err, _ = C._runtime_execute("a_kernel_the_reference_does_not_have", 1, 1, 1, [], 0)
    assert rc == -1 and "not in the registry" in err


def test_kernel_without_decoder_returns_an_error_not_success():
    # rope_inplace_kernel keeps its rope and hidden sizes as compile-time
    # constants of the reference binary, so its buffer cannot be decoded
    assert not C._runtime_has_decoder("rope_inplace_kernel")
    rc, err, size = C._runtime_execute("rope_inplace_kernel", 4, 1, 1,
                                       [("ptr", 16), ("ptr", 16), ("ptr", 16), ("i32", 1),
                                        ("i32", 128), ("i32", 64)], 0)
    assert rc == -2 and "no decoder" in err
    # [ffts, lock, workspace] + 3 pointers + 3 int32 + grid (3 int32)
    assert size == 6 * 8 + 6 * 4


def test_malformed_buffer_is_rejected_before_launch():
    assert C._runtime_has_decoder("layer_norm_fwd_kernel_fast_rms_bf16_z_nobias")
    rc, err, _ = C._runtime_execute("layer_norm_fwd_kernel_fast_rms_bf16_z_nobias", 1, 1, 1,
                                    [("ptr", 16), ("ptr", 16)], 0)
    assert rc == -3 and "do not match" in err


@pytest.mark.parametrize("name", [
    "layer_norm_fwd_kernel", "layer_norm_fwd_kernel_fast", "layer_norm_fwd_kernel_fast_rms_bf16_z_bias",
    "l2norm_fwd_kernel2_loop", "fused_gdn_gating_decode_kernel",
    "_causal_conv1d_update_qwen_decode_kernel", "fused_recurrent_gated_delta_rule_fwd_kernel",
    "split_rmsnorm_rope_kernel_bias0_eps0000001_hd256_qh4096_kvh512"])
def test_decoded_kernel_names(name):
    assert C._runtime_has_decoder(name)
