"""B200 (sm_100a) build of the xLLM GDN linear-attention and normalisation
hot path: hand-written CUDA kernels behind a C ABI (``include/xops_b200.h``,
``libxops_b200.so``) and a host-side mirror of the reference's operator API
(``xllm::kernel::npu`` / ``npu_ops`` / ``npu_python_extension_lib``)."""

from .ops import (  # noqa: F401
    npu_l2norm_last_dim,
    layer_norm_fwd,
    layer_norm_fwd_with_stats,
    npu_gemma_rms_norm,
    npu_split_rmsnorm_rope,
    rope_inplace,
    npu_causal_conv1d_update,
    npu_causal_conv1d_update_v2,
    causal_conv1d_varlen_qk_l2norm,
    causal_conv1d_varlen_qkvz,
    npu_fused_recurrent_gated_delta_rule,
    npu_fused_gdn_gating,
    npu_fused_qkvzba_split_reshape_cat,
    npu_fused_sigmoid_gating_delta_rule_update,
    npu_chunk_gated_delta_rule,
    chunk_gated_delta_rule_gated,
    chunk_gated_delta_rule_out_norm,
    chunk_gated_delta_rule_gated_out_norm,
    npu_chunk_local_cumsum,
    npu_chunk_scaled_dot_kkt_fwd,
    npu_solve_tril,
    npu_recompute_w_u_fwd,
    npu_chunk_gated_delta_rule_fwd_h,
    npu_chunk_fwd_o,
)
from . import npu_python_extension_lib  # noqa: F401
