// One OperationBase subclass per reference kernel name, with the class names
// and kernel-name strings of triton_npu/operations.h:26-223 (callers include
// this header and name these classes).  Each class only binds its name; the
// launch is OperationBase::execute.
#pragma once

#include <string>
#include <utility>

#include "operation_base.h"

namespace xllm::kernel::npu {

#define XOPS_DECLARE_OP(Class, name) \
  class Class final : public OperationBase { \
   public: \
    Class() : OperationBase(name) {} \
  };

XOPS_DECLARE_OP(L2NormFwdOp, "l2norm_fwd_kernel2_loop")
XOPS_DECLARE_OP(RopeInplaceOp, "rope_inplace_kernel")
XOPS_DECLARE_OP(FusedGdnGatingOp, "fused_gdn_gating_decode_kernel")
XOPS_DECLARE_OP(LayerNormFwdOp, "layer_norm_fwd_kernel")
XOPS_DECLARE_OP(LayerNormFwdFastOp, "layer_norm_fwd_kernel_fast")
XOPS_DECLARE_OP(LayerNormFwdFastRMSBiasOp, "layer_norm_fwd_kernel_fast_rms_bias")
XOPS_DECLARE_OP(LayerNormFwdFastRMSNoBiasOp, "layer_norm_fwd_kernel_fast_rms_nobias")
XOPS_DECLARE_OP(LayerNormFwdFastBF16Op, "layer_norm_fwd_kernel_fast_bf16")
XOPS_DECLARE_OP(LayerNormFwdFastRMSBF16BiasOp, "layer_norm_fwd_kernel_fast_rms_bf16_bias")
XOPS_DECLARE_OP(LayerNormFwdFastRMSBF16NoBiasOp, "layer_norm_fwd_kernel_fast_rms_bf16_nobias")
XOPS_DECLARE_OP(LayerNormFwdFastZOp, "layer_norm_fwd_kernel_fast_z")
XOPS_DECLARE_OP(LayerNormFwdFastRMSZBiasOp, "layer_norm_fwd_kernel_fast_rms_z_bias")
XOPS_DECLARE_OP(LayerNormFwdFastRMSZNoBiasOp, "layer_norm_fwd_kernel_fast_rms_z_nobias")
XOPS_DECLARE_OP(LayerNormFwdFastBF16ZOp, "layer_norm_fwd_kernel_fast_bf16_z")
XOPS_DECLARE_OP(LayerNormFwdFastRMSBF16ZBiasOp, "layer_norm_fwd_kernel_fast_rms_bf16_z_bias")
XOPS_DECLARE_OP(LayerNormFwdFastRMSBF16ZNoBiasOp, "layer_norm_fwd_kernel_fast_rms_bf16_z_nobias")
XOPS_DECLARE_OP(LayerNormFwdFastRMSBF16ZNoBiasNoMaskOp,
                "layer_norm_fwd_kernel_fast_rms_bf16_z_nobias_nomask")
XOPS_DECLARE_OP(RecurrentGatedDeltaRuleFwdOp, "fused_recurrent_gated_delta_rule_fwd_kernel")
XOPS_DECLARE_OP(RecurrentGatedDeltaRuleSpecFwdOp, "fused_recurrent_gated_delta_rule_spec_fwd_kernel")
XOPS_DECLARE_OP(FusedSigmoidGatingDeltaRuleUpdateOp,
                "fused_sigmoid_gating_delta_rule_update_kernel")
XOPS_DECLARE_OP(ChunkGatedDeltaRuleFwdHOp, "chunk_gated_delta_rule_fwd_kernel_h_blockdim64")
XOPS_DECLARE_OP(ChunkLocalCumsumScalarOp, "chunk_local_cumsum_scalar_kernel")
XOPS_DECLARE_OP(ChunkScaledDotKktFwdOp, "chunk_scaled_dot_kkt_fwd_kernel")
XOPS_DECLARE_OP(SolveTril16x16Op, "solve_tril_16x16_kernel")
XOPS_DECLARE_OP(Merge16x16To64x64InverseOp, "merge_16x16_to_64x64_inverse_kernel")
XOPS_DECLARE_OP(RecomputeWUForwardOp, "recompute_w_u_fwd_kernel")
XOPS_DECLARE_OP(ChunkForwardOOp, "chunk_fwd_kernel_o")
XOPS_DECLARE_OP(CausalConv1dUpdateNoCacheNoMtpOp, "_causal_conv1d_update_kernel_no_cache_len_no_mtp")
XOPS_DECLARE_OP(CausalConv1dUpdateQwenDecodeOp, "_causal_conv1d_update_qwen_decode_kernel")
XOPS_DECLARE_OP(CausalConv1dUpdateTiledV2Op, "_causal_conv1d_update_kernel_npu_tiled_v2")
XOPS_DECLARE_OP(FusedQkvzbaSplitReshapeGqaR1Op, "fused_qkvzba_split_reshape_cat_gqa_r1_kernel")
XOPS_DECLARE_OP(FusedQkvzbaSplitReshapeGqaR2Op, "fused_qkvzba_split_reshape_cat_gqa_r2_kernel")
XOPS_DECLARE_OP(FusedQkvzbaSplitReshapeGqaR3Op, "fused_qkvzba_split_reshape_cat_gqa_r3_kernel")
XOPS_DECLARE_OP(FusedQkvzbaSplitReshapeGqaR4Op, "fused_qkvzba_split_reshape_cat_gqa_r4_kernel")
#undef XOPS_DECLARE_OP

// split_rmsnorm_rope kernels are specialised per (bias, eps, head_dim, q and
// kv hidden sizes), so the name is a constructor argument
class SplitRmsnormRopeOp final : public OperationBase {
 public:
  explicit SplitRmsnormRopeOp(std::string kernel_name) : OperationBase(std::move(kernel_name)) {}
};

}  // namespace xllm::kernel::npu
