// Process-wide op cache with the accessors of the reference's
// OperationFactory (triton_npu/torch_api/operation_factory.h:27-230).  Unlike
// the reference's unsynchronised map it is safe to call from several threads.
// One addition: by_kernel_name(), which returns the op bound to any kernel
// name of the registry (the named accessors cover the same ops).
#pragma once

#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>

#include "operations.h"

namespace xllm::kernel::npu {

class OperationFactory final {
 public:
  static OperationFactory& instance() {
    static OperationFactory f;
    return f;
  }

#define XOPS_ACCESSOR(fn, Class, name) \
  Class& fn() { return get<Class>(name); }
  XOPS_ACCESSOR(l2norm_fwd, L2NormFwdOp, "l2norm_fwd_kernel2_loop")
  XOPS_ACCESSOR(rope_inplace, RopeInplaceOp, "rope_inplace_kernel")
  XOPS_ACCESSOR(fused_gdn_gating, FusedGdnGatingOp, "fused_gdn_gating_decode_kernel")
  XOPS_ACCESSOR(layer_norm_fwd, LayerNormFwdOp, "layer_norm_fwd_kernel")
  XOPS_ACCESSOR(layer_norm_fwd_fast, LayerNormFwdFastOp, "layer_norm_fwd_kernel_fast")
  XOPS_ACCESSOR(layer_norm_fwd_fast_rms_bias, LayerNormFwdFastRMSBiasOp,
                "layer_norm_fwd_kernel_fast_rms_bias")
  XOPS_ACCESSOR(layer_norm_fwd_fast_rms_nobias, LayerNormFwdFastRMSNoBiasOp,
                "layer_norm_fwd_kernel_fast_rms_nobias")
  XOPS_ACCESSOR(layer_norm_fwd_fast_bf16, LayerNormFwdFastBF16Op, "layer_norm_fwd_kernel_fast_bf16")
  XOPS_ACCESSOR(layer_norm_fwd_fast_rms_bf16_bias, LayerNormFwdFastRMSBF16BiasOp,
                "layer_norm_fwd_kernel_fast_rms_bf16_bias")
  XOPS_ACCESSOR(layer_norm_fwd_fast_rms_bf16_nobias, LayerNormFwdFastRMSBF16NoBiasOp,
                "layer_norm_fwd_kernel_fast_rms_bf16_nobias")
  XOPS_ACCESSOR(layer_norm_fwd_fast_z, LayerNormFwdFastZOp, "layer_norm_fwd_kernel_fast_z")
  XOPS_ACCESSOR(layer_norm_fwd_fast_rms_z_bias, LayerNormFwdFastRMSZBiasOp,
                "layer_norm_fwd_kernel_fast_rms_z_bias")
  XOPS_ACCESSOR(layer_norm_fwd_fast_rms_z_nobias, LayerNormFwdFastRMSZNoBiasOp,
                "layer_norm_fwd_kernel_fast_rms_z_nobias")
  XOPS_ACCESSOR(layer_norm_fwd_fast_bf16_z, LayerNormFwdFastBF16ZOp,
                "layer_norm_fwd_kernel_fast_bf16_z")
  XOPS_ACCESSOR(layer_norm_fwd_fast_rms_bf16_z_bias, LayerNormFwdFastRMSBF16ZBiasOp,
                "layer_norm_fwd_kernel_fast_rms_bf16_z_bias")
  XOPS_ACCESSOR(layer_norm_fwd_fast_rms_bf16_z_nobias, LayerNormFwdFastRMSBF16ZNoBiasOp,
                "layer_norm_fwd_kernel_fast_rms_bf16_z_nobias")
  XOPS_ACCESSOR(layer_norm_fwd_fast_rms_bf16_z_nobias_nomask,
                LayerNormFwdFastRMSBF16ZNoBiasNoMaskOp,
                "layer_norm_fwd_kernel_fast_rms_bf16_z_nobias_nomask")
  XOPS_ACCESSOR(recurrent_gated_delta_rule_fwd, RecurrentGatedDeltaRuleFwdOp,
                "fused_recurrent_gated_delta_rule_fwd_kernel")
  XOPS_ACCESSOR(recurrent_gated_delta_rule_spec_fwd, RecurrentGatedDeltaRuleSpecFwdOp,
                "fused_recurrent_gated_delta_rule_spec_fwd_kernel")
  XOPS_ACCESSOR(fused_sigmoid_gating_delta_rule_update, FusedSigmoidGatingDeltaRuleUpdateOp,
                "fused_sigmoid_gating_delta_rule_update_kernel")
  XOPS_ACCESSOR(chunk_gated_delta_rule_fwd_h, ChunkGatedDeltaRuleFwdHOp,
                "chunk_gated_delta_rule_fwd_kernel_h_blockdim64")
  XOPS_ACCESSOR(chunk_local_cumsum_scalar, ChunkLocalCumsumScalarOp,
                "chunk_local_cumsum_scalar_kernel")
  XOPS_ACCESSOR(chunk_scaled_dot_kkt_fwd, ChunkScaledDotKktFwdOp, "chunk_scaled_dot_kkt_fwd_kernel")
  XOPS_ACCESSOR(solve_tril_16x16, SolveTril16x16Op, "solve_tril_16x16_kernel")
  XOPS_ACCESSOR(merge_16x16_to_64x64_inverse, Merge16x16To64x64InverseOp,
                "merge_16x16_to_64x64_inverse_kernel")
  XOPS_ACCESSOR(recompute_w_u_fwd, RecomputeWUForwardOp, "recompute_w_u_fwd_kernel")
  XOPS_ACCESSOR(chunk_fwd_o, ChunkForwardOOp, "chunk_fwd_kernel_o")
  XOPS_ACCESSOR(causal_conv1d_update_no_cache_no_mtp, CausalConv1dUpdateNoCacheNoMtpOp,
                "_causal_conv1d_update_kernel_no_cache_len_no_mtp")
  XOPS_ACCESSOR(causal_conv1d_update_qwen_decode, CausalConv1dUpdateQwenDecodeOp,
                "_causal_conv1d_update_qwen_decode_kernel")
  XOPS_ACCESSOR(causal_conv1d_update_tiled_v2, CausalConv1dUpdateTiledV2Op,
                "_causal_conv1d_update_kernel_npu_tiled_v2")
  XOPS_ACCESSOR(fused_qkvzba_split_reshape_gqa_r1, FusedQkvzbaSplitReshapeGqaR1Op,
                "fused_qkvzba_split_reshape_cat_gqa_r1_kernel")
  XOPS_ACCESSOR(fused_qkvzba_split_reshape_gqa_r2, FusedQkvzbaSplitReshapeGqaR2Op,
                "fused_qkvzba_split_reshape_cat_gqa_r2_kernel")
  XOPS_ACCESSOR(fused_qkvzba_split_reshape_gqa_r3, FusedQkvzbaSplitReshapeGqaR3Op,
                "fused_qkvzba_split_reshape_cat_gqa_r3_kernel")
  XOPS_ACCESSOR(fused_qkvzba_split_reshape_gqa_r4, FusedQkvzbaSplitReshapeGqaR4Op,
                "fused_qkvzba_split_reshape_cat_gqa_r4_kernel")
#undef XOPS_ACCESSOR

  SplitRmsnormRopeOp& split_rmsnorm_rope(const std::string& kernel_name) {
    std::lock_guard<std::mutex> g(mu_);
    auto& slot = ops_[kernel_name];
    if (!slot) slot = std::make_unique<SplitRmsnormRopeOp>(kernel_name);
    return static_cast<SplitRmsnormRopeOp&>(*slot);
  }

  // An op bound to `kernel_name` (launching an unknown name returns -1).
  // Kept apart from the named accessors' ops, so references handed out by
  // either stay valid.
  OperationBase& by_kernel_name(const std::string& kernel_name) {
    std::lock_guard<std::mutex> g(mu_);
    auto& slot = generic_[kernel_name];
    if (!slot) slot = std::make_unique<OperationBase>(kernel_name);
    return *slot;
  }

 private:
  OperationFactory() = default;

  template <class T>
  T& get(const char* key) {
    std::lock_guard<std::mutex> g(mu_);
    auto& slot = ops_[key];
    if (!slot) slot = std::make_unique<T>();
    return static_cast<T&>(*slot);
  }

  std::mutex mu_;
  std::unordered_map<std::string, std::unique_ptr<OperationBase>> ops_;
  std::unordered_map<std::string, std::unique_ptr<OperationBase>> generic_;
};

}  // namespace xllm::kernel::npu
