// OperationBase / op classes / OperationFactory with the interface of the
// reference runtime (triton_npu/operation_base.h:128-329, operations.h,
// torch_api/operation_factory.h).  The reference's execute() packs a raw
// argument buffer for an AOT binary; in this build the torch API calls the
// typed C-ABI entry points directly, so execute() only resolves the kernel
// name: it returns 0 when the name maps to a linked entry point and -1
// otherwise, and never launches.  Callers should use the torch API
// functions (triton_ops_api.h) or include/xops_b200.h.
#pragma once

#include <cstdint>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <utility>

#include "args_builder.h"
#include "kernel_registry.h"

namespace xllm::kernel::npu {

class OperationBase {
 public:
  explicit OperationBase(std::string kernel_name, std::string binary_path = "")
      : kernel_name_(std::move(kernel_name)), binary_path_(std::move(binary_path)) {}
  virtual ~OperationBase() = default;

  template <class BuildArgsFn>
  int32_t execute(void* /*stream*/, int32_t /*gridX*/, int32_t /*gridY*/, int32_t /*gridZ*/,
                  BuildArgsFn&& build_args) {
    ArgsBuilder ab;
    build_args(ab);
    last_args_size_ = ab.size();
    return ensure_registered() ? 0 : -1;
  }

  const std::string& kernel_name() const { return kernel_name_; }
  size_t last_args_size() const { return last_args_size_; }

 protected:
  bool ensure_registered() {
    auto& reg = KernelRegistry::get_instance();
    return reg.is_kernel_registered(kernel_name_) || reg.register_kernel(kernel_name_, binary_path_);
  }

 private:
  std::string kernel_name_;
  std::string binary_path_;
  size_t last_args_size_ = 0;
};

#define XOPS_DECLARE_OP(Class, name) \
  class Class final : public OperationBase { \
   public: \
    Class() : OperationBase(name) {} \
  };

XOPS_DECLARE_OP(L2NormFwdOp, "l2norm_fwd_kernel2_loop")
XOPS_DECLARE_OP(LayerNormFwdOp, "layer_norm_fwd_kernel")
XOPS_DECLARE_OP(RecurrentGatedDeltaRuleFwdOp, "fused_recurrent_gated_delta_rule_fwd_kernel")
XOPS_DECLARE_OP(RecurrentGatedDeltaRuleSpecFwdOp, "fused_recurrent_gated_delta_rule_spec_fwd_kernel")
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
XOPS_DECLARE_OP(FusedGdnGatingOp, "fused_gdn_gating_decode_kernel")
XOPS_DECLARE_OP(RopeInplaceOp, "rope_inplace_kernel")
XOPS_DECLARE_OP(FusedSigmoidGatingDeltaRuleUpdateOp, "fused_sigmoid_gating_delta_rule_update_kernel")
XOPS_DECLARE_OP(FusedQkvzbaSplitReshapeGqaR1Op, "fused_qkvzba_split_reshape_cat_gqa_r1_kernel")
XOPS_DECLARE_OP(FusedQkvzbaSplitReshapeGqaR2Op, "fused_qkvzba_split_reshape_cat_gqa_r2_kernel")
XOPS_DECLARE_OP(FusedQkvzbaSplitReshapeGqaR3Op, "fused_qkvzba_split_reshape_cat_gqa_r3_kernel")
XOPS_DECLARE_OP(FusedQkvzbaSplitReshapeGqaR4Op, "fused_qkvzba_split_reshape_cat_gqa_r4_kernel")
#undef XOPS_DECLARE_OP

class SplitRmsnormRopeOp final : public OperationBase {
 public:
  explicit SplitRmsnormRopeOp(std::string name) : OperationBase(std::move(name)) {}
};

// Process-wide op cache keyed by kernel name (thread-safe, unlike the
// reference's unsynchronised map).
class OperationFactory {
 public:
  static OperationFactory& instance() {
    static OperationFactory f;
    return f;
  }
  L2NormFwdOp& l2norm_fwd() { return get<L2NormFwdOp>("l2norm_fwd_kernel2_loop"); }
  LayerNormFwdOp& layer_norm_fwd() { return get<LayerNormFwdOp>("layer_norm_fwd_kernel"); }
  RecurrentGatedDeltaRuleFwdOp& recurrent_gated_delta_rule_fwd() {
    return get<RecurrentGatedDeltaRuleFwdOp>("fused_recurrent_gated_delta_rule_fwd_kernel");
  }
  RecurrentGatedDeltaRuleSpecFwdOp& recurrent_gated_delta_rule_spec_fwd() {
    return get<RecurrentGatedDeltaRuleSpecFwdOp>("fused_recurrent_gated_delta_rule_spec_fwd_kernel");
  }
  ChunkGatedDeltaRuleFwdHOp& chunk_gated_delta_rule_fwd_h() {
    return get<ChunkGatedDeltaRuleFwdHOp>("chunk_gated_delta_rule_fwd_kernel_h_blockdim64");
  }
  ChunkLocalCumsumScalarOp& chunk_local_cumsum_scalar() {
    return get<ChunkLocalCumsumScalarOp>("chunk_local_cumsum_scalar_kernel");
  }
  ChunkScaledDotKktFwdOp& chunk_scaled_dot_kkt_fwd() {
    return get<ChunkScaledDotKktFwdOp>("chunk_scaled_dot_kkt_fwd_kernel");
  }
  SolveTril16x16Op& solve_tril_16x16() { return get<SolveTril16x16Op>("solve_tril_16x16_kernel"); }
  Merge16x16To64x64InverseOp& merge_16x16_to_64x64_inverse() {
    return get<Merge16x16To64x64InverseOp>("merge_16x16_to_64x64_inverse_kernel");
  }
  RecomputeWUForwardOp& recompute_w_u_fwd() {
    return get<RecomputeWUForwardOp>("recompute_w_u_fwd_kernel");
  }
  ChunkForwardOOp& chunk_fwd_o() { return get<ChunkForwardOOp>("chunk_fwd_kernel_o"); }
  CausalConv1dUpdateNoCacheNoMtpOp& causal_conv1d_update_no_cache_no_mtp() {
    return get<CausalConv1dUpdateNoCacheNoMtpOp>("_causal_conv1d_update_kernel_no_cache_len_no_mtp");
  }
  CausalConv1dUpdateQwenDecodeOp& causal_conv1d_update_qwen_decode() {
    return get<CausalConv1dUpdateQwenDecodeOp>("_causal_conv1d_update_qwen_decode_kernel");
  }
  CausalConv1dUpdateTiledV2Op& causal_conv1d_update_tiled_v2() {
    return get<CausalConv1dUpdateTiledV2Op>("_causal_conv1d_update_kernel_npu_tiled_v2");
  }
  RopeInplaceOp& rope_inplace() { return get<RopeInplaceOp>("rope_inplace_kernel"); }
  FusedGdnGatingOp& fused_gdn_gating() {
    return get<FusedGdnGatingOp>("fused_gdn_gating_decode_kernel");
  }
  FusedSigmoidGatingDeltaRuleUpdateOp& fused_sigmoid_gating_delta_rule_update() {
    return get<FusedSigmoidGatingDeltaRuleUpdateOp>(
        "fused_sigmoid_gating_delta_rule_update_kernel");
  }
  FusedQkvzbaSplitReshapeGqaR1Op& fused_qkvzba_split_reshape_gqa_r1() {
    return get<FusedQkvzbaSplitReshapeGqaR1Op>("fused_qkvzba_split_reshape_cat_gqa_r1_kernel");
  }
  FusedQkvzbaSplitReshapeGqaR2Op& fused_qkvzba_split_reshape_gqa_r2() {
    return get<FusedQkvzbaSplitReshapeGqaR2Op>("fused_qkvzba_split_reshape_cat_gqa_r2_kernel");
  }
  FusedQkvzbaSplitReshapeGqaR3Op& fused_qkvzba_split_reshape_gqa_r3() {
    return get<FusedQkvzbaSplitReshapeGqaR3Op>("fused_qkvzba_split_reshape_cat_gqa_r3_kernel");
  }
  FusedQkvzbaSplitReshapeGqaR4Op& fused_qkvzba_split_reshape_gqa_r4() {
    return get<FusedQkvzbaSplitReshapeGqaR4Op>("fused_qkvzba_split_reshape_cat_gqa_r4_kernel");
  }
  SplitRmsnormRopeOp& split_rmsnorm_rope(const std::string& kernel_name) {
    std::lock_guard<std::mutex> g(mu_);
    auto& slot = ops_[kernel_name];
    if (!slot) slot = std::make_unique<SplitRmsnormRopeOp>(kernel_name);
    return static_cast<SplitRmsnormRopeOp&>(*slot);
  }

 private:
  template <class T>
  T& get(const char* key) {
    std::lock_guard<std::mutex> g(mu_);
    auto& slot = ops_[key];
    if (!slot) slot = std::make_unique<T>();
    return static_cast<T&>(*slot);
  }
  std::mutex mu_;
  std::unordered_map<std::string, std::unique_ptr<OperationBase>> ops_;
};

}  // namespace xllm::kernel::npu
