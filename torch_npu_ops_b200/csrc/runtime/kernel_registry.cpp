#include "kernel_registry.h"

#include <mutex>
#include <unordered_set>
#include <utility>

#include "xops_b200.h"

namespace xllm::kernel::npu {
namespace {

struct Entry {
  const char* kernel;  // reference kernel name (or name prefix ending in '*')
  const char* symbol;
  void* fn;
};

// Reference kernel names (triton_npu/operations.h:26-223) -> linked entry points.
const Entry kTable[] = {
    {"l2norm_fwd_kernel2_loop", "xops_l2norm_last_dim", (void*)&xops_l2norm_last_dim},
    {"layer_norm_fwd_kernel*", "xops_layer_norm_fwd", (void*)&xops_layer_norm_fwd},
    {"split_rmsnorm_rope_kernel*", "xops_split_rmsnorm_rope", (void*)&xops_split_rmsnorm_rope},
    {"_causal_conv1d_update_kernel_no_cache_len_no_mtp", "xops_causal_conv1d_update",
     (void*)&xops_causal_conv1d_update},
    {"_causal_conv1d_update_qwen_decode_kernel", "xops_causal_conv1d_update",
     (void*)&xops_causal_conv1d_update},
    {"_causal_conv1d_update_kernel_npu_tiled_v2", "xops_causal_conv1d_varlen",
     (void*)&xops_causal_conv1d_varlen},
    {"fused_recurrent_gated_delta_rule_fwd_kernel", "xops_fused_recurrent_gated_delta_rule",
     (void*)&xops_fused_recurrent_gated_delta_rule},
    {"fused_recurrent_gated_delta_rule_spec_fwd_kernel", "xops_fused_recurrent_gated_delta_rule",
     (void*)&xops_fused_recurrent_gated_delta_rule},
    {"fused_gdn_gating_decode_kernel", "xops_fused_gdn_gating", (void*)&xops_fused_gdn_gating},
    {"rope_inplace_kernel", "xops_rope_inplace", (void*)&xops_rope_inplace},
    {"fused_qkvzba_split_reshape_cat_gqa_r*", "xops_fused_qkvzba_split_reshape_cat",
     (void*)&xops_fused_qkvzba_split_reshape_cat},
    {"fused_sigmoid_gating_delta_rule_update_kernel",
     "xops_fused_sigmoid_gating_delta_rule_update",
     (void*)&xops_fused_sigmoid_gating_delta_rule_update},
    {"chunk_local_cumsum_scalar_kernel", "xops_chunk_local_cumsum",
     (void*)&xops_chunk_local_cumsum},
    {"chunk_scaled_dot_kkt_fwd_kernel", "xops_chunk_scaled_dot_kkt_fwd",
     (void*)&xops_chunk_scaled_dot_kkt_fwd},
    {"solve_tril_16x16_kernel", "xops_solve_tril", (void*)&xops_solve_tril},
    {"merge_16x16_to_64x64_inverse_kernel", "xops_solve_tril", (void*)&xops_solve_tril},
    {"recompute_w_u_fwd_kernel", "xops_recompute_w_u_fwd", (void*)&xops_recompute_w_u_fwd},
    {"chunk_gated_delta_rule_fwd_kernel_h_blockdim64", "xops_chunk_gated_delta_rule_fwd_h",
     (void*)&xops_chunk_gated_delta_rule_fwd_h},
    {"chunk_fwd_kernel_o", "xops_chunk_fwd_o", (void*)&xops_chunk_fwd_o},
};

const Entry* find(const std::string& name) {
  for (const auto& e : kTable) {
    const std::string k = e.kernel;
    if (!k.empty() && k.back() == '*') {
      if (name.compare(0, k.size() - 1, k, 0, k.size() - 1) == 0) return &e;
    } else if (name == k) {
      return &e;
    }
  }
  return nullptr;
}

std::mutex g_mu;
std::unordered_set<std::string> g_registered;

}  // namespace

KernelRegistry& KernelRegistry::get_instance() {
  static KernelRegistry r;
  return r;
}

bool KernelRegistry::register_kernel(const std::string& kernel_name, const std::string&) {
  if (!find(kernel_name)) return false;
  std::lock_guard<std::mutex> g(g_mu);
  g_registered.insert(kernel_name);
  return true;
}

KernelStubHandle KernelRegistry::get_kernel_stub(const std::string& kernel_name) const {
  const Entry* e = find(kernel_name);
  return e ? e->fn : nullptr;
}

bool KernelRegistry::is_kernel_registered(const std::string& kernel_name) const {
  std::lock_guard<std::mutex> g(g_mu);
  return g_registered.count(kernel_name) != 0;
}

void KernelRegistry::cleanup() {
  std::lock_guard<std::mutex> g(g_mu);
  g_registered.clear();
}

bool KernelRegistry::get_kernel_workspace_config(const std::string& kernel_name,
                                                 int64_t& workspace_size, int64_t& lock_init_value,
                                                 int64_t& lock_num) const {
  workspace_size = 0;
  lock_init_value = 0;
  lock_num = 0;
  return find(kernel_name) != nullptr;
}

std::string KernelRegistry::entry_point(const std::string& kernel_name) const {
  const Entry* e = find(kernel_name);
  return e ? e->symbol : "";
}

}  // namespace xllm::kernel::npu
