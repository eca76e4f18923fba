// C++ operator API of the hot path, signature-compatible with the reference's
// xllm::kernel::npu torch API (triton_npu/torch_api/triton_ops_api.h:29-198),
// backed by the sm_100a kernels through the C ABI in include/xops_b200.h.
//
// Tensors live on a CUDA device; every op launches on the current CUDA stream
// of its input's device and never synchronises, except where the reference's
// own op reads cu_seqlens on the host (npu_chunk_gated_delta_rule_fwd_h
// without chunk_offsets).  Bad arguments raise c10::Error (TORCH_CHECK), as
// in the reference; a failing launch raises too instead of being logged.
// Ops of the reference API outside this build's scope are declared and throw
// when called.
#pragma once

#include <torch/torch.h>

#include <optional>
#include <tuple>
#include <utility>

namespace xllm::kernel::npu {

torch::Tensor npu_l2norm_last_dim(torch::Tensor& x, double eps = 1e-6);

torch::Tensor npu_chunk_local_cumsum(const torch::Tensor& g, int64_t chunk_size,
                                     const std::optional<torch::Tensor>& cu_seqlens);

torch::Tensor npu_chunk_scaled_dot_kkt_fwd(const torch::Tensor& k, const torch::Tensor& beta,
                                           const torch::Tensor& g_cumsum, int64_t chunk_size,
                                           const std::optional<torch::Tensor>& cu_seqlens);

torch::Tensor npu_solve_tril(const torch::Tensor& A, int64_t chunk_size,
                             const std::optional<torch::Tensor>& cu_seqlens,
                             torch::ScalarType output_dtype);

std::pair<torch::Tensor, torch::Tensor> npu_recompute_w_u_fwd(
    const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& beta,
    const torch::Tensor& g_cumsum, const torch::Tensor& A,
    const std::optional<torch::Tensor>& cu_seqlens);

torch::Tensor npu_chunk_fwd_o(const torch::Tensor& q, const torch::Tensor& k,
                              const torch::Tensor& v, const torch::Tensor& h,
                              const torch::Tensor& g_cumsum, float scale, int64_t chunk_size,
                              const std::optional<torch::Tensor>& cu_seqlens);

// Interleaved RoPE on the last rope_dim dims of x (MLA tail), in place.
void rope_inplace(torch::Tensor& x, torch::Tensor& sin, torch::Tensor& cos,
                  uint32_t rope_dim = 64);

// GDN gates from the projections: g = -exp(A_log) softplus(a + dt_bias) fp32,
// beta = sigmoid(b); both [1, batch, heads].
std::pair<torch::Tensor, torch::Tensor> npu_fused_gdn_gating(torch::Tensor& A_log,
                                                             torch::Tensor& a, torch::Tensor& b,
                                                             torch::Tensor& dt_bias,
                                                             float beta = 1.0f,
                                                             float threshold = 20.0f);

std::pair<torch::Tensor, torch::Tensor> npu_fused_recurrent_gated_delta_rule(
    torch::Tensor& q, torch::Tensor& k, torch::Tensor& v, torch::Tensor& g,
    const std::optional<torch::Tensor>& beta = std::nullopt,
    const std::optional<float>& scale = std::nullopt,
    const std::optional<torch::Tensor>& initial_state = std::nullopt,
    bool inplace_final_state = true,
    const std::optional<torch::Tensor>& cu_seqlens = std::nullopt,
    const std::optional<torch::Tensor>& ssm_state_indices = std::nullopt,
    const std::optional<torch::Tensor>& num_accepted_tokens = std::nullopt,
    bool use_qk_l2norm_in_kernel = false);

// The recurrent update with the gates computed from the projections in the
// step; updates initial_state_source in place, returns o [B, T, HV, V].
torch::Tensor npu_fused_sigmoid_gating_delta_rule_update(
    torch::Tensor& A_log, torch::Tensor& a, torch::Tensor& dt_bias, torch::Tensor& q,
    torch::Tensor& k, torch::Tensor& v, torch::Tensor& b, torch::Tensor& initial_state_source,
    torch::Tensor& initial_state_indices, torch::Tensor& cu_seqlens,
    const std::optional<float>& scale = std::nullopt, bool use_qk_l2norm_in_kernel = false,
    float softplus_beta = 1.0f, float softplus_threshold = 20.0f);

std::pair<torch::Tensor, torch::Tensor> npu_chunk_gated_delta_rule(
    torch::Tensor& q, torch::Tensor& k, torch::Tensor& v, torch::Tensor& g, torch::Tensor& beta,
    const std::optional<float>& scale = std::nullopt,
    const std::optional<torch::Tensor>& initial_state = std::nullopt,
    bool output_final_state = false,
    const std::optional<torch::Tensor>& cu_seqlens = std::nullopt, bool head_first = false,
    bool use_qk_l2norm_in_kernel = false);

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> npu_chunk_gated_delta_rule_fwd_h(
    torch::Tensor& k, torch::Tensor& w, torch::Tensor& u,
    const std::optional<torch::Tensor>& g = std::nullopt,
    const std::optional<torch::Tensor>& initial_state = std::nullopt,
    bool output_final_state = false, int64_t chunk_size = 64, bool save_new_value = true,
    const std::optional<torch::Tensor>& cu_seqlens = std::nullopt,
    const std::optional<torch::Tensor>& chunk_offsets = std::nullopt);

torch::Tensor layer_norm_fwd(torch::Tensor& x, torch::Tensor& weight, torch::Tensor& bias,
                             double eps, const std::optional<torch::Tensor>& z = std::nullopt,
                             int64_t group_size = -1, bool norm_before_gate = true,
                             bool is_rms_norm = false);

torch::Tensor npu_causal_conv1d_update(
    torch::Tensor& x, torch::Tensor& conv_state, torch::Tensor& weight, bool activation = true,
    const std::optional<torch::Tensor>& bias = std::nullopt,
    const std::optional<torch::Tensor>& cache_seqlens = std::nullopt,
    const std::optional<torch::Tensor>& conv_state_indices = std::nullopt,
    const std::optional<torch::Tensor>& num_accepted_tokens = std::nullopt,
    const std::optional<torch::Tensor>& query_start_loc = std::nullopt,
    int32_t max_query_len = -1,
    const std::optional<torch::Tensor>& intermediate_conv_window = std::nullopt,
    int32_t pad_slot_id = -1, bool validate_data = false);

torch::Tensor npu_causal_conv1d_update_v2(
    torch::Tensor& x, torch::Tensor& conv_state, torch::Tensor& weight, bool activation = true,
    const std::optional<torch::Tensor>& bias = std::nullopt,
    const std::optional<torch::Tensor>& conv_state_indices = std::nullopt,
    const std::optional<torch::Tensor>& query_start_loc = std::nullopt,
    int32_t max_query_len = -1, int32_t pad_slot_id = -1,
    const std::optional<torch::Tensor>& block_idx_last_scheduled_token = std::nullopt,
    const std::optional<torch::Tensor>& initial_state_idx = std::nullopt,
    bool validate_data = false,
    const std::optional<torch::Tensor>& num_accepted_tokens = std::nullopt);

// De-interleave of the GDN input projections -> (mixed_qkv, z [rows, nv, hv], b, a).
std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor>
npu_fused_qkvzba_split_reshape_cat(torch::Tensor& mixed_qkvz, torch::Tensor& mixed_ba,
                                   int32_t num_heads_qk, int32_t num_heads_v, int32_t head_qk,
                                   int32_t head_v);

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> npu_split_rmsnorm_rope(
    torch::Tensor& input, torch::Tensor& sin, torch::Tensor& cos, torch::Tensor& q_weight,
    torch::Tensor& k_weight, int64_t q_hidden_size, int64_t kv_hidden_size, int64_t head_dim,
    double eps, const std::optional<torch::Tensor>& q_bias = std::nullopt,
    const std::optional<torch::Tensor>& k_bias = std::nullopt, bool bias = false);

}  // namespace xllm::kernel::npu
