// npu_ops API (ascendc_npu/ascendc_ops_api.h:24-39 of the reference), backed
// by the sm_100a norm kernels through the C ABI.
#pragma once

#include <torch/torch.h>

namespace npu_ops {

// Gemma RMSNorm: yOut = x * rsqrt(mean(x^2) + eps) * (1 + gamma) over the
// trailing gamma.dim() axes; rstdOut fp32 of shape x.shape[:-gamma.dim()] +
// (1,) * gamma.dim().
void npu_gemma_rms_norm(const torch::Tensor& x, const torch::Tensor& gamma, double epsilon,
                        torch::Tensor& rstdOut, torch::Tensor& yOut);

torch::Tensor layer_norm_fwd(const torch::Tensor& x, const torch::Tensor& weight,
                             const c10::optional<torch::Tensor>& bias, double eps,
                             const c10::optional<torch::Tensor>& z, int64_t group_size,
                             bool norm_before_gate, bool is_rms_norm);

}  // namespace npu_ops
