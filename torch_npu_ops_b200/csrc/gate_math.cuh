// GDN gate arithmetic shared by the standalone gating kernel and the chunked
// gated delta rule's prologue, so that the fused path computes bit for bit
// the gates the two-kernel path stores.
//
// fused_gdn_gating (triton_npu/triton_src/test_fused_gdn_gating.py:10-57):
//   g    = -exp(A_log[h]) * softplus(a + dt_bias[h])      (fp32)
//   beta = sigmoid(b), rounded to b's dtype
// with torch's Softplus(beta, threshold): log(1 + e^{beta x}) / beta, or x
// where beta x > threshold.
#pragma once
#include "common.cuh"

namespace xops {

__device__ __forceinline__ float gate_softplus(float x, float beta, float thr) {
  const float bx = beta * x;
  return bx <= thr ? log1pf(expf(bx)) / beta : x;
}
// g of one element; nega = -expf(A_log[h])
__device__ __forceinline__ float gate_g(float nega, float a, float dt_bias, float sp_beta,
                                        float sp_thr) {
  return nega * gate_softplus(a + dt_bias, sp_beta, sp_thr);
}
// sigmoid(b) before rounding to b's dtype: 16-bit outputs use the fast exp
// and divide (below one ulp of the rounded result), fp32 the full-precision ones
template <typename TB>
__device__ __forceinline__ float gate_beta_f32(float b) {
  if constexpr (sizeof(TB) == 2)
    return __fdividef(1.0f, 1.0f + __expf(-b));
  else
    return 1.0f / (1.0f + expf(-b));
}
// sigmoid(b) as stored in b's dtype, widened back to fp32
template <typename TB>
__device__ __forceinline__ float gate_beta(float b) {
  return to_f32<TB>(from_f32<TB>(gate_beta_f32<TB>(b)));
}

}  // namespace xops
