// Fused recurrent gated delta rule (decode), token-serial.
//
// Follows fused_recurrent_gated_delta_rule_fwd_kernel
// (triton_npu/triton_src/test_fused_recurrent_gated_delta_rule.py:31-190):
// per token  S *= e^g;  v' = beta (v - S^T k);  S += k v'^T;  o = scale S^T q,
// with the optional in-kernel L2 norm  x / sqrt(sum x^2 + 1e-6)  on q and k,
// initial state from slot ssm_state_indices[n] (or n) and the final state
// written to the same slot of ht (in place when ht == h0).
//
// The op is HBM-bound on the fp32 state (K*V*4 bytes read + written per
// sequence and head).  One CTA of 4 warps per (sequence, value head) keeps
// the whole K x V state in registers: warp w owns rows [w*K/4, (w+1)*K/4),
// lane l owns V/32 adjacent columns, so every state load/store is a
// coalesced 16-byte vector (for V = 128) and each thread has K/4
// independent loads in flight.  The two reductions over K (S^T k and S^T q)
// finish across the 4 warps through shared memory.
#include "common.cuh"

namespace xops {
namespace {

template <int K, int V>
__global__ void __launch_bounds__(128) recurrent_gdn_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, const float* __restrict__ g,
    const float* __restrict__ beta, __nv_bfloat16* __restrict__ o,
    const float* h0, float* ht, const int32_t* __restrict__ cu,
    const int32_t* __restrict__ slots, int64_t T, int64_t H, int64_t HV, int64_t h0_stride,
    int64_t ht_stride, float scale, bool l2norm) {
  constexpr int ROWS = K / 4;    // state rows per warp
  constexpr int COLS = V / 32;   // state columns per lane
  __shared__ float s_q[K], s_k[K];
  __shared__ float s_red[4][V];
  __shared__ float s_scal[2];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t n = blockIdx.x / HV;
  const int hv = (int)(blockIdx.x - n * HV);
  const int hk = (int)(hv / (HV / H));
  int64_t bos, eos;
  if (cu) {
    bos = cu[n];
    eos = cu[n + 1];
  } else {
    bos = n * T;
    eos = bos + T;
  }
  const int64_t slot = slots ? (int64_t)slots[n] : n;
  const float* hsrc = h0 + slot * h0_stride + (int64_t)hv * K * V;
  // in place (ht == h0): back into the same slot; otherwise ht is indexed by
  // sequence (the reference's INPLACE_FINAL_STATE split, :169-188)
  float* hdst = ht + ((const float*)ht == h0 ? slot : n) * ht_stride + (int64_t)hv * K * V;
  const int r0 = warp * ROWS, c0 = lane * COLS;

  // h0 and ht may be the same buffer (in-place update): each thread reads
  // its slice once here and writes it once at the end, so plain loads.
  float S[ROWS][COLS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    float tmp[COLS];
    const float* src = hsrc + (int64_t)(r0 + r) * V + c0;
    if constexpr (COLS == 4) {
      const float4 t4 = *reinterpret_cast<const float4*>(src);
      tmp[0] = t4.x; tmp[1] = t4.y; tmp[2] = t4.z; tmp[3] = t4.w;
    } else {
      const float2 t2 = *reinterpret_cast<const float2*>(src);
      tmp[0] = t2.x; tmp[1] = t2.y;
    }
#pragma unroll
    for (int c = 0; c < COLS; ++c) S[r][c] = tmp[c];
  }

  for (int64_t t = bos; t < eos; ++t) {
    // stage q, k (fp32) in shared memory, optionally L2-normalised
    const __nv_bfloat16* qp = q + (t * H + hk) * K;
    const __nv_bfloat16* kp = k + (t * H + hk) * K;
    for (int i = threadIdx.x; i < K; i += 128) {
      s_q[i] = __bfloat162float(qp[i]);
      s_k[i] = __bfloat162float(kp[i]);
    }
    __syncthreads();
    if (warp == 0) {
      float sq = 0.f, sk = 0.f;
      for (int i = lane; i < K; i += 32) {
        sq += s_q[i] * s_q[i];
        sk += s_k[i] * s_k[i];
      }
      sq = warp_sum(sq);
      sk = warp_sum(sk);
      if (lane == 0) {
        s_scal[0] = (l2norm ? 1.0f / sqrtf(sq + 1e-6f) : 1.0f) * scale;
        s_scal[1] = l2norm ? 1.0f / sqrtf(sk + 1e-6f) : 1.0f;
      }
    }
    __syncthreads();
    const float qs = s_scal[0], ks = s_scal[1];
    const float decay = __expf(g[t * HV + hv]);
    const float b = beta ? beta[t * HV + hv] : 1.0f;

    float part[COLS];
#pragma unroll
    for (int c = 0; c < COLS; ++c) part[c] = 0.f;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const float kk = s_k[r0 + r] * ks;
#pragma unroll
      for (int c = 0; c < COLS; ++c) {
        S[r][c] *= decay;
        part[c] = fmaf(S[r][c], kk, part[c]);
      }
    }
#pragma unroll
    for (int c = 0; c < COLS; ++c) s_red[warp][c0 + c] = part[c];
    __syncthreads();
    float vn[COLS];
    {
      float vv[COLS];
      load_vec<__nv_bfloat16, COLS>(v + (t * HV + hv) * V + c0, vv);
#pragma unroll
      for (int c = 0; c < COLS; ++c) {
        const float sk = s_red[0][c0 + c] + s_red[1][c0 + c] + s_red[2][c0 + c] + s_red[3][c0 + c];
        vn[c] = (vv[c] - sk) * b;
      }
    }
    __syncthreads();  // s_red reused below
#pragma unroll
    for (int c = 0; c < COLS; ++c) part[c] = 0.f;
#pragma unroll
    for (int r = 0; r < ROWS; ++r) {
      const float kk = s_k[r0 + r] * ks;
      const float qq = s_q[r0 + r] * qs;
#pragma unroll
      for (int c = 0; c < COLS; ++c) {
        S[r][c] = fmaf(kk, vn[c], S[r][c]);
        part[c] = fmaf(S[r][c], qq, part[c]);
      }
    }
#pragma unroll
    for (int c = 0; c < COLS; ++c) s_red[warp][c0 + c] = part[c];
    __syncthreads();
    if (warp == 0) {
      float ov[COLS];
#pragma unroll
      for (int c = 0; c < COLS; ++c)
        ov[c] = s_red[0][c0 + c] + s_red[1][c0 + c] + s_red[2][c0 + c] + s_red[3][c0 + c];
      store_vec<__nv_bfloat16, COLS>(o + (t * HV + hv) * V + c0, ov);
    }
    __syncthreads();  // s_q/s_k/s_red reused by the next token
  }

#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    float tmp[COLS];
#pragma unroll
    for (int c = 0; c < COLS; ++c) tmp[c] = S[r][c];
    store_vec<float, COLS>(hdst + (int64_t)(r0 + r) * V + c0, tmp);
  }
}

}  // namespace
}  // namespace xops

using namespace xops;

extern "C" int xops_fused_recurrent_gated_delta_rule(
    const void* q, const void* k, const void* v, const float* g, const float* beta, void* o,
    const float* h0, float* ht, const int32_t* cu_seqlens, const int32_t* ssm_state_indices,
    int64_t B, int64_t T, int64_t N, int64_t H, int64_t HV, int64_t K, int64_t V,
    int64_t h0_stride, int64_t ht_stride, float scale, int use_qk_l2norm_in_kernel,
    void* stream) {
  XOPS_REQUIRE(B >= 1 && T >= 0 && N >= 0 && H >= 1 && HV >= 1,
               "fused_recurrent_gated_delta_rule: bad shape");
  XOPS_REQUIRE(HV % H == 0, "fused_recurrent_gated_delta_rule: HV=%lld not divisible by H=%lld",
               (long long)HV, (long long)H);
  XOPS_REQUIRE(cu_seqlens || N == B,
               "fused_recurrent_gated_delta_rule: without cu_seqlens N must equal B");
  XOPS_REQUIRE(!cu_seqlens || B == 1,
               "fused_recurrent_gated_delta_rule: cu_seqlens requires B == 1");
  XOPS_UNSUPPORTED((K == 128 || K == 64) && (V == 128 || V == 64),
                   "fused_recurrent_gated_delta_rule: K, V must be 64 or 128 (got %lld, %lld)",
                   (long long)K, (long long)V);
  XOPS_REQUIRE(h0_stride >= HV * K * V && ht_stride >= HV * K * V,
               "fused_recurrent_gated_delta_rule: state slot stride too small");
  if (N == 0) return XOPS_OK;
  XOPS_REQUIRE(q && k && v && g && o && h0 && ht,
               "fused_recurrent_gated_delta_rule: null pointer");
  XOPS_REQUIRE(aligned16(h0) && aligned16(ht) && aligned16(v) && aligned16(o) &&
                   (h0_stride % 4) == 0 && (ht_stride % 4) == 0,
               "fused_recurrent_gated_delta_rule: state/v/o must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const unsigned grid = (unsigned)(N * HV);
  const bool l2 = use_qk_l2norm_in_kernel != 0;
#define XOPS_REC(KK, VV)                                                                      \
  if (K == KK && V == VV) {                                                                   \
    recurrent_gdn_kernel<KK, VV><<<grid, 128, 0, st>>>(                                       \
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, g, beta,   \
        (__nv_bfloat16*)o, h0, ht, cu_seqlens, ssm_state_indices, T, H, HV, h0_stride,        \
        ht_stride, scale, l2);                                                                \
    return check_launch("fused_recurrent_gated_delta_rule");                                  \
  }
  XOPS_REC(128, 128)
  XOPS_REC(64, 64)
  XOPS_REC(128, 64)
  XOPS_REC(64, 128)
#undef XOPS_REC
  return set_error(XOPS_ERR_UNSUPPORTED, "fused_recurrent_gated_delta_rule: unreachable");
}
