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
//
// Speculative decoding (fused_recurrent_gated_delta_rule_spec_fwd_kernel,
// test_fused_recurrent_gated_delta_rule.py:193-307): the initial state is
// read from slot (n, num_accepted_tokens[n] - 1) of a per-token index table
// and the state after every token t is stored to slot (n, t); the plain
// in-place path with a [N, T] index table stores per token the same way
// (:124-165).
//
// The same kernel serves fused_sigmoid_gating_delta_rule_update
// (triton_npu/triton_src/test_fused_sigmoid_gating_delta_rule_update.py:11-117):
// there the gates come from the projections inside the step,
//   g = -exp(A_log[h]) softplus(a + dt_bias[h]),  beta = sigmoid(b),
// and a negative slot index means "start from zeros, write nothing back".
// A negative slot gets that meaning on the plain path too (the reference
// kernel there would address memory before the state buffer).
#include "common.cuh"

namespace xops {
namespace {

// Where a sequence's states live.  idx == nullptr: slot n.  Otherwise the
// slot of (sequence n, token t) is idx[n * stride_seq + t * stride_tok]; the
// initial state comes from token i0 = accepted[n] - 1 (speculative decoding)
// or 0.  per_token: the state after every token t is stored to slot (n, t)
// (the reference's speculative / multi-token in-place path); otherwise the
// final state is stored once.
struct SlotSrc {
  const int32_t* idx;
  int64_t stride_seq, stride_tok;
  const int32_t* accepted;
  bool per_token;
};

// Gates computed in the step from the projections (a.a == nullptr: the
// precomputed g / beta arrays are used instead).
struct GateSrc {
  const float* A_log;
  const void* a;
  const float* dt_bias;
  const void* b;
  int ab_dtype;
  float sp_beta, sp_thr;
};

__device__ __forceinline__ float load_any(const void* p, int64_t i, int dtype) {
  if (dtype == XOPS_F32) return static_cast<const float*>(p)[i];
  if (dtype == XOPS_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  return __half2float(static_cast<const __half*>(p)[i]);
}

// torch Softplus: log(1 + e^{beta x}) / beta, or x once beta x > threshold
__device__ __forceinline__ float softplus_f(float x, float beta, float thr) {
  const float bx = beta * x;
  return bx <= thr ? log1pf(expf(bx)) / beta : x;
}

// PT: the per-token state stores of speculative decoding, compiled separately
// so the plain decode step keeps its register budget (three CTAs per SM for
// the 128 x 128 state).
template <int K, int V, bool PT>
__global__ void __launch_bounds__(128, PT ? 1 : 3) recurrent_gdn_kernel(
    const __nv_bfloat16* __restrict__ q, const __nv_bfloat16* __restrict__ k,
    const __nv_bfloat16* __restrict__ v, const float* __restrict__ g,
    const float* __restrict__ beta, __nv_bfloat16* __restrict__ o,
    const float* h0, float* ht, const int32_t* __restrict__ cu, SlotSrc sl, int64_t T,
    int64_t H, int64_t HV, int64_t h0_stride, int64_t ht_stride, float scale, bool l2norm,
    GateSrc gs) {
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
  if (PT && eos == bos) return;  // nothing to read back or store
  // without per-token stores there is no accepted-token count (it implies
  // them), so the initial slot is the sequence's first index entry
  const int64_t i0 = PT && sl.accepted ? (int64_t)sl.accepted[n] - 1 : 0;
  const int64_t slot =
      sl.idx ? (int64_t)sl.idx[n * sl.stride_seq + (PT ? i0 * sl.stride_tok : 0)] : n;
  const bool inplace = (const float*)ht == h0;
  // a negative slot: zero initial state, and (in place) no write-back
  const bool has_slot = slot >= 0;
  const float* hsrc = h0 + (has_slot ? slot : 0) * h0_stride + (int64_t)hv * K * V;
  // in place (ht == h0): back into the same slot; otherwise ht is indexed by
  // sequence (the reference's INPLACE_FINAL_STATE split, :169-188)
  float* hdst = ht + (inplace ? (has_slot ? slot : 0) : n) * ht_stride + (int64_t)hv * K * V;
  const bool write_back = !PT && (!inplace || has_slot);
  const int r0 = warp * ROWS, c0 = lane * COLS;

  // h0 and ht may be the same buffer (in-place update): each thread reads
  // its slice once here and writes it once at the end, so plain loads.
  float S[ROWS][COLS];
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    float tmp[COLS];
    const float* src = hsrc + (int64_t)(r0 + r) * V + c0;
    if (!has_slot) {
#pragma unroll
      for (int c = 0; c < COLS; ++c) tmp[c] = 0.f;
    } else if constexpr (COLS == 4) {
      const float4 t4 = *reinterpret_cast<const float4*>(src);
      tmp[0] = t4.x; tmp[1] = t4.y; tmp[2] = t4.z; tmp[3] = t4.w;
    } else {
      const float2 t2 = *reinterpret_cast<const float2*>(src);
      tmp[0] = t2.x; tmp[1] = t2.y;
    }
#pragma unroll
    for (int c = 0; c < COLS; ++c) S[r][c] = tmp[c];
  }
  const float neg_a = gs.a ? -expf(gs.A_log[hv]) : 0.f;
  const float dtb = gs.a ? gs.dt_bias[hv] : 0.f;

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
    float decay, b;
    if (gs.a) {
      decay = __expf(neg_a * softplus_f(load_any(gs.a, t * HV + hv, gs.ab_dtype) + dtb,
                                        gs.sp_beta, gs.sp_thr));
      b = 1.0f / (1.0f + expf(-load_any(gs.b, t * HV + hv, gs.ab_dtype)));
    } else {
      decay = __expf(g[t * HV + hv]);
      b = beta ? beta[t * HV + hv] : 1.0f;
    }

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
    if constexpr (PT) {  // the state after token t, to slot (n, t)
      const int64_t st = sl.idx[n * sl.stride_seq + (t - bos) * sl.stride_tok];
      if (st >= 0) {
        float* dst = ht + st * ht_stride + (int64_t)hv * K * V;
#pragma unroll
        for (int r = 0; r < ROWS; ++r) {
          float tmp[COLS];
#pragma unroll
          for (int c = 0; c < COLS; ++c) tmp[c] = S[r][c];
          store_vec<float, COLS>(dst + (int64_t)(r0 + r) * V + c0, tmp);
        }
      }
    }
    __syncthreads();  // s_q/s_k/s_red reused by the next token
  }

  if (!write_back) return;
#pragma unroll
  for (int r = 0; r < ROWS; ++r) {
    float tmp[COLS];
#pragma unroll
    for (int c = 0; c < COLS; ++c) tmp[c] = S[r][c];
    store_vec<float, COLS>(hdst + (int64_t)(r0 + r) * V + c0, tmp);
  }
}

int launch_recurrent(const void* q, const void* k, const void* v, const float* g,
                     const float* beta, void* o, const float* h0, float* ht,
                     const int32_t* cu_seqlens, SlotSrc slots, int64_t T, int64_t N,
                     int64_t H, int64_t HV, int64_t K, int64_t V, int64_t h0_stride,
                     int64_t ht_stride, float scale, bool l2, GateSrc gs, cudaStream_t st,
                     const char* what) {
  const unsigned grid = (unsigned)(N * HV);
#define XOPS_REC(KK, VV)                                                                      \
  if (K == KK && V == VV) {                                                                   \
    auto kern = slots.per_token ? recurrent_gdn_kernel<KK, VV, true>                          \
                                : recurrent_gdn_kernel<KK, VV, false>;                        \
    kern<<<grid, 128, 0, st>>>(                                                               \
        (const __nv_bfloat16*)q, (const __nv_bfloat16*)k, (const __nv_bfloat16*)v, g, beta,   \
        (__nv_bfloat16*)o, h0, ht, cu_seqlens, slots, T, H, HV, h0_stride, ht_stride, scale,  \
        l2, gs);                                                                              \
    return check_launch(what);                                                                \
  }
  XOPS_REC(128, 128)
  XOPS_REC(64, 64)
  XOPS_REC(128, 64)
  XOPS_REC(64, 128)
#undef XOPS_REC
  return set_error(XOPS_ERR_UNSUPPORTED, "%s: unreachable", what);
}

}  // namespace
}  // namespace xops

using namespace xops;

extern "C" int xops_fused_recurrent_gated_delta_rule(
    const void* q, const void* k, const void* v, const float* g, const float* beta, void* o,
    const float* h0, float* ht, const int32_t* cu_seqlens, const int32_t* ssm_state_indices,
    int64_t idx_stride_seq, int64_t idx_stride_tok, const int32_t* num_accepted_tokens,
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
  XOPS_REQUIRE(!num_accepted_tokens || (cu_seqlens && ssm_state_indices),
               "fused_recurrent_gated_delta_rule: speculative decoding needs cu_seqlens and "
               "ssm_state_indices");
  XOPS_REQUIRE(!ssm_state_indices || (idx_stride_seq >= 0 && idx_stride_tok >= 0),
               "fused_recurrent_gated_delta_rule: bad state index strides");
  GateSrc none{};
  // speculative decoding stores every token's state; so does an in-place
  // update with a per-token index table (idx_stride_tok != 0)
  const bool per_token = num_accepted_tokens != nullptr ||
                         (ssm_state_indices && idx_stride_tok != 0 && (const float*)ht == h0);
  SlotSrc sl{ssm_state_indices, ssm_state_indices ? idx_stride_seq : 0,
             ssm_state_indices ? idx_stride_tok : 0, num_accepted_tokens, per_token};
  return launch_recurrent(q, k, v, g, beta, o, h0, ht, cu_seqlens, sl, T, N, H, HV, K, V,
                          h0_stride, ht_stride, scale, use_qk_l2norm_in_kernel != 0, none,
                          (cudaStream_t)stream, "fused_recurrent_gated_delta_rule");
}

extern "C" int xops_fused_sigmoid_gating_delta_rule_update(
    const float* A_log, const void* a, const float* dt_bias, float softplus_beta,
    float softplus_threshold, const void* q, const void* k, const void* v, const void* b,
    void* o, float* initial_state_source, const int32_t* initial_state_indices,
    const int32_t* cu_seqlens, float scale, int64_t B, int64_t T, int64_t N, int64_t H,
    int64_t HV, int64_t K, int64_t V, int ab_dtype, int use_qk_l2norm_in_kernel,
    void* stream) {
  const char* what = "fused_sigmoid_gating_delta_rule_update";
  XOPS_REQUIRE(B >= 1 && T >= 0 && N >= 0 && H >= 1 && HV >= 1, "%s: bad shape", what);
  XOPS_REQUIRE(HV % H == 0, "%s: HV=%lld not divisible by H=%lld", what, (long long)HV,
               (long long)H);
  XOPS_REQUIRE(ab_dtype == XOPS_F32 || ab_dtype == XOPS_BF16 || ab_dtype == XOPS_F16,
               "%s: a/b dtype must be fp32, bf16 or fp16", what);
  XOPS_REQUIRE(softplus_beta > 0.f, "%s: softplus_beta must be positive", what);
  XOPS_UNSUPPORTED((K == 128 || K == 64) && (V == 128 || V == 64),
                   "%s: K, V must be 64 or 128 (got %lld, %lld)", what, (long long)K,
                   (long long)V);
  if (N == 0) return XOPS_OK;
  XOPS_REQUIRE(A_log && a && dt_bias && q && k && v && b && o && initial_state_source &&
                   initial_state_indices && cu_seqlens,
               "%s: null pointer", what);
  XOPS_REQUIRE(aligned16(initial_state_source) && aligned16(v) && aligned16(o),
               "%s: state/v/o must be 16-byte aligned", what);
  GateSrc gs{A_log, a, dt_bias, b, ab_dtype, softplus_beta, softplus_threshold};
  // cu_seqlens index the flattened B*T tokens; the kernel's T only matters
  // without cu_seqlens
  SlotSrc sl{initial_state_indices, 1, 0, nullptr, false};
  return launch_recurrent(q, k, v, nullptr, nullptr, o, initial_state_source,
                          initial_state_source, cu_seqlens, sl, T, N, H, HV, K, V, HV * K * V,
                          HV * K * V, scale, use_qk_l2norm_in_kernel != 0, gs,
                          (cudaStream_t)stream, what);
}
