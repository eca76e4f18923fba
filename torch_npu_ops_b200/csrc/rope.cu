// Fused q/k RMSNorm + NeoX RoPE (full or partial rotary) + v copy.
//
// Semantics follow split_rmsnorm_rope_kernel
// (triton_npu/triton_src/test_split_rmsnorm_rope.py:63-221): split the packed
// row into q | k | v, RMS-normalise every q and k head with the shared
// weight (and bias), rotate with x*cos + rotate_half(x)*sin, copy v.  The
// rotation here covers the first rotary_dim dims of each head (the reference
// kernel only handles rotary_dim == head_dim); the rest pass through.
//
// HBM-bound: every input element is read once and written once.  One warp
// per (token, head); a lane owns head_dim/32 contiguous elements (16-byte
// vectors for head_dim 256 in fp32/bf16), the RMS statistic is a warp
// shuffle reduction and the rotate-half partner comes from a per-warp
// shared-memory row, so any even rotary_dim works.
#include "common.cuh"

namespace xops {
namespace {

template <typename T, typename TW, typename TS, int EPL>
__global__ void __launch_bounds__(256) split_rmsnorm_rope_kernel(
    const T* __restrict__ in, const TS* __restrict__ sin_t, const TS* __restrict__ cos_t,
    T* __restrict__ qo, T* __restrict__ ko, T* __restrict__ vo, const TW* __restrict__ qw,
    const TW* __restrict__ qb, const TW* __restrict__ kw, const TW* __restrict__ kb,
    int64_t T_, int qh, int kvh, int rd, float eps) {
  constexpr int HD = EPL * 32;
  __shared__ float rowbuf[8][HD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = qh + 2 * kvh;
  const int64_t item = (int64_t)blockIdx.x * 8 + warp;
  if (item >= T_ * heads) return;
  const int64_t t = item / heads;
  const int hh = (int)(item - t * heads);
  const int64_t total = (int64_t)heads * HD;
  const T* src = in + t * total + (int64_t)hh * HD + lane * EPL;
  float v[EPL];
  load_vec<T, EPL>(src, v);
  if (hh >= qh + kvh) {  // v head: plain copy
    store_vec<T, EPL>(vo + t * (int64_t)kvh * HD + (int64_t)(hh - qh - kvh) * HD + lane * EPL, v);
    return;
  }
  const bool is_q = hh < qh;
  const TW* w = is_q ? qw : kw;
  const TW* b = is_q ? qb : kb;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) ss += v[i] * v[i];
  const float r = 1.0f / sqrtf(warp_sum(ss) * (1.0f / HD) + eps);
  float wv[EPL];
  load_vec<TW, EPL>(w + lane * EPL, wv);
  if (b != nullptr) {
    float bv[EPL];
    load_vec<TW, EPL>(b + lane * EPL, bv);
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = v[i] * r * wv[i] + bv[i];
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = v[i] * r * wv[i];
  }
#pragma unroll
  for (int i = 0; i < EPL; ++i) rowbuf[warp][lane * EPL + i] = v[i];
  __syncwarp();
  const int half = rd >> 1;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int d = lane * EPL + i;
    if (d < rd) {
      const float c = to_f32<TS>(cos_t[t * rd + d]);
      const float s = to_f32<TS>(sin_t[t * rd + d]);
      const float partner = d < half ? -rowbuf[warp][d + half] : rowbuf[warp][d - half];
      v[i] = v[i] * c + partner * s;
    }
  }
  T* dst = is_q ? qo + t * (int64_t)qh * HD + (int64_t)hh * HD
                : ko + t * (int64_t)kvh * HD + (int64_t)(hh - qh) * HD;
  store_vec<T, EPL>(dst + lane * EPL, v);
}

template <typename T, typename TW, typename TS>
int dispatch_rope(const void* in, const void* s, const void* c, void* q, void* k, void* v,
                  const void* qw, const void* qb, const void* kw, const void* kb, int64_t T_,
                  int qh, int kvh, int hd, int rd, float eps, cudaStream_t st) {
  const int64_t items = T_ * (qh + 2 * kvh);
  const unsigned blocks = (unsigned)cdiv64(items, 8);
  switch (hd) {
#define XOPS_R_CASE(EPL)                                                                      \
  case 32 * EPL:                                                                              \
    split_rmsnorm_rope_kernel<T, TW, TS, EPL><<<blocks, 256, 0, st>>>(                        \
        (const T*)in, (const TS*)s, (const TS*)c, (T*)q, (T*)k, (T*)v, (const TW*)qw,         \
        (const TW*)qb, (const TW*)kw, (const TW*)kb, T_, qh, kvh, rd, eps);                   \
    return check_launch("split_rmsnorm_rope");
    XOPS_R_CASE(2)
    XOPS_R_CASE(4)
    XOPS_R_CASE(8)
    XOPS_R_CASE(16)
#undef XOPS_R_CASE
    default:
      return set_error(XOPS_ERR_UNSUPPORTED,
                       "split_rmsnorm_rope: head_dim %d not in {64,128,256,512}", hd);
  }
}

}  // namespace
}  // namespace xops

using namespace xops;

extern "C" int xops_split_rmsnorm_rope(const void* input, const void* sin, const void* cos,
                                       void* q_out, void* k_out, void* v_out,
                                       const void* q_weight, const void* q_bias,
                                       const void* k_weight, const void* k_bias,
                                       int64_t num_tokens, int64_t q_hidden, int64_t kv_hidden,
                                       int64_t head_dim, int64_t rotary_dim, float eps,
                                       int dtype, int w_dtype, int sincos_dtype, void* stream) {
  XOPS_REQUIRE(num_tokens >= 0, "split_rmsnorm_rope: bad num_tokens");
  XOPS_REQUIRE(head_dim > 0 && (head_dim & (head_dim - 1)) == 0,
               "split_rmsnorm_rope head_dim must be a power of two");
  XOPS_REQUIRE(kv_hidden > 0 && kv_hidden % head_dim == 0,
               "split_rmsnorm_rope kv_hidden_size must be divisible by head_dim");
  XOPS_REQUIRE(q_hidden % kv_hidden == 0,
               "split_rmsnorm_rope q_hidden_size must be divisible by kv_hidden_size");
  XOPS_REQUIRE(rotary_dim > 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0,
               "split_rmsnorm_rope: rotary_dim must be even and in (0, head_dim]");
  XOPS_REQUIRE(dtype == XOPS_F32 || dtype == XOPS_BF16, "split_rmsnorm_rope: bad dtype");
  XOPS_REQUIRE(w_dtype == XOPS_F32 || w_dtype == XOPS_BF16, "split_rmsnorm_rope: bad weight dtype");
  XOPS_REQUIRE(sincos_dtype == XOPS_F32 || sincos_dtype == XOPS_BF16,
               "split_rmsnorm_rope: bad sin/cos dtype");
  if (num_tokens == 0) return XOPS_OK;
  XOPS_REQUIRE(input && sin && cos && q_out && k_out && v_out && q_weight && k_weight,
               "split_rmsnorm_rope: null pointer");
  XOPS_REQUIRE((q_bias == nullptr) == (k_bias == nullptr),
               "split_rmsnorm_rope: q_bias and k_bias must both be given or both be null");
  XOPS_REQUIRE(aligned16(input) && aligned16(q_out) && aligned16(k_out) && aligned16(v_out) &&
                   aligned16(q_weight) && aligned16(k_weight),
               "split_rmsnorm_rope: tensors must be 16-byte aligned");
  const int qh = (int)(q_hidden / head_dim), kvh = (int)(kv_hidden / head_dim);
  cudaStream_t st = (cudaStream_t)stream;
  auto run = [&](auto t, auto tw, auto ts) {
    return dispatch_rope<decltype(t), decltype(tw), decltype(ts)>(
        input, sin, cos, q_out, k_out, v_out, q_weight, q_bias, k_weight, k_bias, num_tokens, qh,
        kvh, (int)head_dim, (int)rotary_dim, eps, st);
  };
  auto with_s = [&](auto t, auto tw) {
    return sincos_dtype == XOPS_F32 ? run(t, tw, float{}) : run(t, tw, __nv_bfloat16{});
  };
  auto with_w = [&](auto t) {
    return w_dtype == XOPS_F32 ? with_s(t, float{}) : with_s(t, __nv_bfloat16{});
  };
  return dtype == XOPS_F32 ? with_w(float{}) : with_w(__nv_bfloat16{});
}
