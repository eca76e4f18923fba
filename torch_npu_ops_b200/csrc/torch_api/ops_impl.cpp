// xllm::kernel::npu / npu_ops implementations over the C ABI: validation
// mirrors the reference's TORCH_CHECKs, outputs are allocated with the
// torch caching allocator, launches go to the current CUDA stream.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cmath>
#include <vector>

#include "ascendc_ops_api.h"
#include "triton_ops_api.h"
#include "xops_b200.h"

namespace {

void* P(const torch::Tensor& t) { return t.defined() ? t.data_ptr() : nullptr; }
template <typename T>
T* PT(const torch::Tensor& t) { return t.defined() ? t.data_ptr<T>() : nullptr; }

void* stream_of(const torch::Tensor& t) {
  return at::cuda::getCurrentCUDAStream(t.device().index()).stream();
}

int dtype_code(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case torch::kFloat32: return XOPS_F32;
    case torch::kBFloat16: return XOPS_BF16;
    case torch::kFloat16: return XOPS_F16;
    default: TORCH_CHECK(false, "unsupported dtype ", t.scalar_type());
  }
  return -1;
}

void on_cuda(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(!t.defined() || t.is_cuda(), name, " must be a CUDA tensor");
}

void ok(int rc, const char* what) {
  TORCH_CHECK(rc == XOPS_OK, what, " failed (status ", rc, "): ", xops_last_error());
}

torch::Tensor i32(const std::optional<torch::Tensor>& t) {
  return t.has_value() ? t->to(torch::kInt32).contiguous() : torch::Tensor();
}

// [B, T, H, D] view whose heads/dims are contiguous inside a token, with a
// 16-byte aligned token stride (slices of a packed projection); else a copy.
torch::Tensor token_rows(const torch::Tensor& x) {
  const bool good = x.stride(3) == 1 && x.stride(2) == x.size(3) && x.stride(1) % 8 == 0 &&
                    (x.size(0) == 1 || x.stride(0) == x.size(1) * x.stride(1)) &&
                    reinterpret_cast<uintptr_t>(x.data_ptr()) % 16 == 0;
  return good ? x : x.contiguous();
}

int64_t host_total_chunks(const torch::Tensor& cu, int64_t B, int64_t T, int64_t N) {
  if (!cu.defined()) return B * ((T + 63) / 64);
  auto h = cu.to(torch::kCPU).contiguous();
  return xops_total_chunks(h.data_ptr<int32_t>(), B, T, N, 64);
}

}  // namespace

namespace xllm::kernel::npu {

torch::Tensor npu_l2norm_last_dim(torch::Tensor& x, double eps) {
  on_cuda(x, "x");
  TORCH_CHECK(x.scalar_type() == torch::kBFloat16 || x.scalar_type() == torch::kFloat32,
              "x tensor must be bfloat16");
  TORCH_CHECK(x.dim() >= 1, "npu_l2norm_last_dim expects x.dim() >= 1");
  const int64_t cols = x.size(-1);
  TORCH_CHECK(cols > 0, "npu_l2norm_last_dim expects hidden dim > 0");
  auto xc = x.contiguous();
  auto y = torch::empty_like(xc);
  const int64_t rows = xc.numel() / cols;
  TORCH_CHECK(rows > 0, "npu_l2norm_last_dim expects non-empty input");
  ok(xops_l2norm_last_dim(P(xc), P(y), rows, cols, (float)eps, dtype_code(x), stream_of(x)),
     "npu_l2norm_last_dim");
  return y.view(x.sizes());
}

torch::Tensor npu_chunk_local_cumsum(const torch::Tensor& g2, int64_t chunk_size,
                                     const std::optional<torch::Tensor>& cu_seqlens) {
  auto g = g2.to(torch::kFloat32).contiguous();
  TORCH_CHECK(g.dim() == 3, "chunk_local_cumsum expects g to have shape [B, T, H].");
  TORCH_CHECK(chunk_size > 0 && (chunk_size & (chunk_size - 1)) == 0,
              "chunk_local_cumsum expects chunk_size to be a power of two, got ", chunk_size);
  on_cuda(g, "g");
  auto cu = i32(cu_seqlens);
  const int64_t B = g.size(0), T = g.size(1), H = g.size(2);
  const int64_t N = cu.defined() ? cu.numel() - 1 : B;
  auto out = torch::empty_like(g);
  ok(xops_chunk_local_cumsum(PT<float>(g), PT<float>(out), PT<int32_t>(cu), B, T, N, H,
                             chunk_size, stream_of(g)),
     "npu_chunk_local_cumsum");
  return out;
}

torch::Tensor npu_chunk_scaled_dot_kkt_fwd(const torch::Tensor& k, const torch::Tensor& beta,
                                           const torch::Tensor& g_cumsum, int64_t chunk_size,
                                           const std::optional<torch::Tensor>& cu_seqlens) {
  on_cuda(k, "k");
  TORCH_CHECK(k.scalar_type() == torch::kBFloat16, "chunk_scaled_dot_kkt_fwd expects bf16 k");
  auto cu = i32(cu_seqlens);
  const int64_t B = k.size(0), T = k.size(1), Hg = k.size(2), K = k.size(3), H = beta.size(-1);
  const int64_t N = cu.defined() ? cu.numel() - 1 : B;
  auto A = torch::zeros({B, T, H, chunk_size}, k.options().dtype(torch::kFloat32));
  auto kc = k.contiguous();
  auto bb = beta.to(torch::kFloat32).contiguous();
  auto gc = g_cumsum.defined() ? g_cumsum.to(torch::kFloat32).contiguous() : torch::Tensor();
  ok(xops_chunk_scaled_dot_kkt_fwd(P(kc), PT<float>(bb), PT<float>(gc), PT<float>(A),
                                   PT<int32_t>(cu), B, T, N, Hg, H, K, chunk_size, stream_of(k)),
     "npu_chunk_scaled_dot_kkt_fwd");
  return A;
}

torch::Tensor npu_solve_tril(const torch::Tensor& A, int64_t chunk_size,
                             const std::optional<torch::Tensor>& cu_seqlens,
                             torch::ScalarType output_dtype) {
  on_cuda(A, "A");
  auto Af = A.to(torch::kFloat32).contiguous();
  auto cu = i32(cu_seqlens);
  const int64_t B = Af.size(0), T = Af.size(1), H = Af.size(2);
  const int64_t N = cu.defined() ? cu.numel() - 1 : B;
  auto Ai = torch::zeros(Af.sizes(), Af.options().dtype(output_dtype));
  ok(xops_solve_tril(PT<float>(Af), P(Ai), PT<int32_t>(cu), B, T, N, H, chunk_size,
                     dtype_code(Ai), stream_of(A)),
     "npu_solve_tril");
  return Ai;
}

std::pair<torch::Tensor, torch::Tensor> npu_recompute_w_u_fwd(
    const torch::Tensor& k, const torch::Tensor& v, const torch::Tensor& beta,
    const torch::Tensor& g_cumsum, const torch::Tensor& A,
    const std::optional<torch::Tensor>& cu_seqlens) {
  on_cuda(k, "k");
  auto cu = i32(cu_seqlens);
  const int64_t B = k.size(0), T = k.size(1), Hg = k.size(2), K = k.size(3);
  const int64_t H = v.size(2), V = v.size(3);
  const int64_t N = cu.defined() ? cu.numel() - 1 : B;
  auto w = torch::empty({B, T, H, K}, k.options());
  auto u = torch::empty_like(v);
  auto kc = k.contiguous(), vc = v.contiguous(), Ac = A.contiguous();
  auto bb = beta.to(torch::kFloat32).contiguous(), gc = g_cumsum.to(torch::kFloat32).contiguous();
  ok(xops_recompute_w_u_fwd(P(kc), P(vc), PT<float>(bb), PT<float>(gc), P(Ac), dtype_code(Ac),
                            P(w), P(u), PT<int32_t>(cu), B, T, N, Hg, H, K, V, stream_of(k)),
     "npu_recompute_w_u_fwd");
  return {w, u};
}

torch::Tensor npu_chunk_fwd_o(const torch::Tensor& q, const torch::Tensor& k,
                              const torch::Tensor& v, const torch::Tensor& h,
                              const torch::Tensor& g_cumsum, float scale, int64_t chunk_size,
                              const std::optional<torch::Tensor>& cu_seqlens) {
  TORCH_CHECK(chunk_size == 64, "chunk_fwd_o only supports chunk_size=64");
  on_cuda(q, "q");
  auto cu = i32(cu_seqlens);
  const int64_t B = q.size(0), T = q.size(1), Hg = q.size(2), K = q.size(3);
  const int64_t H = v.size(2), V = v.size(3);
  const int64_t N = cu.defined() ? cu.numel() - 1 : B;
  auto o = torch::empty_like(v);
  auto qc = q.contiguous(), kc = k.contiguous(), vc = v.contiguous();
  auto hh = h.to(torch::kBFloat16).contiguous();
  auto gc = g_cumsum.defined() ? g_cumsum.to(torch::kFloat32).contiguous() : torch::Tensor();
  ok(xops_chunk_fwd_o(P(qc), P(kc), P(vc), P(hh), PT<float>(gc), P(o), PT<int32_t>(cu), B, T, N,
                      Hg, H, K, V, hh.size(1), scale, stream_of(q)),
     "npu_chunk_fwd_o");
  return o;
}

void rope_inplace(torch::Tensor& x, torch::Tensor& sin, torch::Tensor& cos, uint32_t rope_dim) {
  on_cuda(x, "x");
  TORCH_CHECK(x.dim() == 2 || x.dim() == 3,
              "rope_inplace expects x of shape [bsz, hidden] or [bsz, heads, hidden]");
  TORCH_CHECK(x.stride(-1) == 1, "rope_inplace expects x's last dimension to be contiguous");
  auto x3 = x.dim() == 3 ? x : x.unsqueeze(1);
  const int64_t bsz = x3.size(0), heads = x3.size(1), hidden = x3.size(2);
  TORCH_CHECK(sin.dim() == 2 && cos.dim() == 2 && sin.sizes() == cos.sizes() &&
                  sin.size(0) == bsz && sin.size(1) >= (int64_t)rope_dim,
              "rope_inplace expects sin and cos of shape [bsz, rope_dim]");
  TORCH_CHECK(sin.stride(-1) == 1 && cos.stride(-1) == 1 && sin.stride(0) == cos.stride(0),
              "rope_inplace expects sin and cos rows with the same stride");
  ok(xops_rope_inplace(P(x), P(sin), P(cos), bsz, heads, hidden, rope_dim, x3.stride(0),
                       x3.stride(1), sin.stride(0), dtype_code(x), dtype_code(sin),
                       stream_of(x)),
     "rope_inplace");
}

std::pair<torch::Tensor, torch::Tensor> npu_fused_gdn_gating(torch::Tensor& A_log,
                                                             torch::Tensor& a, torch::Tensor& b,
                                                             torch::Tensor& dt_bias, float beta,
                                                             float threshold) {
  for (auto* t : {&A_log, &a, &b, &dt_bias}) {
    TORCH_CHECK(t->defined(), "gating tensor is not defined");
    TORCH_CHECK(t->is_contiguous(), "gating tensors must be contiguous");
    on_cuda(*t, "gating tensor");
  }
  TORCH_CHECK(A_log.scalar_type() == torch::kFloat32, "A_log must be float32");
  TORCH_CHECK(dt_bias.scalar_type() == torch::kFloat32, "dt_bias must be float32");
  TORCH_CHECK(A_log.dim() == 1, "A_log must be 1D tensor");
  TORCH_CHECK(a.dim() == 2, "a must be 2D tensor (batch, num_heads)");
  TORCH_CHECK(b.dim() == 2, "b must be 2D tensor (batch, num_heads)");
  TORCH_CHECK(dt_bias.dim() == 1, "dt_bias must be 1D tensor");
  const int64_t batch = a.size(0), heads = a.size(1);
  TORCH_CHECK(b.sizes() == a.sizes(), "a and b must have the same shape");
  TORCH_CHECK(A_log.numel() == heads && dt_bias.numel() == heads,
              "A_log and dt_bias must have num_heads elements");
  auto g = torch::empty({1, batch, heads}, a.options().dtype(torch::kFloat32));
  auto beta_output = torch::empty({1, batch, heads}, b.options());
  ok(xops_fused_gdn_gating(PT<float>(A_log), P(a), P(b), PT<float>(dt_bias), PT<float>(g),
                           P(beta_output), batch, heads, dtype_code(a), dtype_code(b), beta,
                           threshold, stream_of(a)),
     "npu_fused_gdn_gating");
  return {g, beta_output};
}

std::pair<torch::Tensor, torch::Tensor> npu_fused_recurrent_gated_delta_rule(
    torch::Tensor& q, torch::Tensor& k, torch::Tensor& v, torch::Tensor& g,
    const std::optional<torch::Tensor>& beta, const std::optional<float>& scale,
    const std::optional<torch::Tensor>& initial_state, bool inplace_final_state,
    const std::optional<torch::Tensor>& cu_seqlens,
    const std::optional<torch::Tensor>& ssm_state_indices,
    const std::optional<torch::Tensor>& num_accepted_tokens, bool use_qk_l2norm_in_kernel) {
  const bool spec = num_accepted_tokens.has_value();
  if (!cu_seqlens.has_value())
    TORCH_CHECK(q.size(0) == 1, "batch size is not 1 when cu_seqlens is not provided");
  TORCH_CHECK(initial_state.has_value(), "initial_state must be provided when inplace_final_state is ",
              inplace_final_state ? "true" : "false");
  if (spec) {
    TORCH_CHECK(cu_seqlens.has_value(), "cu_seqlens must be provided for spec decoding");
    TORCH_CHECK(ssm_state_indices.has_value(),
                "ssm_state_indices must be provided for spec decoding");
  }
  on_cuda(q, "q");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && k.scalar_type() == torch::kBFloat16 &&
                  v.scalar_type() == torch::kBFloat16,
              "npu_fused_recurrent_gated_delta_rule expects q/k/v to be bfloat16");
  const auto& h0 = initial_state.value();
  TORCH_CHECK(h0.scalar_type() == torch::kFloat32, "initial_state must be float32");
  const int64_t B = k.size(0), T = k.size(1), H = k.size(2), K = k.size(3);
  const int64_t HV = v.size(2), V = v.size(3);
  const float sc = scale.has_value() ? scale.value() : 1.0f / std::sqrt((float)K);
  auto cu = i32(cu_seqlens);
  const int64_t N = cu.defined() ? cu.numel() - 1 : B;
  torch::Tensor idx;
  int64_t ss = 0, st = 0;
  if (ssm_state_indices.has_value()) {
    idx = ssm_state_indices->to(torch::kInt32);
    TORCH_CHECK(idx.dim() == 1 || idx.dim() == 2, "ssm_state_indices must be 1D or 2D");
    TORCH_CHECK(idx.size(0) == N, "ssm_state_indices must have one row per sequence");
    ss = idx.stride(0);
    // a [N] table under speculative decoding is addressed like the
    // reference's (token stride 1); otherwise one slot per sequence
    st = idx.dim() == 2 ? idx.stride(1) : (spec ? 1 : 0);
  }
  auto acc = i32(num_accepted_tokens);
  auto gg = g.to(torch::kFloat32).contiguous();
  auto bb = beta.has_value() ? beta->to(torch::kFloat32).contiguous() : torch::Tensor();
  torch::Tensor final_state =
      inplace_final_state ? h0 : torch::empty({N, HV, K, V}, h0.options());
  auto o = torch::empty({B, T, HV, V}, q.options());
  auto qc = q.contiguous(), kc = k.contiguous(), vc = v.contiguous();
  ok(xops_fused_recurrent_gated_delta_rule(
         P(qc), P(kc), P(vc), PT<float>(gg), PT<float>(bb), P(o), PT<float>(h0),
         PT<float>(final_state), PT<int32_t>(cu), PT<int32_t>(idx), ss, st, PT<int32_t>(acc), B,
         T, N, H, HV, K, V, h0.stride(0), final_state.stride(0), sc,
         use_qk_l2norm_in_kernel ? 1 : 0, stream_of(q)),
     "npu_fused_recurrent_gated_delta_rule");
  return {o, final_state};
}

torch::Tensor npu_fused_sigmoid_gating_delta_rule_update(
    torch::Tensor& A_log, torch::Tensor& a, torch::Tensor& dt_bias, torch::Tensor& q,
    torch::Tensor& k, torch::Tensor& v, torch::Tensor& b, torch::Tensor& initial_state_source,
    torch::Tensor& initial_state_indices, torch::Tensor& cu_seqlens,
    const std::optional<float>& scale, bool use_qk_l2norm_in_kernel, float softplus_beta,
    float softplus_threshold) {
  const std::pair<const char*, torch::Tensor*> named[] = {
      {"A_log", &A_log}, {"a", &a}, {"dt_bias", &dt_bias}, {"q", &q}, {"k", &k}, {"v", &v},
      {"b", &b}, {"initial_state_source", &initial_state_source},
      {"initial_state_indices", &initial_state_indices}, {"cu_seqlens", &cu_seqlens}};
  for (const auto& nt : named) {
    TORCH_CHECK(nt.second->defined(), nt.first, " must be defined");
    TORCH_CHECK(nt.second->is_contiguous(), nt.first, " must be contiguous");
    on_cuda(*nt.second, nt.first);
  }
  TORCH_CHECK(q.dim() == 4, "q must be 4D [B, T, H, K]");
  TORCH_CHECK(k.dim() == 4, "k must be 4D [B, T, H, K]");
  TORCH_CHECK(v.dim() == 4, "v must be 4D [B, T, HV, V]");
  TORCH_CHECK(a.dim() == 3, "a must be 3D [B, T, HV]");
  TORCH_CHECK(b.dim() == 3, "b must be 3D [B, T, HV]");
  TORCH_CHECK(A_log.dim() == 1, "A_log must be 1D [HV]");
  TORCH_CHECK(dt_bias.dim() == 1, "dt_bias must be 1D [HV]");
  TORCH_CHECK(initial_state_source.dim() == 4,
              "initial_state_source must be 4D [slots, HV, K, V]");
  TORCH_CHECK(initial_state_indices.dim() == 1, "initial_state_indices must be 1D [N]");
  TORCH_CHECK(cu_seqlens.dim() == 1, "cu_seqlens must be 1D [N + 1]");
  const int64_t B = k.size(0), T = k.size(1), H = k.size(2), K = k.size(3);
  const int64_t HV = v.size(2), V = v.size(3), N = cu_seqlens.numel() - 1;
  TORCH_CHECK(q.sizes() == k.sizes(), "q/k shape mismatch");
  TORCH_CHECK(v.size(0) == B && v.size(1) == T, "v B/T mismatch");
  TORCH_CHECK(a.size(0) == B && a.size(1) == T && a.size(2) == HV, "a shape mismatch");
  TORCH_CHECK(b.sizes() == a.sizes(), "a/b shape mismatch");
  TORCH_CHECK(A_log.numel() == HV, "A_log HV mismatch");
  TORCH_CHECK(dt_bias.numel() == HV, "dt_bias HV mismatch");
  TORCH_CHECK(initial_state_source.size(1) == HV && initial_state_source.size(2) == K &&
                  initial_state_source.size(3) == V,
              "initial_state_source shape mismatch");
  TORCH_CHECK(initial_state_indices.numel() == N,
              "initial_state_indices size must equal cu_seqlens size - 1");
  TORCH_CHECK(HV % H == 0, "HV must be divisible by H");
  TORCH_CHECK(A_log.scalar_type() == torch::kFloat32, "A_log must be float32");
  TORCH_CHECK(dt_bias.scalar_type() == torch::kFloat32, "dt_bias must be float32");
  TORCH_CHECK(initial_state_source.scalar_type() == torch::kFloat32,
              "initial_state_source must be float32");
  TORCH_CHECK(initial_state_indices.scalar_type() == torch::kInt32,
              "initial_state_indices must be int32");
  TORCH_CHECK(cu_seqlens.scalar_type() == torch::kInt32, "cu_seqlens must be int32");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && k.scalar_type() == torch::kBFloat16 &&
                  v.scalar_type() == torch::kBFloat16,
              "npu_fused_sigmoid_gating_delta_rule_update expects q/k/v to be bfloat16");
  TORCH_CHECK(a.scalar_type() == b.scalar_type(), "a and b must have the same dtype");
  const float sc = scale.has_value() ? scale.value() : 1.0f / std::sqrt((float)K);
  auto o = torch::empty({B, T, HV, V}, q.options());
  ok(xops_fused_sigmoid_gating_delta_rule_update(
         PT<float>(A_log), P(a), PT<float>(dt_bias), softplus_beta, softplus_threshold, P(q),
         P(k), P(v), P(b), P(o), PT<float>(initial_state_source),
         PT<int32_t>(initial_state_indices), PT<int32_t>(cu_seqlens), sc, B, T, N, H, HV, K, V,
         dtype_code(a), use_qk_l2norm_in_kernel ? 1 : 0, stream_of(q)),
     "npu_fused_sigmoid_gating_delta_rule_update");
  return o;
}

std::pair<torch::Tensor, torch::Tensor> npu_chunk_gated_delta_rule(
    torch::Tensor& q, torch::Tensor& k, torch::Tensor& v, torch::Tensor& g, torch::Tensor& beta,
    const std::optional<float>& scale, const std::optional<torch::Tensor>& initial_state,
    bool output_final_state, const std::optional<torch::Tensor>& cu_seqlens, bool head_first,
    bool use_qk_l2norm_in_kernel) {
  TORCH_CHECK(!head_first, "chunk_gated_delta_rule torch_api only supports head_first=false.");
  TORCH_CHECK(q.scalar_type() == torch::kBFloat16 && k.scalar_type() == torch::kBFloat16 &&
                  v.scalar_type() == torch::kBFloat16,
              "chunk_gated_delta_rule expects q/k/v to be bfloat16.");
  if (initial_state.has_value())
    TORCH_CHECK(initial_state->scalar_type() == torch::kBFloat16 ||
                    initial_state->scalar_type() == torch::kFloat32,
                "chunk_gated_delta_rule expects initial_state to be bfloat16 or float32, got ",
                initial_state->scalar_type());
  on_cuda(q, "q");
  const int64_t B = q.size(0), T = q.size(1), Hg = q.size(2), K = q.size(3);
  const int64_t H = v.size(2), V = v.size(3);
  TORCH_CHECK(q.sizes() == k.sizes(), "q and k must have the same shape.");
  TORCH_CHECK(H % Hg == 0, "chunk_gated_delta_rule expects num_heads_v to be divisible by "
                           "num_heads_qk, got ", H, " and ", Hg);
  TORCH_CHECK(beta.dim() == 3 && beta.size(0) == B && beta.size(1) == T && beta.size(2) == H,
              "beta must have shape [B, T, H].");
  TORCH_CHECK(g.dim() == 3 && g.size(0) == B && g.size(1) == T && g.size(2) == H,
              "g must have shape [B, T, H].");
  auto cu = i32(cu_seqlens);
  TORCH_CHECK(!cu.defined() || B == 1, "variable-length mode expects batch size B=1");
  const int64_t N = cu.defined() ? cu.numel() - 1 : B;
  const float sc = scale.has_value() ? scale.value() : std::pow((float)K, -0.5f);
  auto h0 = initial_state.has_value() ? initial_state->to(torch::kFloat32).contiguous()
                                      : torch::Tensor();
  auto o = torch::empty({B, T, H, V}, v.options());
  auto ht = output_final_state ? torch::empty({N, H, K, V}, v.options().dtype(torch::kFloat32))
                               : torch::Tensor();
  auto qc = token_rows(q), kc = token_rows(k), vc = token_rows(v);
  auto gg = g.to(torch::kFloat32).contiguous(), bb = beta.to(torch::kFloat32).contiguous();
  const int l2 = use_qk_l2norm_in_kernel ? 1 : 0;
  const int64_t wsb =
      xops_chunk_gated_delta_rule_workspace_size(B, T, N, Hg, H, K, l2, cu.defined() ? 1 : 0);
  auto ws = torch::empty({std::max<int64_t>(wsb, 16)}, q.options().dtype(torch::kUInt8));
  ok(xops_chunk_gated_delta_rule(P(qc), P(kc), P(vc), PT<float>(gg), PT<float>(bb), PT<float>(h0),
                                 P(o), PT<float>(ht), PT<int32_t>(cu), B, T, N, Hg, H, K, V,
                                 qc.stride(1), kc.stride(1), vc.stride(1), sc, l2, P(ws),
                                 ws.numel(), stream_of(q)),
     "npu_chunk_gated_delta_rule");
  return {o, ht};
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> npu_chunk_gated_delta_rule_fwd_h(
    torch::Tensor& k, torch::Tensor& w, torch::Tensor& u, const std::optional<torch::Tensor>& g,
    const std::optional<torch::Tensor>& initial_state, bool output_final_state,
    int64_t chunk_size, bool save_new_value, const std::optional<torch::Tensor>& cu_seqlens,
    const std::optional<torch::Tensor>& chunk_offsets) {
  TORCH_CHECK(chunk_size == 64, "chunk_gated_delta_rule_fwd_h only supports chunk_size=64 in "
                                "the current compiled binary.");
  TORCH_CHECK(k.scalar_type() == torch::kBFloat16, "chunk_gated_delta_rule_fwd_h expects k to be "
                                                   "bfloat16, got ", k.scalar_type());
  TORCH_CHECK(w.scalar_type() == torch::kBFloat16, "chunk_gated_delta_rule_fwd_h expects w to be "
                                                   "bfloat16, got ", w.scalar_type());
  TORCH_CHECK(u.scalar_type() == torch::kBFloat16, "chunk_gated_delta_rule_fwd_h expects u to be "
                                                   "bfloat16, got ", u.scalar_type());
  on_cuda(k, "k");
  const int64_t B = k.size(0), T = k.size(1), Hg = k.size(2), K = k.size(3);
  const int64_t H = u.size(2), V = u.size(3);
  auto cu = i32(cu_seqlens);
  const int64_t N = cu.defined() ? cu.numel() - 1 : B;
  int64_t NT;
  if (cu.defined()) {
    NT = chunk_offsets.has_value()
             ? chunk_offsets->to(torch::kCPU).to(torch::kInt64).reshape({-1})[-1].item<int64_t>()
             : host_total_chunks(cu, B, T, N);
  } else {
    NT = (T + 63) / 64;
  }
  auto h = torch::empty({B, NT, H, K, V}, k.options());
  auto v_new = save_new_value ? torch::empty_like(u) : torch::Tensor();
  auto ht = output_final_state ? torch::empty({N, H, K, V}, k.options().dtype(torch::kFloat32))
                               : torch::Tensor();
  auto h0 = initial_state.has_value() ? initial_state->to(torch::kFloat32).contiguous()
                                      : torch::Tensor();
  auto gc = g.has_value() ? g->to(torch::kFloat32).contiguous() : torch::Tensor();
  auto kc = k.contiguous(), wc = w.contiguous(), uc = u.contiguous();
  ok(xops_chunk_gated_delta_rule_fwd_h(P(kc), P(wc), P(uc), PT<float>(gc), PT<float>(h0), P(h),
                                       P(v_new), PT<float>(ht), PT<int32_t>(cu), B, T, N, Hg, H,
                                       K, V, cu.defined() ? NT : B * NT, stream_of(k)),
     "npu_chunk_gated_delta_rule_fwd_h");
  return std::make_tuple(h, v_new, ht);
}

static std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> layer_norm_impl(
    const torch::Tensor& x, const torch::Tensor& weight, const torch::Tensor& bias, double eps,
    const std::optional<torch::Tensor>& z, int64_t group_size, bool norm_before_gate,
    bool is_rms_norm) {
  on_cuda(x, "x");
  const int64_t n = x.size(-1);
  auto x2 = x.reshape({-1, n});
  if (x2.stride(-1) != 1) x2 = x2.contiguous();
  const int64_t m = x2.size(0);
  const int64_t gs = group_size < 0 ? n : group_size;
  TORCH_CHECK(gs > 0 && n % gs == 0, "layer_norm_fwd: N=", n, " not divisible by group_size=", gs);
  TORCH_CHECK(weight.numel() == n, "layer_norm_fwd: weight must have shape (N,)");
  torch::Tensor z2;
  if (z.has_value()) {
    z2 = z->reshape({-1, n});
    if (z2.stride(-1) != 1) z2 = z2.contiguous();
  }
  auto w = weight.contiguous();
  auto b = bias.defined() ? bias.to(w.scalar_type()).contiguous() : torch::Tensor();
  const int64_t ng = n / gs;
  auto y = torch::empty({m, n}, x.options());
  auto f32 = x.options().dtype(torch::kFloat32);
  auto rstd = torch::empty({ng * m}, f32);
  auto mean = is_rms_norm ? torch::Tensor() : torch::empty({ng * m}, f32);
  ok(xops_layer_norm_fwd(P(x2), P(w), P(b), P(z2), P(y), PT<float>(mean), PT<float>(rstd), m, n, gs,
                         x2.stride(0), z2.defined() ? z2.stride(0) : 0, y.stride(0), (float)eps,
                         norm_before_gate ? 1 : 0, is_rms_norm ? 1 : 0, dtype_code(x),
                         dtype_code(w), stream_of(x)),
     "layer_norm_fwd");
  return {y.view(x.sizes()), mean, rstd};
}

torch::Tensor layer_norm_fwd(torch::Tensor& x, torch::Tensor& weight, torch::Tensor& bias,
                             double eps, const std::optional<torch::Tensor>& z,
                             int64_t group_size, bool norm_before_gate, bool is_rms_norm) {
  return std::get<0>(
      layer_norm_impl(x, weight, bias, eps, z, group_size, norm_before_gate, is_rms_norm));
}

torch::Tensor npu_causal_conv1d_update(
    torch::Tensor& x, torch::Tensor& conv_state, torch::Tensor& weight, bool activation,
    const std::optional<torch::Tensor>& bias, const std::optional<torch::Tensor>& cache_seqlens,
    const std::optional<torch::Tensor>& conv_state_indices,
    const std::optional<torch::Tensor>& num_accepted_tokens,
    const std::optional<torch::Tensor>& query_start_loc, int32_t max_query_len,
    const std::optional<torch::Tensor>& intermediate_conv_window, int32_t pad_slot_id,
    bool validate_data) {
  (void)max_query_len;
  (void)intermediate_conv_window;
  (void)validate_data;
  TORCH_CHECK(!query_start_loc.has_value(),
              "Current op does not support non-empty values for query_start_loc.");
  TORCH_CHECK(!cache_seqlens.has_value() && !num_accepted_tokens.has_value(),
              "currently causal_conv1d_update don't support input cache_len and mtp scenerios.");
  on_cuda(x, "x");
  const bool squeeze = x.dim() == 2;
  auto x3 = squeeze ? x.unsqueeze(-1) : x;
  TORCH_CHECK(x3.dim() == 3 && conv_state.dim() == 3 && weight.dim() == 2,
              "causal_conv1d_update: bad tensor ranks");
  const int64_t batch = x3.size(0), dim = x3.size(1), seqlen = x3.size(2), width = weight.size(1);
  TORCH_CHECK(conv_state.is_contiguous(), "causal_conv1d_update: conv_state must be contiguous");
  auto w = weight.contiguous();
  auto b = bias.has_value() ? bias->to(x.scalar_type()).contiguous() : torch::Tensor();
  auto idx = i32(conv_state_indices);
  auto out = torch::empty({batch, dim, seqlen}, x.options());
  ok(xops_causal_conv1d_update(P(x3), P(conv_state), P(w), P(b), PT<int32_t>(idx), P(out), batch,
                               dim, seqlen, width, conv_state.size(2), conv_state.size(0),
                               x3.stride(0), x3.stride(1), x3.stride(2), activation ? 1 : 0,
                               pad_slot_id, dtype_code(x), stream_of(x)),
     "npu_causal_conv1d_update");
  return squeeze ? out.squeeze(-1) : out;
}

torch::Tensor npu_causal_conv1d_update_v2(
    torch::Tensor& x, torch::Tensor& conv_state, torch::Tensor& weight, bool activation,
    const std::optional<torch::Tensor>& bias,
    const std::optional<torch::Tensor>& conv_state_indices,
    const std::optional<torch::Tensor>& query_start_loc, int32_t max_query_len,
    int32_t pad_slot_id, const std::optional<torch::Tensor>& block_idx_last_scheduled_token,
    const std::optional<torch::Tensor>& initial_state_idx, bool validate_data,
    const std::optional<torch::Tensor>& num_accepted_tokens) {
  (void)max_query_len;
  (void)validate_data;
  TORCH_CHECK(weight.dim() == 2, "causal_conv1d_update_v2 expects weight shape [dim, width].");
  TORCH_CHECK(block_idx_last_scheduled_token.has_value() == initial_state_idx.has_value(),
              "causal_conv1d_update_v2 expects both APC tensors or neither.");
  TORCH_CHECK(conv_state.dim() == 3, "causal_conv1d_update_v2 expects conv_state shape "
                                     "[num_cache_lines, dim, state_len].");
  on_cuda(x, "x");
  const int64_t width = weight.size(1);
  TORCH_CHECK(width >= 2 && width <= 6, "causal_conv1d_update_v2 expects width in [2, 6], got ",
              width);
  torch::Tensor xv, qsl;
  int64_t batch;
  bool unsq = false;
  int64_t seqlen = 0;
  if (query_start_loc.has_value()) {
    TORCH_CHECK(x.dim() == 2, "causal_conv1d_update_v2 expects x to be 2D [num_tokens, dim] "
                              "when query_start_loc is provided.");
    qsl = query_start_loc->to(torch::kInt32).contiguous();
    xv = x.contiguous();
    batch = qsl.numel() - 1;
  } else {
    unsq = x.dim() == 2;
    auto xw = unsq ? x.unsqueeze(-1) : x;
    TORCH_CHECK(xw.dim() == 3, "causal_conv1d_update_v2 expects x to have shape [B, D] or [B, D, T]");
    batch = xw.size(0);
    seqlen = xw.size(2);
    xv = xw.transpose(1, 2).contiguous().view({batch * seqlen, xw.size(1)});
    qsl = torch::arange(0, (batch + 1) * seqlen, seqlen, x.options().dtype(torch::kInt32));
  }
  const int64_t dim = xv.size(1);
  TORCH_CHECK(weight.size(0) == dim, "weight dim mismatch. Expected ", dim, ", got ", weight.size(0));
  TORCH_CHECK(conv_state.size(1) == dim, "conv_state dim mismatch. Expected ", dim, ", got ",
              conv_state.size(1));
  TORCH_CHECK(conv_state.size(2) >= width - 1,
              "causal_conv1d_update_v2: conv_state must hold at least width - 1 history columns");
  auto b = bias.has_value() ? bias->to(xv.scalar_type()).contiguous() : torch::Tensor();
  auto idx = i32(conv_state_indices);
  auto w = weight.contiguous();
  const bool slots = num_accepted_tokens.has_value() || initial_state_idx.has_value() ||
                     (idx.defined() && idx.dim() == 2 && idx.size(1) > 1) ||
                     conv_state.size(2) != width - 1;
  if (slots) {  // speculative decoding / prefix-cache block tables
    if (idx.defined())
      TORCH_CHECK((idx.dim() == 1 || idx.dim() == 2) && idx.size(0) == batch,
                  "conv_state_indices batch mismatch. Expected ", batch, ", got ", idx.size(0));
    auto acc = i32(num_accepted_tokens), ini = i32(initial_state_idx),
         last = i32(block_idx_last_scheduled_token);
    for (const auto* t : {&acc, &ini, &last})
      TORCH_CHECK(!t->defined() || t->numel() == batch,
                  "slot tables must have one entry per sequence");
    auto out = torch::empty_like(xv);
    ok(xops_causal_conv1d_update_v2_slots(
           P(xv), P(conv_state), P(w), P(b), PT<int32_t>(idx), idx.defined() ? idx.stride(0) : 0,
           PT<int32_t>(acc), PT<int32_t>(ini), PT<int32_t>(last), PT<int32_t>(qsl), P(out),
           batch, dim, width, conv_state.size(2), conv_state.size(0), activation ? 1 : 0,
           pad_slot_id, dtype_code(xv), stream_of(x)),
       "npu_causal_conv1d_update_v2");
    if (query_start_loc.has_value()) return out;
    auto o3 = out.view({batch, seqlen, dim}).transpose(1, 2);
    return unsq ? o3.squeeze(-1) : o3;
  }
  if (idx.defined() && idx.dim() == 2) idx = idx.select(1, 0).contiguous();
  auto out = torch::empty_like(xv);
  ok(xops_causal_conv1d_varlen(P(xv), P(conv_state), P(w), P(b), PT<int32_t>(qsl),
                               PT<int32_t>(idx), P(out), batch, xv.size(0), dim, width,
                               conv_state.size(0), activation ? 1 : 0, pad_slot_id,
                               dtype_code(xv), stream_of(x)),
     "npu_causal_conv1d_update_v2");
  if (query_start_loc.has_value()) return out;
  auto o3 = out.view({batch, seqlen, dim}).transpose(1, 2);
  return unsq ? o3.squeeze(-1) : o3;
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor, torch::Tensor>
npu_fused_qkvzba_split_reshape_cat(torch::Tensor& mixed_qkvz, torch::Tensor& mixed_ba,
                                   int32_t num_heads_qk, int32_t num_heads_v, int32_t head_qk,
                                   int32_t head_v) {
  on_cuda(mixed_qkvz, "mixed_qkvz");
  on_cuda(mixed_ba, "mixed_ba");
  TORCH_CHECK(num_heads_qk > 0, "num_heads_qk must be positive");
  const int64_t rows = mixed_qkvz.size(0);
  const int32_t r = num_heads_v / num_heads_qk;
  TORCH_CHECK(r >= 1 && r <= 4,
              "npu_fused_qkvzba_split_reshape_cat only supports v_heads_per_qk in [1, 4], but got ",
              r, " for num_heads_qk=", num_heads_qk, " num_heads_v=", num_heads_v);
  auto qkvz = mixed_qkvz.contiguous();
  auto ba = mixed_ba.contiguous();
  TORCH_CHECK(qkvz.numel() == rows * num_heads_qk * (2 * head_qk + 2 * r * head_v) &&
                  ba.numel() == rows * num_heads_qk * 2 * r,
              "npu_fused_qkvzba_split_reshape_cat: projection widths do not match the head counts");
  auto qkv = torch::empty({rows, (int64_t)2 * num_heads_qk * head_qk + (int64_t)num_heads_v * head_v},
                          qkvz.options());
  auto z = torch::empty({rows, (int64_t)num_heads_v, (int64_t)head_v}, qkvz.options());
  auto b = torch::empty({rows, (int64_t)num_heads_v}, ba.options());
  auto a = torch::empty({rows, (int64_t)num_heads_v}, ba.options());
  ok(xops_fused_qkvzba_split_reshape_cat(P(qkvz), P(ba), P(qkv), P(z), P(b), P(a), rows,
                                         num_heads_qk, num_heads_v, head_qk, head_v,
                                         dtype_code(qkvz), dtype_code(ba), stream_of(qkvz)),
     "npu_fused_qkvzba_split_reshape_cat");
  return {qkv, z, b, a};
}

std::tuple<torch::Tensor, torch::Tensor, torch::Tensor> npu_split_rmsnorm_rope(
    torch::Tensor& input, torch::Tensor& sin, torch::Tensor& cos, torch::Tensor& q_weight,
    torch::Tensor& k_weight, int64_t q_hidden_size, int64_t kv_hidden_size, int64_t head_dim,
    double eps, const std::optional<torch::Tensor>& q_bias,
    const std::optional<torch::Tensor>& k_bias, bool bias) {
  TORCH_CHECK(input.dim() == 2, "split_rmsnorm_rope input must be a 2D tensor");
  TORCH_CHECK(sin.dim() == 2 && cos.dim() == 2, "split_rmsnorm_rope sin and cos must be 2D tensors");
  TORCH_CHECK(q_weight.dim() == 1 && k_weight.dim() == 1,
              "split_rmsnorm_rope q_weight and k_weight must be 1D tensors");
  TORCH_CHECK(head_dim > 0 && (head_dim & (head_dim - 1)) == 0,
              "split_rmsnorm_rope head_dim must be a power of two");
  TORCH_CHECK(kv_hidden_size > 0 && q_hidden_size % kv_hidden_size == 0,
              "split_rmsnorm_rope q_hidden_size must be divisible by kv_hidden_size");
  TORCH_CHECK(kv_hidden_size % head_dim == 0,
              "split_rmsnorm_rope kv_hidden_size must be divisible by head_dim");
  TORCH_CHECK(input.size(1) == q_hidden_size + 2 * kv_hidden_size,
              "split_rmsnorm_rope input hidden size mismatch");
  const int64_t rd = sin.size(1);
  TORCH_CHECK(sin.size(0) == input.size(0) && cos.size(0) == input.size(0) && cos.size(1) == rd &&
                  rd > 0 && rd <= head_dim,
              "split_rmsnorm_rope sin/cos shape mismatch");
  TORCH_CHECK(q_weight.size(0) == head_dim && k_weight.size(0) == head_dim,
              "split_rmsnorm_rope q/k weight shape mismatch");
  on_cuda(input, "input");
  const int64_t t = input.size(0);
  auto inp = input.contiguous(), s = sin.contiguous(), c = cos.contiguous();
  auto qw = q_weight.contiguous(), kw = k_weight.contiguous();
  const bool use_b = bias && q_bias.has_value() && k_bias.has_value();
  auto qb = use_b ? q_bias->to(qw.scalar_type()).contiguous() : torch::Tensor();
  auto kb = use_b ? k_bias->to(qw.scalar_type()).contiguous() : torch::Tensor();
  auto q = torch::empty({t, q_hidden_size}, input.options());
  auto k = torch::empty({t, kv_hidden_size}, input.options());
  auto v = torch::empty({t, kv_hidden_size}, input.options());
  ok(xops_split_rmsnorm_rope(P(inp), P(s), P(c), P(q), P(k), P(v), P(qw), P(qb), P(kw), P(kb), t,
                             q_hidden_size, kv_hidden_size, head_dim, rd, (float)eps,
                             dtype_code(input), dtype_code(qw), dtype_code(s), stream_of(input)),
     "npu_split_rmsnorm_rope");
  return std::make_tuple(q, k, v);
}

}  // namespace xllm::kernel::npu

namespace npu_ops {

void npu_gemma_rms_norm(const torch::Tensor& x, const torch::Tensor& gamma, double epsilon,
                        torch::Tensor& rstdOut, torch::Tensor& yOut) {
  on_cuda(x, "x");
  const int64_t gd = gamma.dim(), xd = x.dim();
  TORCH_CHECK(gd >= 1 && xd >= gd, "gemma_rms_norm: gamma must match the trailing dims of x");
  std::vector<int64_t> shape;
  if (xd > gd) {
    for (int64_t i = 0; i < xd - gd; ++i) shape.push_back(x.size(i));
    for (int64_t i = 0; i < gd; ++i) shape.push_back(1);
  } else {
    shape.assign(xd, 1);
  }
  auto xc = x.contiguous(), gc = gamma.contiguous();
  const int64_t n = gamma.numel();
  auto y = torch::empty_like(xc);
  auto rstd = torch::empty(shape, x.options().dtype(torch::kFloat32));
  ok(xops_gemma_rms_norm(P(xc), P(gc), P(y), PT<float>(rstd), n ? xc.numel() / n : 0, n,
                         (float)epsilon, dtype_code(x), dtype_code(gc), stream_of(x)),
     "npu_gemma_rms_norm");
  yOut = y;
  rstdOut = rstd;
}

torch::Tensor layer_norm_fwd(const torch::Tensor& x, const torch::Tensor& weight,
                             const c10::optional<torch::Tensor>& bias, double eps,
                             const c10::optional<torch::Tensor>& z, int64_t group_size,
                             bool norm_before_gate, bool is_rms_norm) {
  return std::get<0>(xllm::kernel::npu::layer_norm_impl(
      x, weight, bias.has_value() ? bias.value() : torch::Tensor(), eps, z, group_size,
      norm_before_gate, is_rms_norm));
}

}  // namespace npu_ops
