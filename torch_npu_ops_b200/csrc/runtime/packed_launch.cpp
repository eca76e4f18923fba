// Decoders from the reference's packed launch buffers to the C ABI
// (see packed_launch.h).  Reference paths are relative to the reference
// project root; each decoder cites the call site whose packing it reads.
#include "packed_launch.h"

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>

#include "xops_b200.h"

namespace xllm::kernel::npu {
namespace {

// Reads values back in the order and alignment ArgsBuilder::add wrote them
// (each value padded to its natural alignment).
class ArgReader {
 public:
  ArgReader(const void* p, size_t n) : p_(static_cast<const unsigned char*>(p)), n_(n) {}

  template <typename T>
  T get() {
    const size_t a = alignof(T);
    off_ = (off_ + a - 1) / a * a;
    T v{};
    if (off_ + sizeof(T) > n_) {
      ok_ = false;
      return v;
    }
    std::memcpy(&v, p_ + off_, sizeof(T));
    off_ += sizeof(T);
    return v;
  }
  const void* ptr() { return get<void*>(); }
  // the three grid dimensions the reference appends, then the end of the buffer
  bool finish() {
    get<int32_t>();
    get<int32_t>();
    get<int32_t>();
    return ok_ && off_ == n_;
  }
  bool ok() const { return ok_; }

 private:
  const unsigned char* p_;
  size_t n_;
  size_t off_ = 0;
  bool ok_ = true;
};

bool starts_with(const std::string& s, const char* prefix) {
  return s.compare(0, std::strlen(prefix), prefix) == 0;
}
bool has_token(const std::string& s, const char* tok) { return s.find(tok) != std::string::npos; }

struct Launch {
  int32_t gx, gy, gz;
  void* stream;
};

// layer_norm_fwd_kernel_fast{,_rms}{,_bf16}{,_z}{,_bias,_nobias}{,_nomask}
// (triton_npu/torch_api/npu_triton_layernorm_fwd.cpp:112-293).  The name gives
// RMS vs LayerNorm, bf16 vs fp32 x, gate z and bias; gridY = ngroups, so
// N = gridY * group_size.  Assumed constants: weight/bias in x's dtype and
// NORM_BEFORE_GATE = true (the reference's fast path ignores the
// norm_before_gate argument, so its binaries carry one value: the GDN layer's).
int32_t layer_norm_fast(const std::string& name, ArgReader& r, const Launch& l) {
  const std::string tail = name.substr(std::strlen("layer_norm_fwd_kernel_fast"));
  const bool rms = has_token(tail, "_rms"), bf16 = has_token(tail, "_bf16"),
             has_z = has_token(tail, "_z");
  // LayerNorm variants always pack a bias slot (it may be null); RMS variants
  // name it
  const bool bias_slot = rms ? has_token(tail, "_bias") : true;
  const void* x = r.ptr();
  void* y = const_cast<void*>(r.ptr());
  const void* w = r.ptr();
  const void* b = bias_slot ? r.ptr() : nullptr;
  const void* z = has_z ? r.ptr() : nullptr;
  float* mean = rms ? nullptr : static_cast<float*>(const_cast<void*>(r.ptr()));
  float* rstd = static_cast<float*>(const_cast<void*>(r.ptr()));
  const int32_t sx = r.get<int32_t>(), sy = r.get<int32_t>(), sz = r.get<int32_t>();
  const int32_t M = r.get<int32_t>(), G = r.get<int32_t>();
  const float eps = r.get<float>();
  (void)r.get<int32_t>();  // N_CORES (the reference's grid-stride width)
  if (!r.finish()) return kPackedBadBuffer;
  const int dt = bf16 ? XOPS_BF16 : XOPS_F32;
  return xops_layer_norm_fwd(x, w, b, z, y, mean, rstd, M, (int64_t)l.gy * G, G, sx, sz, sy, eps,
                             1, rms ? 1 : 0, dt, dt, l.stream);
}

// layer_norm_fwd_kernel, the reference's group_size > 128 fallback
// (npu_triton_layernorm_fwd.cpp:295-333): RMSNorm without bias, optional z.
// Assumed constants: bf16 x and weight, NORM_BEFORE_GATE = true.
int32_t layer_norm_fallback(ArgReader& r, const Launch& l) {
  const void* x = r.ptr();
  void* y = const_cast<void*>(r.ptr());
  const void* w = r.ptr();
  const void* z = r.ptr();
  float* rstd = static_cast<float*>(const_cast<void*>(r.ptr()));
  const int32_t sx = r.get<int32_t>(), sy = r.get<int32_t>(), sz = r.get<int32_t>();
  const int32_t M = r.get<int32_t>(), G = r.get<int32_t>();
  const float eps = r.get<float>();
  if (!r.finish()) return kPackedBadBuffer;
  return xops_layer_norm_fwd(x, w, nullptr, z, y, nullptr, rstd, M, (int64_t)l.gy * G, G, sx, sz,
                             sy, eps, 1, 1, XOPS_BF16, XOPS_BF16, l.stream);
}

// l2norm_fwd_kernel2_loop (npu_triton_l2norm.cpp:88-101): x, y, eps, rows,
// cols and the reference's row / column chunk counts.  Assumed: bf16 (the
// dtype of the reference's test, test_l2norm.py:109).
int32_t l2norm(ArgReader& r, const Launch& l) {
  const void* x = r.ptr();
  void* y = const_cast<void*>(r.ptr());
  const float eps = r.get<float>();
  const int32_t rows = r.get<int32_t>(), cols = r.get<int32_t>();
  (void)r.get<int32_t>();
  (void)r.get<int32_t>();
  if (!r.finish()) return kPackedBadBuffer;
  return xops_l2norm_last_dim(x, y, rows, cols, eps, XOPS_BF16, l.stream);
}

// split_rmsnorm_rope_kernel_bias{0,1}_eps{E}_hd{D}_qh{Q}_kvh{KV}
// (npu_triton_split_rmsnorm_rope.cpp:39-48 for the name, :123-135 for the
// arguments).  E is std::to_string(eps) without '.', 'e' and '-', i.e. eps
// in millionths.  Assumed: bf16 input, weights and sin/cos (the dtype of the
// reference's test, test_split_rmsnorm_rope.py:364), full-width rotation.
int32_t split_rmsnorm_rope(const std::string& name, ArgReader& r, const Launch& l) {
  long long bias = 0, eps_m = 0, hd = 0, qh = 0, kvh = 0;
  {
    const std::string t = name.substr(std::strlen("split_rmsnorm_rope_kernel"));
    char eps_s[64] = {0};
    if (std::sscanf(t.c_str(), "_bias%lld_eps%63[0-9]_hd%lld_qh%lld_kvh%lld", &bias, eps_s, &hd,
                    &qh, &kvh) != 5)
      return kPackedBadBuffer;
    eps_m = std::atoll(eps_s);
  }
  const void* in = r.ptr();
  const void* sn = r.ptr();
  const void* cs = r.ptr();
  void* q = const_cast<void*>(r.ptr());
  void* k = const_cast<void*>(r.ptr());
  void* v = const_cast<void*>(r.ptr());
  const void* qw = r.ptr();
  const void* qb = r.ptr();
  const void* kw = r.ptr();
  const void* kb = r.ptr();
  const int32_t T = r.get<int32_t>();
  if (!r.finish()) return kPackedBadBuffer;
  if (!bias) qb = kb = nullptr;
  return xops_split_rmsnorm_rope(in, sn, cs, q, k, v, qw, qb, kw, kb, T, qh, kvh, hd, hd,
                                 (float)((double)eps_m / 1e6), XOPS_BF16, XOPS_BF16, XOPS_BF16,
                                 l.stream);
}

// fused_gdn_gating_decode_kernel (npu_triton_fused_gdn_gating.cpp:84-90):
// g, beta_out, A_log, a, b, dt_bias, num_heads; rows = gridX.  Assumed: bf16
// a and b (the reference test's default dtype, test_fused_gdn_gating.py:52)
// and the softplus beta 1 / threshold 20 of the reference wrapper's callers.
int32_t gdn_gating(ArgReader& r, const Launch& l) {
  float* g = static_cast<float*>(const_cast<void*>(r.ptr()));
  void* beta = const_cast<void*>(r.ptr());
  const float* A_log = static_cast<const float*>(r.ptr());
  const void* a = r.ptr();
  const void* b = r.ptr();
  const float* dt_bias = static_cast<const float*>(r.ptr());
  const int32_t heads = r.get<int32_t>();
  if (!r.finish()) return kPackedBadBuffer;
  return xops_fused_gdn_gating(A_log, a, b, dt_bias, g, beta, l.gx, heads, XOPS_BF16, XOPS_BF16,
                               1.f, 20.f, l.stream);
}

// _causal_conv1d_update_qwen_decode_kernel
// (npu_triton_causal_conv1d_update.cpp:61-101): width 4, state_len 3, one
// token, no bias, SiLU, contiguous x [batch, dim, 1], state [lines, dim, 3].
// Assumed: bf16.  The number of state lines is not packed: without a slot
// table the rows use lines 0..batch-1; with one, every entry must name a line
// of conv_state (or be pad_slot_id), as the reference kernel requires.
int32_t conv_qwen_decode(ArgReader& r, const Launch& l) {
  const void* x = r.ptr();
  void* st = const_cast<void*>(r.ptr());
  const void* w = r.ptr();
  const int32_t* idx = static_cast<const int32_t*>(r.ptr());
  void* out = const_cast<void*>(r.ptr());
  const int32_t pad = r.get<int32_t>(), batch = r.get<int32_t>(), dim = r.get<int32_t>();
  if (!r.finish()) return kPackedBadBuffer;
  return xops_causal_conv1d_update(x, st, w, nullptr, idx, out, batch, dim, 1, 4, 3,
                                   /*num_cache_lines=*/batch, dim, 1, 1, 1, pad, XOPS_BF16,
                                   l.stream);
}

// fused_recurrent_gated_delta_rule_fwd_kernel
// (npu_triton_recurrent_gated_delta_rule.cpp:216-246); grid (1, NV, N * HV)
// with BV = 64.  Assumed: bf16 q/k/v/o, K = V = 64 * gridY, q/k L2
// normalised in the kernel (USE_QK_L2NORM_IN_KERNEL of the GDN layer), one
// slot per sequence in ssm_state_indices.  In place when the final-state
// pointer equals the initial-state pointer.
int32_t recurrent(ArgReader& r, const Launch& l) {
  const void* q = r.ptr();
  const void* k = r.ptr();
  const void* v = r.ptr();
  const float* g = static_cast<const float*>(r.ptr());
  const float* beta = static_cast<const float*>(r.ptr());
  void* o = const_cast<void*>(r.ptr());
  const float* h0 = static_cast<const float*>(r.ptr());
  float* ht = static_cast<float*>(const_cast<void*>(r.ptr()));
  const int32_t* cu = static_cast<const int32_t*>(r.ptr());
  const int32_t* idx = static_cast<const int32_t*>(r.ptr());
  const float scale = r.get<float>();
  const int64_t N = r.get<int64_t>(), T = r.get<int64_t>(), H = r.get<int64_t>(),
                HV = r.get<int64_t>(), s0 = r.get<int64_t>(), s1 = r.get<int64_t>();
  if (!r.finish()) return kPackedBadBuffer;
  const int64_t KV = 64 * (int64_t)l.gy;
  const int64_t B = cu ? 1 : N;
  return xops_fused_recurrent_gated_delta_rule(q, k, v, g, beta, o, h0, ht, cu, idx, 1, 0, nullptr,
                                               B, T, N, H, HV, KV, KV, s0, s1, scale, 1, l.stream);
}

enum class Kind { None, LnFast, LnFallback, L2, SplitRope, Gating, ConvQwen, Recurrent };

Kind kind_of(const std::string& n) {
  if (starts_with(n, "layer_norm_fwd_kernel_fast")) return Kind::LnFast;
  if (n == "layer_norm_fwd_kernel") return Kind::LnFallback;
  if (n == "l2norm_fwd_kernel2_loop") return Kind::L2;
  if (starts_with(n, "split_rmsnorm_rope_kernel_bias")) return Kind::SplitRope;
  if (n == "fused_gdn_gating_decode_kernel") return Kind::Gating;
  if (n == "_causal_conv1d_update_qwen_decode_kernel") return Kind::ConvQwen;
  if (n == "fused_recurrent_gated_delta_rule_fwd_kernel") return Kind::Recurrent;
  return Kind::None;
}

}  // namespace

bool has_packed_decoder(const std::string& kernel_name) {
  return kind_of(kernel_name) != Kind::None;
}

int32_t launch_packed(const std::string& kernel_name, const void* args, size_t size,
                      int32_t grid_x, int32_t grid_y, int32_t grid_z, void* stream,
                      std::string* error) {
  const Kind kind = kind_of(kernel_name);
  if (kind == Kind::None) {
    if (error)
      *error = "no decoder for the packed arguments of '" + kernel_name +
               "' (its reference binary keeps sizes or dtypes as compile-time constants); call "
               "the torch API function or the C ABI entry point instead";
    return kPackedNoDecoder;
  }
  ArgReader r(args, size);
  // the reference's prefix: ffts control address, lock, workspace
  r.ptr();
  r.ptr();
  r.ptr();
  const Launch l{grid_x, grid_y, grid_z, stream};
  int32_t rc = kPackedBadBuffer;
  switch (kind) {
    case Kind::LnFast: rc = layer_norm_fast(kernel_name, r, l); break;
    case Kind::LnFallback: rc = layer_norm_fallback(r, l); break;
    case Kind::L2: rc = l2norm(r, l); break;
    case Kind::SplitRope: rc = split_rmsnorm_rope(kernel_name, r, l); break;
    case Kind::Gating: rc = gdn_gating(r, l); break;
    case Kind::ConvQwen: rc = conv_qwen_decode(r, l); break;
    case Kind::Recurrent: rc = recurrent(r, l); break;
    case Kind::None: break;
  }
  if (error) {
    if (rc == kPackedBadBuffer)
      *error = "the packed arguments do not match the layout of '" + kernel_name + "'";
    else if (rc > 0)
      *error = xops_last_error();
    else
      error->clear();
  }
  return rc;
}

}  // namespace xllm::kernel::npu
