// Python module of the C++ torch API.  The first two functions keep the
// schemas of the reference's pybind module npu_python_extension_lib
// (npu_python_extension/op_register.cpp:52-63); the rest expose the
// xllm::kernel::npu operators and the runtime registry.
#include <ATen/cuda/CUDAContext.h>
#include <torch/extension.h>

#include "../runtime/kernel_registry.h"
#include "ascendc_ops_api.h"
#include "operation_factory.h"
#include "triton_ops_api.h"

namespace py = pybind11;
namespace xn = xllm::kernel::npu;

namespace {

// The reference runtime's launch path, driven from Python for tests: packs
// `args` (pairs of kind and value; kinds "ptr", "i32", "i64", "f32") with
// ArgsBuilder in order, exactly as a reference call site's build_args lambda
// does, and calls OperationBase::execute of the op bound to `kernel_name`.
std::tuple<int64_t, std::string, int64_t> py_runtime_execute(const std::string& kernel_name,
                                                             int32_t gx, int32_t gy, int32_t gz,
                                                             const py::list& args,
                                                             uintptr_t stream) {
  auto& op = xn::OperationFactory::instance().by_kernel_name(kernel_name);
  const int32_t rc = op.execute(reinterpret_cast<void*>(stream), gx, gy, gz,
                                [&](xn::ArgsBuilder& ab) {
    for (const auto& item : args) {
      auto t = item.cast<py::tuple>();
      const std::string kind = t[0].cast<std::string>();
      if (kind == "ptr")
        ab.add<void*>(t[1].is_none() ? nullptr
                                     : reinterpret_cast<void*>(t[1].cast<uintptr_t>()));
      else if (kind == "i32")
        ab.add<int32_t>(t[1].cast<int32_t>());
      else if (kind == "i64")
        ab.add<int64_t>(t[1].cast<int64_t>());
      else if (kind == "f32")
        ab.add<float>(t[1].cast<float>());
      else
        throw std::invalid_argument("argument kind must be ptr, i32, i64 or f32");
    }
  });
  return std::make_tuple((int64_t)rc, op.last_error(), (int64_t)op.last_args_size());
}

// The reference's group_size > 128 layer_norm_fwd launch
// (triton_npu/torch_api/npu_triton_layernorm_fwd.cpp:295-333) written as a
// caller of the reference runtime writes it: OperationFactory's
// layer_norm_fwd() op, execute() with the same argument list, on the current
// stream.  Returns (y, rstd).
std::tuple<torch::Tensor, torch::Tensor> py_runtime_layer_norm_fwd(const torch::Tensor& x,
                                                                   const torch::Tensor& weight,
                                                                   const c10::optional<torch::Tensor>& z,
                                                                   double eps, int64_t group_size) {
  TORCH_CHECK(x.dim() == 2 && x.scalar_type() == torch::kBFloat16, "x must be [M, N] bf16");
  const int64_t M = x.size(0), N = x.size(1), ngroups = N / group_size;
  auto y = torch::empty_like(x);
  auto rstd = torch::empty({ngroups * M}, x.options().dtype(torch::kFloat32));
  void* zp = z.has_value() ? z->data_ptr() : nullptr;
  const int32_t sx = (int32_t)x.stride(0), sy = (int32_t)y.stride(0),
                sz = z.has_value() ? (int32_t)z->stride(0) : 0;
  const int32_t gridX = (int32_t)std::max<int64_t>(1, std::min<int64_t>(40, M));
  auto& op = xn::OperationFactory::instance().layer_norm_fwd();
  const int32_t rc = op.execute(at::cuda::getCurrentCUDAStream().stream(), gridX,
                                (int32_t)ngroups, 1, [&](xn::ArgsBuilder& ab) {
    ab.constructArgs(x.data_ptr(), y.data_ptr(), weight.data_ptr(), zp, rstd.data_ptr(), sx, sy,
                     sz, static_cast<int32_t>(M), static_cast<int32_t>(group_size),
                     static_cast<float>(eps));
  });
  TORCH_CHECK(rc == 0, "OperationBase::execute failed (", rc, "): ", op.last_error());
  return std::make_tuple(y, rstd);
}

std::tuple<torch::Tensor, torch::Tensor> py_gemma_rms_norm(const torch::Tensor& x,
                                                           const torch::Tensor& gamma,
                                                           double epsilon) {
  torch::Tensor rstd, y;
  npu_ops::npu_gemma_rms_norm(x, gamma, epsilon, rstd, y);
  return std::make_tuple(rstd, y);
}

torch::Tensor py_layer_norm_fwd(const torch::Tensor& x, const torch::Tensor& weight,
                                const c10::optional<torch::Tensor>& bias, double eps,
                                const c10::optional<torch::Tensor>& z, int64_t group_size,
                                bool norm_before_gate, bool is_rms_norm) {
  return npu_ops::layer_norm_fwd(x, weight, bias, eps, z, group_size, norm_before_gate,
                                 is_rms_norm);
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("gemma_rms_norm", &py_gemma_rms_norm, "Gemma RMSNorm -> (rstd, y)");
  m.def("layer_norm_fwd", &py_layer_norm_fwd, "grouped LayerNorm/RMSNorm with SiLU gate",
        py::arg("x"), py::arg("weight"), py::arg("bias"), py::arg("eps"), py::arg("z"),
        py::arg("group_size"), py::arg("norm_before_gate"), py::arg("is_rms_norm"));
  m.def("npu_l2norm_last_dim",
        [](torch::Tensor x, double eps) { return xn::npu_l2norm_last_dim(x, eps); },
        py::arg("x"), py::arg("eps") = 1e-6);
  m.def("npu_split_rmsnorm_rope",
        [](torch::Tensor input, torch::Tensor sin, torch::Tensor cos, torch::Tensor qw,
           torch::Tensor kw, int64_t qh, int64_t kvh, int64_t hd, double eps,
           std::optional<torch::Tensor> qb, std::optional<torch::Tensor> kb, bool bias) {
          return xn::npu_split_rmsnorm_rope(input, sin, cos, qw, kw, qh, kvh, hd, eps, qb, kb,
                                            bias);
        },
        py::arg("input"), py::arg("sin"), py::arg("cos"), py::arg("q_weight"),
        py::arg("k_weight"), py::arg("q_hidden_size"), py::arg("kv_hidden_size"),
        py::arg("head_dim"), py::arg("eps"), py::arg("q_bias") = py::none(),
        py::arg("k_bias") = py::none(), py::arg("bias") = false);
  m.def("npu_causal_conv1d_update",
        [](torch::Tensor x, torch::Tensor st, torch::Tensor w, bool act,
           std::optional<torch::Tensor> b, std::optional<torch::Tensor> idx, int32_t pad) {
          return xn::npu_causal_conv1d_update(x, st, w, act, b, std::nullopt, idx, std::nullopt,
                                              std::nullopt, -1, std::nullopt, pad, false);
        },
        py::arg("x"), py::arg("conv_state"), py::arg("weight"), py::arg("activation") = true,
        py::arg("bias") = py::none(), py::arg("conv_state_indices") = py::none(),
        py::arg("pad_slot_id") = -1);
  m.def("npu_causal_conv1d_update_v2",
        [](torch::Tensor x, torch::Tensor st, torch::Tensor w, bool act,
           std::optional<torch::Tensor> b, std::optional<torch::Tensor> idx,
           std::optional<torch::Tensor> qsl, int32_t max_q, int32_t pad,
           std::optional<torch::Tensor> last, std::optional<torch::Tensor> init, bool validate,
           std::optional<torch::Tensor> acc) {
          return xn::npu_causal_conv1d_update_v2(x, st, w, act, b, idx, qsl, max_q, pad, last,
                                                 init, validate, acc);
        },
        py::arg("x"), py::arg("conv_state"), py::arg("weight"), py::arg("activation") = true,
        py::arg("bias") = py::none(), py::arg("conv_state_indices") = py::none(),
        py::arg("query_start_loc") = py::none(), py::arg("max_query_len") = -1,
        py::arg("pad_slot_id") = -1, py::arg("block_idx_last_scheduled_token") = py::none(),
        py::arg("initial_state_idx") = py::none(), py::arg("validate_data") = false,
        py::arg("num_accepted_tokens") = py::none());
  m.def("npu_fused_recurrent_gated_delta_rule",
        [](torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g,
           std::optional<torch::Tensor> beta, std::optional<float> scale,
           std::optional<torch::Tensor> h0, bool inplace, std::optional<torch::Tensor> cu,
           std::optional<torch::Tensor> idx, std::optional<torch::Tensor> acc, bool l2) {
          return xn::npu_fused_recurrent_gated_delta_rule(q, k, v, g, beta, scale, h0, inplace,
                                                          cu, idx, acc, l2);
        },
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("g"), py::arg("beta") = py::none(),
        py::arg("scale") = py::none(), py::arg("initial_state") = py::none(),
        py::arg("inplace_final_state") = true, py::arg("cu_seqlens") = py::none(),
        py::arg("ssm_state_indices") = py::none(), py::arg("num_accepted_tokens") = py::none(),
        py::arg("use_qk_l2norm_in_kernel") = false);
  m.def("rope_inplace",
        [](torch::Tensor x, torch::Tensor sin, torch::Tensor cos, uint32_t rope_dim) {
          xn::rope_inplace(x, sin, cos, rope_dim);
          return x;
        },
        py::arg("x"), py::arg("sin"), py::arg("cos"), py::arg("rope_dim") = 64);
  m.def("npu_fused_qkvzba_split_reshape_cat",
        [](torch::Tensor qkvz, torch::Tensor ba, int32_t nqk, int32_t nv, int32_t hqk,
           int32_t hv) { return xn::npu_fused_qkvzba_split_reshape_cat(qkvz, ba, nqk, nv, hqk, hv); },
        py::arg("mixed_qkvz"), py::arg("mixed_ba"), py::arg("num_heads_qk"),
        py::arg("num_heads_v"), py::arg("head_qk"), py::arg("head_v"));
  m.def("npu_fused_gdn_gating",
        [](torch::Tensor A_log, torch::Tensor a, torch::Tensor b, torch::Tensor dt_bias,
           float beta, float threshold) {
          return xn::npu_fused_gdn_gating(A_log, a, b, dt_bias, beta, threshold);
        },
        py::arg("A_log"), py::arg("a"), py::arg("b"), py::arg("dt_bias"), py::arg("beta") = 1.0f,
        py::arg("threshold") = 20.0f);
  m.def("npu_fused_sigmoid_gating_delta_rule_update",
        [](torch::Tensor A_log, torch::Tensor a, torch::Tensor dt_bias, torch::Tensor q,
           torch::Tensor k, torch::Tensor v, torch::Tensor b, torch::Tensor h0,
           torch::Tensor idx, torch::Tensor cu, std::optional<float> scale, bool l2,
           float sp_beta, float sp_thr) {
          return xn::npu_fused_sigmoid_gating_delta_rule_update(A_log, a, dt_bias, q, k, v, b,
                                                                h0, idx, cu, scale, l2, sp_beta,
                                                                sp_thr);
        },
        py::arg("A_log"), py::arg("a"), py::arg("dt_bias"), py::arg("q"), py::arg("k"),
        py::arg("v"), py::arg("b"), py::arg("initial_state_source"),
        py::arg("initial_state_indices"), py::arg("cu_seqlens"), py::arg("scale") = py::none(),
        py::arg("use_qk_l2norm_in_kernel") = false, py::arg("softplus_beta") = 1.0f,
        py::arg("softplus_threshold") = 20.0f);
  m.def("npu_chunk_gated_delta_rule",
        [](torch::Tensor q, torch::Tensor k, torch::Tensor v, torch::Tensor g, torch::Tensor beta,
           std::optional<float> scale, std::optional<torch::Tensor> h0, bool out_final,
           std::optional<torch::Tensor> cu, bool head_first, bool l2) {
          return xn::npu_chunk_gated_delta_rule(q, k, v, g, beta, scale, h0, out_final, cu,
                                                head_first, l2);
        },
        py::arg("q"), py::arg("k"), py::arg("v"), py::arg("g"), py::arg("beta"),
        py::arg("scale") = py::none(), py::arg("initial_state") = py::none(),
        py::arg("output_final_state") = false, py::arg("cu_seqlens") = py::none(),
        py::arg("head_first") = false, py::arg("use_qk_l2norm_in_kernel") = false);
  m.def("kernel_entry_point", [](const std::string& name) {
    return xn::KernelRegistry::get_instance().entry_point(name);
  });
  m.def("_runtime_execute", &py_runtime_execute, py::arg("kernel_name"), py::arg("grid_x"),
        py::arg("grid_y"), py::arg("grid_z"), py::arg("args"), py::arg("stream"));
  m.def("_runtime_layer_norm_fwd", &py_runtime_layer_norm_fwd, py::arg("x"), py::arg("weight"),
        py::arg("z"), py::arg("eps"), py::arg("group_size"));
  m.def("_runtime_has_decoder", [](const std::string& name) {
    return xn::has_packed_decoder(name);
  });
}
