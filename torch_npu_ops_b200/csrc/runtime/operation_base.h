// OperationBase with the interface of the reference runtime's
// (triton_npu/operation_base.h:128-329).
//
// execute(stream, gridX, gridY, gridZ, build_args) packs the kernel's
// arguments exactly as the reference does -- [ffts, lock, workspace,
// <build_args>, gridX, gridY, gridZ] through ArgsBuilder -- and launches the
// kernel on `stream`.  Where the reference hands the buffer to
// rtKernelLaunch with an AOT binary, this build decodes it for the kernel
// name (packed_launch.h) and runs the C-ABI entry point that replaces the
// binary.  The three leading slots carry null pointers: the launches here
// need no cross-core control address, lock or per-launch workspace.
//
// Return value (the reference returns rtError_t, 0 on success):
//   0                 launched
//   > 0               the entry point's xops_status_t (bad argument, CUDA error)
//   -1                kernel name unknown to the registry (as the reference)
//   kPackedNoDecoder  name known, but its packed layout is not decodable
//   kPackedBadBuffer  the buffer does not hold that kernel's argument list
// Nothing is launched on a non-zero return; last_error() gives the message.
#pragma once

#include <cstdint>
#include <string>
#include <utility>

#include "args_builder.h"
#include "kernel_registry.h"
#include "packed_launch.h"

namespace xllm::kernel::npu {

class OperationBase {
 public:
  explicit OperationBase(std::string kernel_name, std::string binary_path = "")
      : kernel_name_(std::move(kernel_name)), binary_path_(std::move(binary_path)) {}
  virtual ~OperationBase() = default;

  template <class BuildArgsFn>
  int32_t execute(void* stream, int32_t gridX, int32_t gridY, int32_t gridZ,
                  BuildArgsFn&& build_args) {
    if (!ensure_registered()) {
      last_error_ = "kernel '" + kernel_name_ + "' is not in the registry";
      return -1;
    }
    ArgsBuilder ab;
    ab.add_aligned<void*>(nullptr, 8);  // ffts control address
    ab.add_aligned<void*>(nullptr, 8);  // lock
    ab.add_aligned<void*>(nullptr, 8);  // workspace
    build_args(ab);
    ab.add_aligned<int32_t>(gridX, 4);
    ab.add_aligned<int32_t>(gridY, 4);
    ab.add_aligned<int32_t>(gridZ, 4);
    last_args_size_ = ab.size();
    return launch_packed(kernel_name_, ab.data(), ab.size(), gridX, gridY, gridZ, stream,
                         &last_error_);
  }

  const std::string& kernel_name() const { return kernel_name_; }
  size_t last_args_size() const { return last_args_size_; }
  const std::string& last_error() const { return last_error_; }

 protected:
  bool ensure_registered() {
    auto& reg = KernelRegistry::get_instance();
    return reg.is_kernel_registered(kernel_name_) || reg.register_kernel(kernel_name_, binary_path_);
  }

 private:
  std::string kernel_name_;
  std::string binary_path_;
  size_t last_args_size_ = 0;
  std::string last_error_;
};

}  // namespace xllm::kernel::npu
