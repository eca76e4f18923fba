// Kernel registry with the interface of the reference's KernelRegistry
// (triton_npu/kernel_registry.h:68-117).  The reference loads one AOT binary
// per kernel name from disk; here every kernel is linked into
// libxops_b200.so, so the registry is a static table from the reference's
// kernel names to the C-ABI entry points (include/xops_b200.h) that replace
// them.  register_kernel() succeeds for every compiled name (the binary path
// is ignored) and get_kernel_stub() returns the entry point's address.
#pragma once

#include <cstdint>
#include <string>

namespace xllm::kernel::npu {

using KernelStubHandle = void*;

class KernelRegistry {
 public:
  static KernelRegistry& get_instance();

  KernelRegistry(const KernelRegistry&) = delete;
  KernelRegistry& operator=(const KernelRegistry&) = delete;

  bool register_kernel(const std::string& kernel_name, const std::string& binary_path);
  KernelStubHandle get_kernel_stub(const std::string& kernel_name) const;
  bool is_kernel_registered(const std::string& kernel_name) const;
  void cleanup();
  // Workspace/lock sizes of a kernel: always 0 here (scratch is passed to
  // the entry points explicitly).
  bool get_kernel_workspace_config(const std::string& kernel_name, int64_t& workspace_size,
                                   int64_t& lock_init_value, int64_t& lock_num) const;
  // Name of the C-ABI entry point serving `kernel_name` ("" if none).
  std::string entry_point(const std::string& kernel_name) const;

 private:
  KernelRegistry() = default;
};

}  // namespace xllm::kernel::npu
