// Launch of a kernel from the reference's packed argument buffer.
//
// The reference's OperationBase::execute (triton_npu/operation_base.h:137-192)
// packs [ffts, lock, workspace, <kernel arguments>, gridX, gridY, gridZ] with
// ArgsBuilder and hands the buffer to rtKernelLaunch.  Here the same buffer is
// decoded, per kernel name, back into the kernel's arguments, and the C-ABI
// entry point (include/xops_b200.h) that replaces that kernel runs with them
// on the given stream.  The argument order of every decoder is the one the
// reference's torch API packs for that kernel (file:line at each decoder).
//
// The reference's AOT binaries also carry compile-time constants that the
// buffer does not (Triton constexprs: dtypes, head sizes, flags).  For every
// name decoded here they are fixed by the kernel name or by the reference's
// own launch wrapper, and each decoder states the values it assumes.  Names
// whose computation cannot be recovered from the buffer (for example
// rope_inplace_kernel, whose rope and hidden sizes are constexprs) are not
// decoded: launching them returns kPackedNoDecoder and does nothing.
#pragma once

#include <cstddef>
#include <cstdint>
#include <string>

namespace xllm::kernel::npu {

// Status of launch_packed: 0 = launched; > 0 = the C ABI's xops_status_t of
// the entry point that ran (its message in *error); < 0 = nothing launched.
constexpr int32_t kPackedNoDecoder = -2;   // no decoder for this kernel name
constexpr int32_t kPackedBadBuffer = -3;   // the buffer does not hold this kernel's arguments

int32_t launch_packed(const std::string& kernel_name, const void* args, size_t size,
                      int32_t grid_x, int32_t grid_y, int32_t grid_z, void* stream,
                      std::string* error);

// True when launch_packed has a decoder for this kernel name.
bool has_packed_decoder(const std::string& kernel_name);

}  // namespace xllm::kernel::npu
