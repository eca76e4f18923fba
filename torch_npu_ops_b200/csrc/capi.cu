// Status plumbing shared by every C-ABI entry point.
#include <cstdarg>
#include <cstdio>
#include <atomic>

#include "common.cuh"

namespace xops {

static thread_local char g_last_error[1024] = "";
std::atomic<uint64_t> g_launches{0};

int set_error(int status, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_last_error, sizeof(g_last_error), fmt, ap);
  va_end(ap);
  return status;
}

// Called right after every launch: counts it and turns a launch-time error
// (bad configuration, missing kernel image) into XOPS_ERR_CUDA.
int check_launch(const char* what) {
  g_launches.fetch_add(1, std::memory_order_relaxed);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess)
    return set_error(XOPS_ERR_CUDA, "%s: launch failed: %s", what, cudaGetErrorString(e));
  return XOPS_OK;
}

}  // namespace xops

extern "C" const char* xops_last_error(void) { return xops::g_last_error; }
extern "C" const char* xops_version(void) { return "xops_b200 0.1 sm_100a"; }
extern "C" uint64_t xops_launch_count(void) { return xops::g_launches.load(); }
