// GDN gates from the layer's projections (fused_gdn_gating).
//
// Follows fused_gdn_gating_decode_kernel
// (triton_npu/triton_src/test_fused_gdn_gating.py:10-43) and its torch
// reference (:45-57); the arithmetic lives in gate_math.cuh, shared with the
// chunked gated delta rule's fused-gating entry.  a and b are [rows, heads]
// (rows = batch for decode, tokens for prefill), g and beta are
// [1, rows, heads].
//
// Elementwise and HBM-bound; each thread handles four adjacent elements
// (one 8- or 16-byte load per input) in a grid-stride loop, and A_log /
// dt_bias are read through the read-only cache.
#include <algorithm>

#include "common.cuh"
#include "gate_math.cuh"

namespace xops {
namespace {

// Per-head constants -exp(A_log[h]) and dt_bias[h] are computed once per
// CTA into shared memory (heads <= GATE_SMEM_HEADS; beyond that they are
// recomputed per element).  Element i belongs to head i % heads; the index
// stays 32-bit (n < 2^31 is checked on the host).
constexpr int GATE_SMEM_HEADS = 2048;

template <typename TA, typename TB>
__global__ void __launch_bounds__(256) gdn_gating_kernel(
    const float* __restrict__ A_log, const TA* __restrict__ a, const TB* __restrict__ b,
    const float* __restrict__ dt_bias, float* __restrict__ g, TB* __restrict__ beta_out,
    int n, int heads, float sp_beta, float sp_thr, bool vec) {
  __shared__ float s_nega[GATE_SMEM_HEADS], s_dtb[GATE_SMEM_HEADS];
  const bool cached = heads <= GATE_SMEM_HEADS;
  if (cached) {
    for (int h = threadIdx.x; h < heads; h += blockDim.x) {
      s_nega[h] = -expf(A_log[h]);
      s_dtb[h] = dt_bias[h];
    }
    __syncthreads();
  }
  const int stride = gridDim.x * blockDim.x * 4;
  for (int i0 = (blockIdx.x * blockDim.x + threadIdx.x) * 4; i0 < n; i0 += stride) {
    float av[4], bv[4], gv[4], ov[4];
    const bool full = vec && i0 + 4 <= n;
    if (full) {
      load_vec<TA, 4>(a + i0, av);
      load_vec<TB, 4>(b + i0, bv);
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        av[u] = i0 + u < n ? to_f32<TA>(a[i0 + u]) : 0.f;
        bv[u] = i0 + u < n ? to_f32<TB>(b[i0 + u]) : 0.f;
      }
    }
    int h = i0 % heads;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float nega = cached ? s_nega[h] : -expf(__ldg(A_log + h));
      const float dtb = cached ? s_dtb[h] : __ldg(dt_bias + h);
      gv[u] = gate_g(nega, av[u], dtb, sp_beta, sp_thr);
      ov[u] = gate_beta_f32<TB>(bv[u]);
      h = h + 1 == heads ? 0 : h + 1;
    }
    if (full) {
      store_vec<float, 4>(g + i0, gv);
      store_vec<TB, 4>(beta_out + i0, ov);
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (i0 + u < n) {
          g[i0 + u] = gv[u];
          beta_out[i0 + u] = from_f32<TB>(ov[u]);
        }
      }
    }
  }
}

}  // namespace
}  // namespace xops

using namespace xops;

extern "C" int xops_fused_gdn_gating(const float* A_log, const void* a, const void* b,
                                     const float* dt_bias, float* g, void* beta_out,
                                     int64_t rows, int64_t heads, int a_dtype, int b_dtype,
                                     float softplus_beta, float softplus_threshold,
                                     void* stream) {
  XOPS_REQUIRE(rows >= 0 && heads >= 1 && rows * heads < (int64_t(1) << 31) - 4096,
               "fused_gdn_gating: bad shape (rows * heads must stay below 2^31)");
  auto ok_dtype = [](int d) { return d == XOPS_F32 || d == XOPS_BF16 || d == XOPS_F16; };
  XOPS_REQUIRE(ok_dtype(a_dtype) && ok_dtype(b_dtype),
               "fused_gdn_gating: a and b must be fp32, bf16 or fp16");
  XOPS_REQUIRE(softplus_beta > 0.f, "fused_gdn_gating: softplus beta must be positive");
  const int64_t n = rows * heads;
  if (n == 0) return XOPS_OK;
  XOPS_REQUIRE(A_log && a && b && dt_bias && g && beta_out, "fused_gdn_gating: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t threads = cdiv64(n, 4);
  const unsigned grid = (unsigned)std::min<int64_t>(cdiv64(threads, 256), 148 * 16);
  auto run = [&](auto ta, auto tb) {
    using TA = decltype(ta);
    using TB = decltype(tb);
    // vector loads need every group of four to start on a vector boundary
    const bool vec = (reinterpret_cast<uintptr_t>(a) % (4 * sizeof(TA))) == 0 &&
                     (reinterpret_cast<uintptr_t>(b) % (4 * sizeof(TB))) == 0 &&
                     (reinterpret_cast<uintptr_t>(beta_out) % (4 * sizeof(TB))) == 0 &&
                     aligned16(g);
    gdn_gating_kernel<TA, TB><<<grid, 256, 0, st>>>(A_log, (const TA*)a, (const TB*)b, dt_bias,
                                                    g, (TB*)beta_out, (int)n, (int)heads,
                                                    softplus_beta, softplus_threshold, vec);
    return check_launch("fused_gdn_gating");
  };
  auto with_b = [&](auto ta) {
    switch (b_dtype) {
      case XOPS_F32: return run(ta, float{});
      case XOPS_BF16: return run(ta, __nv_bfloat16{});
      default: return run(ta, __half{});
    }
  };
  switch (a_dtype) {
    case XOPS_F32: return with_b(float{});
    case XOPS_BF16: return with_b(__nv_bfloat16{});
    default: return with_b(__half{});
  }
}
