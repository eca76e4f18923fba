// De-interleave of the GDN input projections (fused_qkvzba_split_reshape_cat).
//
// Follows fused_qkvzba_split_reshape_cat_gqa_r{1..4}_kernel
// (triton_npu/triton_src/test_fused_qkvzba_split_reshape.py:36-352) and its
// torch reference (:463-506).  Per token row, each of the nqk key-head
// groups holds a contiguous block
//     q (hqk) | k (hqk) | v (r * hv) | z (r * hv)        r = nv / nqk
// in mixed_qkvz and  b (r) | a (r)  in mixed_ba.  The outputs gather them
// into  mixed_qkv = [all q | all k | all v],  z [nv, hv],  b [nv],  a [nv].
//
// A pure permutation, HBM-bound at twice the input bytes.  One CTA per token
// row copies the row's 16-byte vectors: consecutive threads take consecutive
// vectors of a sub-block, so every load and store is a coalesced run, and
// each thread keeps four vectors in flight.  Rows whose sub-blocks are not
// whole vectors take the element-wise path.
#include <type_traits>

#include "common.cuh"

namespace xops {
namespace {

struct QkvzShape {
  int nqk, nv, hqk, hv, r;
};

// destination offset (in elements, within the row) of element e of group g's
// input block; sets *to_z when the element belongs to z
__device__ __forceinline__ int qkvz_dst(const QkvzShape& s, int g, int e, bool* to_z) {
  const int rv = s.r * s.hv;
  *to_z = false;
  if (e < s.hqk) return g * s.hqk + e;                                     // q
  if (e < 2 * s.hqk) return s.nqk * s.hqk + g * s.hqk + (e - s.hqk);        // k
  if (e < 2 * s.hqk + rv) return 2 * s.nqk * s.hqk + g * rv + (e - 2 * s.hqk);  // v
  *to_z = true;
  return g * rv + (e - 2 * s.hqk - rv);                                    // z
}

template <typename T, typename TB, int VEC>
__global__ void __launch_bounds__(256) qkvzba_split_kernel(
    const T* __restrict__ qkvz, const TB* __restrict__ ba, T* __restrict__ qkv,
    T* __restrict__ z, TB* __restrict__ b_out, TB* __restrict__ a_out, QkvzShape s) {
  const int64_t row = blockIdx.x;
  const int W = 2 * s.hqk + 2 * s.r * s.hv;       // elements per group block
  const int nvec = s.nqk * W / VEC;               // vectors per row
  const int wv = W / VEC;
  const int qkv_stride = 2 * s.nqk * s.hqk + s.nv * s.hv;
  const T* src = qkvz + row * (int64_t)s.nqk * W;
  T* qrow = qkv + row * (int64_t)qkv_stride;
  T* zrow = z + row * (int64_t)s.nv * s.hv;
  using V = typename std::conditional<VEC * sizeof(T) == 16, uint4,
            typename std::conditional<VEC * sizeof(T) == 8, uint2, T>::type>::type;
  constexpr int U = 4;
  for (int j0 = threadIdx.x; j0 < nvec; j0 += U * blockDim.x) {
    V val[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * blockDim.x;
      if (j < nvec) val[u] = __ldg(reinterpret_cast<const V*>(src) + j);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * blockDim.x;
      if (j >= nvec) break;
      const int g = j / wv, e = (j - g * wv) * VEC;
      bool to_z;
      const int d = qkvz_dst(s, g, e, &to_z);
      *reinterpret_cast<V*>((to_z ? zrow : qrow) + d) = val[u];
    }
  }
  // b | a: 2 r scalars per group
  const TB* brow = ba + row * (int64_t)s.nqk * 2 * s.r;
  for (int t = threadIdx.x; t < s.nv; t += blockDim.x) {
    const int g = t / s.r, i = t - g * s.r;
    b_out[row * s.nv + t] = brow[g * 2 * s.r + i];
    a_out[row * s.nv + t] = brow[g * 2 * s.r + s.r + i];
  }
}

template <typename T, typename TB>
int launch_qkvz(const void* qkvz, const void* ba, void* qkv, void* z, void* b, void* a,
                int64_t rows, QkvzShape s, cudaStream_t st) {
  constexpr int V16 = 16 / (int)sizeof(T);
  const bool al16 = aligned16(qkvz) && aligned16(qkv) && aligned16(z);
  const bool al8 = ((reinterpret_cast<uintptr_t>(qkvz) | reinterpret_cast<uintptr_t>(qkv) |
                     reinterpret_cast<uintptr_t>(z)) & 7u) == 0;
  auto run = [&](auto vec_tag) {
    constexpr int VEC = decltype(vec_tag)::value;
    qkvzba_split_kernel<T, TB, VEC><<<(unsigned)rows, 256, 0, st>>>(
        (const T*)qkvz, (const TB*)ba, (T*)qkv, (T*)z, (TB*)b, (TB*)a, s);
    return check_launch("fused_qkvzba_split_reshape_cat");
  };
  if (al16 && s.hqk % V16 == 0 && s.hv % V16 == 0)
    return run(std::integral_constant<int, V16>{});
  if constexpr (V16 / 2 >= 1) {
    if (al8 && s.hqk % (V16 / 2) == 0 && s.hv % (V16 / 2) == 0)
      return run(std::integral_constant<int, V16 / 2>{});
  }
  return run(std::integral_constant<int, 1>{});
}

}  // namespace
}  // namespace xops

using namespace xops;

extern "C" int xops_fused_qkvzba_split_reshape_cat(const void* mixed_qkvz, const void* mixed_ba,
                                                   void* mixed_qkv, void* z, void* b, void* a,
                                                   int64_t rows, int64_t num_heads_qk,
                                                   int64_t num_heads_v, int64_t head_qk,
                                                   int64_t head_v, int qkvz_dtype, int ba_dtype,
                                                   void* stream) {
  const char* what = "fused_qkvzba_split_reshape_cat";
  XOPS_REQUIRE(rows >= 0 && rows < (int64_t(1) << 31), "%s: bad row count", what);
  XOPS_REQUIRE(num_heads_qk >= 1 && num_heads_v >= 1 && head_qk >= 1 && head_v >= 1,
               "%s: bad head counts", what);
  const int64_t r = num_heads_v / num_heads_qk;
  XOPS_REQUIRE(num_heads_v % num_heads_qk == 0 && r >= 1 && r <= 4,
               "%s only supports v_heads_per_qk in [1, 4], but got %lld for num_heads_qk=%lld "
               "num_heads_v=%lld", what, (long long)r, (long long)num_heads_qk,
               (long long)num_heads_v);
  XOPS_REQUIRE(num_heads_qk * (2 * head_qk + 2 * r * head_v) < (int64_t(1) << 30),
               "%s: rows too wide", what);
  auto ok = [](int d) { return d == XOPS_F32 || d == XOPS_BF16 || d == XOPS_F16; };
  XOPS_REQUIRE(ok(qkvz_dtype) && ok(ba_dtype), "%s: unsupported dtype", what);
  if (rows == 0) return XOPS_OK;
  XOPS_REQUIRE(mixed_qkvz && mixed_ba && mixed_qkv && z && b && a, "%s: null pointer", what);
  QkvzShape s{(int)num_heads_qk, (int)num_heads_v, (int)head_qk, (int)head_v, (int)r};
  cudaStream_t st = (cudaStream_t)stream;
  auto with_ba = [&](auto t) {
    using T = decltype(t);
    switch (ba_dtype) {
      case XOPS_F32: return launch_qkvz<T, float>(mixed_qkvz, mixed_ba, mixed_qkv, z, b, a, rows, s, st);
      case XOPS_BF16: return launch_qkvz<T, __nv_bfloat16>(mixed_qkvz, mixed_ba, mixed_qkv, z, b, a, rows, s, st);
      default: return launch_qkvz<T, __half>(mixed_qkvz, mixed_ba, mixed_qkv, z, b, a, rows, s, st);
    }
  };
  switch (qkvz_dtype) {
    case XOPS_F32: return with_ba(float{});
    case XOPS_BF16: return with_ba(__nv_bfloat16{});
    default: return with_ba(__half{});
  }
}
