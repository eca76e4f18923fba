// Shared device helpers for the sm_100a kernels behind the xops C ABI.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "xops_b200.h"

namespace xops {

// ---- status plumbing (defined in capi.cu) --------------------------------
int set_error(int status, const char* fmt, ...);
int check_launch(const char* what);
// wait-timeout flags of the streaming kernels: value since the last call
// (then cleared), -1 when the flag cannot be read
int take_norm_error();
int take_conv_error();
int take_rope_error();
int take_subop_error();
// L2-normalise `rows` rows of `heads` bf16 128-element segments (row stride
// x_stride elements) into contiguous y with the bulk-copy streaming kernel;
// -1 when the shape does not suit it (the caller then uses its own kernel)
int l2norm_rows_stream(const void* x, void* y, int64_t rows, int64_t heads, int64_t x_stride,
                       float eps, cudaStream_t st);

#define XOPS_REQUIRE(cond, ...)                                              \
  do {                                                                       \
    if (!(cond)) return ::xops::set_error(XOPS_ERR_INVALID_ARGUMENT,         \
                                          __VA_ARGS__);                      \
  } while (0)

#define XOPS_UNSUPPORTED(cond, ...)                                          \
  do {                                                                       \
    if (!(cond)) return ::xops::set_error(XOPS_ERR_UNSUPPORTED, __VA_ARGS__); \
  } while (0)

// ---- scalar conversions ---------------------------------------------------
template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) {
  return __bfloat162float(v);
}
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) {
  return __float2bfloat16_rn(v);
}
template <> __device__ __forceinline__ __half from_f32<__half>(float v) {
  return __float2half_rn(v);
}

// ---- vector loads: N contiguous elements of T as fp32 ---------------------
// Callers guarantee 16-byte alignment where N*sizeof(T) == 16.
template <typename T, int N>
__device__ __forceinline__ void load_vec(const T* __restrict__ p, float (&out)[N]) {
  constexpr int BYTES = N * (int)sizeof(T);
  if constexpr (BYTES % 16 == 0) {
    constexpr int CH = BYTES / 16;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      uint4 raw = __ldg(reinterpret_cast<const uint4*>(p) + c);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < 16 / (int)sizeof(T); ++i) out[c * (16 / sizeof(T)) + i] = to_f32<T>(e[i]);
    }
  } else if constexpr (BYTES % 8 == 0) {
    constexpr int CH = BYTES / 8;
#pragma unroll
    for (int c = 0; c < CH; ++c) {
      uint2 raw = __ldg(reinterpret_cast<const uint2*>(p) + c);
      const T* e = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int i = 0; i < 8 / (int)sizeof(T); ++i) out[c * (8 / sizeof(T)) + i] = to_f32<T>(e[i]);
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = to_f32<T>(p[i]);
  }
}

template <typename T, int N>
__device__ __forceinline__ void store_vec(T* __restrict__ p, const float (&v)[N]) {
  constexpr int BYTES = N * (int)sizeof(T);
  if constexpr (BYTES % 16 == 0) {
    constexpr int PER = 16 / (int)sizeof(T);
#pragma unroll
    for (int c = 0; c < BYTES / 16; ++c) {
      uint4 raw;
      T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
      for (int i = 0; i < PER; ++i) e[i] = from_f32<T>(v[c * PER + i]);
      reinterpret_cast<uint4*>(p)[c] = raw;
    }
  } else if constexpr (BYTES % 8 == 0) {
    constexpr int PER = 8 / (int)sizeof(T);
#pragma unroll
    for (int c = 0; c < BYTES / 8; ++c) {
      uint2 raw;
      T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
      for (int i = 0; i < PER; ++i) e[i] = from_f32<T>(v[c * PER + i]);
      reinterpret_cast<uint2*>(p)[c] = raw;
    }
  } else {
#pragma unroll
    for (int i = 0; i < N; ++i) p[i] = from_f32<T>(v[i]);
  }
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// fast divide (2 ulp): well inside every output tolerance, and a fraction of
// the instructions of an IEEE divide
__device__ __forceinline__ float silu_f(float x) { return __fdividef(x, 1.0f + __expf(-x)); }
__device__ __forceinline__ float sigmoid_f(float x) { return __fdividef(1.0f, 1.0f + __expf(-x)); }

__host__ __device__ __forceinline__ int64_t cdiv64(int64_t a, int64_t b) { return (a + b - 1) / b; }

// ---- packed fp32 pairs (sm_100: one instruction per two lanes' worth) -----
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)),
        "l"(*reinterpret_cast<const uint64_t*>(&c)));
  return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float2 fmul2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)));
  return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)));
  return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float2 fsub2(float2 a, float2 b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;"
      : "=l"(d)
      : "l"(*reinterpret_cast<const uint64_t*>(&a)), "l"(*reinterpret_cast<const uint64_t*>(&b)));
  return *reinterpret_cast<float2*>(&d);
}
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// SiLU for 16-bit outputs: x * sigmoid(x) = y + y * tanh(y), y = x / 2.  The
// hardware tanh approximation (relative error ~2^-11) is far below one
// bf16 / fp16 ulp of the result; fp32 outputs use silu_f.
__device__ __forceinline__ float2 silu2_lowp(float2 x) {
  const float2 y = fmul2(x, make_float2(0.5f, 0.5f));
  return ffma2(y, make_float2(tanh_approx(y.x), tanh_approx(y.y)), y);
}
// two 16-bit values packed in a 32-bit word <-> fp32 pair
template <typename T>
__device__ __forceinline__ float2 unpack2(uint32_t u);
template <>
__device__ __forceinline__ float2 unpack2<__nv_bfloat16>(uint32_t u) {
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
}
template <>
__device__ __forceinline__ float2 unpack2<__half>(uint32_t u) {
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
template <typename T>
__device__ __forceinline__ uint32_t pack2(float2 v);
template <>
__device__ __forceinline__ uint32_t pack2<__nv_bfloat16>(float2 v) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(v.x, v.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}
template <>
__device__ __forceinline__ uint32_t pack2<__half>(float2 v) {
  const __half2 h = __floats2half2_rn(v.x, v.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Opt a persistent streaming kernel into `bytes` of dynamic shared memory and
// the largest shared-memory carveout: without the carveout the driver may
// pick a smaller split that leaves room for only one of the CTAs an SM is
// meant to hold.
template <typename K>
inline bool set_stream_smem(K kern, int bytes) {
  return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) ==
             cudaSuccess &&
         cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                              (int)cudaSharedmemCarveoutMaxShared) == cudaSuccess;
}

}  // namespace xops
