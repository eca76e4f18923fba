// Building blocks shared by the chunked gated-delta-rule kernels: cp.async
// copies, the 64x64 unit-lower-triangular inverse and per-chunk sequence
// bookkeeping (the tensor-core tile helpers are in gdn_tc.cuh).
#pragma once

#include "common.cuh"

namespace xops {
namespace gdn {

constexpr int BT = 64;     // chunk length (tokens)
constexpr int LDF = 65;     // fp32 row stride of 64x64 tiles

using bf16 = __nv_bfloat16;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// 16-byte async copy global -> shared; src_bytes == 0 zero-fills.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)),
               "l"(gmem), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::); }
// At most N of this thread's committed cp.async groups still pending.
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// T = (I + A)^-1 for a strictly lower 64x64 A (fp32, stride LDF), by blocks:
// 16x16 diagonal inverses (forward substitution, one thread per column),
// then T21 = -T22 A21 T11 merges 16 -> 32 -> 64.  sM is fp32 scratch of
// 32 x 33.  All 256 threads participate; ends with a barrier.
__device__ __forceinline__ void tri_inverse_64(const float* __restrict__ sA, float* __restrict__ sT,
                                               float* __restrict__ sM, int tid) {
  for (int e = tid; e < 64 * 64; e += 256) sT[(e >> 6) * LDF + (e & 63)] = 0.f;
  __syncthreads();
  if (tid < 64) {
    const int b = tid >> 4, c = tid & 15;
    const float* Ab = sA + (16 * b) * LDF + 16 * b;
    float x[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) x[i] = (i == c) ? 1.f : 0.f;
#pragma unroll
    for (int i = 1; i < 16; ++i) {
      float s = 0.f;
#pragma unroll
      for (int m = 0; m < i; ++m) s = fmaf(Ab[i * LDF + m], x[m], s);
      if (i > c) x[i] = -s;
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) sT[(16 * b + i) * LDF + 16 * b + c] = x[i];
  }
  __syncthreads();
  // 16 -> 32: blocks (1,0) and (3,2)
  for (int idx = tid; idx < 512; idx += 256) {
    const int p = idx >> 8, e = idx & 255, rr = e >> 4, cc = e & 15;
    const int r = 2 * p + 1, c = 2 * p;
    float s = 0.f;
    for (int m = cc; m < 16; ++m) s = fmaf(sA[(16 * r + rr) * LDF + 16 * c + m], sT[(16 * c + m) * LDF + 16 * c + cc], s);
    sM[p * 256 + rr * 16 + cc] = s;
  }
  __syncthreads();
  for (int idx = tid; idx < 512; idx += 256) {
    const int p = idx >> 8, e = idx & 255, rr = e >> 4, cc = e & 15;
    const int r = 2 * p + 1, c = 2 * p;
    float s = 0.f;
    for (int m = 0; m <= rr; ++m) s = fmaf(sT[(16 * r + rr) * LDF + 16 * r + m], sM[p * 256 + m * 16 + cc], s);
    sT[(16 * r + rr) * LDF + 16 * c + cc] = -s;
  }
  __syncthreads();
  // 32 -> 64: block rows 32..63, cols 0..31
  for (int idx = tid; idx < 1024; idx += 256) {
    const int rr = idx >> 5, cc = idx & 31;
    float s = 0.f;
    for (int m = cc; m < 32; ++m) s = fmaf(sA[(32 + rr) * LDF + m], sT[m * LDF + cc], s);
    sM[rr * 33 + cc] = s;
  }
  __syncthreads();
  for (int idx = tid; idx < 1024; idx += 256) {
    const int rr = idx >> 5, cc = idx & 31;
    float s = 0.f;
    for (int m = 0; m <= rr; ++m) s = fmaf(sT[(32 + rr) * LDF + 32 + m], sM[m * 33 + cc], s);
    sT[(32 + rr) * LDF + cc] = -s;
  }
  __syncthreads();
}

// In-place variant: sA (strictly lower A, fp32, stride LDF, zero upper part)
// is overwritten by T = (I + A)^-1.  Same blocking as tri_inverse_64; every
// block of T replaces the block of A it no longer needs, products are
// register-tiled (2x2 outputs per thread in the 32x32 merge).  sM: 32 x 33
// fp32 scratch.  All 256 threads participate; ends with a barrier.
__device__ __forceinline__ void tri_inverse_64_inplace(float* __restrict__ sA,
                                                       float* __restrict__ sM, int tid) {
  // 8x8 diagonal blocks: column c of block b by forward substitution (the
  // serial chain is at most 28 FMAs)
  {
    float x[8];
    const int b = tid >> 3, c = tid & 7;
    if (tid < 64) {
      const float* Ab = sA + (8 * b) * LDF + 8 * b;
#pragma unroll
      for (int i = 0; i < 8; ++i) x[i] = (i == c) ? 1.f : 0.f;
#pragma unroll
      for (int i = 1; i < 8; ++i) {
        float s = 0.f;
#pragma unroll
        for (int m = 0; m < i; ++m) s = fmaf(Ab[i * LDF + m], x[m], s);
        if (i > c) x[i] = -s;
      }
    }
    __syncthreads();
    if (tid < 64) {
#pragma unroll
      for (int i = 0; i < 8; ++i) sA[(8 * b + i) * LDF + 8 * b + c] = x[i];
    }
    __syncthreads();
  }
  // 8 -> 16 in each 16x16 diagonal block p: T10 = -T11 (A10 T00), one output
  // per thread
  {
    const int p = tid >> 6, e = tid & 63, rr = e >> 3, cc = e & 7;
    const int r0 = 16 * p + 8, c0 = 16 * p;  // A10 / T10 at rows r0.., cols c0..
    float s = 0.f;
#pragma unroll
    for (int m = 0; m < 8; ++m)
      if (m >= cc) s = fmaf(sA[(r0 + rr) * LDF + c0 + m], sA[(c0 + m) * LDF + c0 + cc], s);
    sM[p * 64 + rr * 8 + cc] = s;
    __syncthreads();
    float t = 0.f;
#pragma unroll
    for (int m = 0; m < 8; ++m)
      if (m <= rr) t = fmaf(sA[(r0 + rr) * LDF + r0 + m], sM[p * 64 + m * 8 + cc], t);
    sA[(r0 + rr) * LDF + c0 + cc] = -t;
  }
  __syncthreads();
  // 16 -> 32: T10 = -T11 A10 T00 and T32 = -T33 A32 T22; one output pair per thread
  {
    const int p = tid >> 7, e = tid & 127, rr = e >> 3, cc = (e & 7) * 2;
    const int r = 2 * p + 1, cb = 2 * p;
    float s0 = 0.f, s1 = 0.f;
    for (int m = cc; m < 16; ++m) {
      const float a = sA[(16 * r + rr) * LDF + 16 * cb + m];
      s0 = fmaf(a, sA[(16 * cb + m) * LDF + 16 * cb + cc], s0);
      s1 = fmaf(a, sA[(16 * cb + m) * LDF + 16 * cb + cc + 1], s1);
    }
    sM[p * 256 + rr * 16 + cc] = s0;
    sM[p * 256 + rr * 16 + cc + 1] = s1;
    __syncthreads();
    s0 = s1 = 0.f;
    for (int m = 0; m <= rr; ++m) {
      const float t = sA[(16 * r + rr) * LDF + 16 * r + m];
      s0 = fmaf(t, sM[p * 256 + m * 16 + cc], s0);
      s1 = fmaf(t, sM[p * 256 + m * 16 + cc + 1], s1);
    }
    sA[(16 * r + rr) * LDF + 16 * cb + cc] = -s0;
    sA[(16 * r + rr) * LDF + 16 * cb + cc + 1] = -s1;
  }
  __syncthreads();
  // 32 -> 64: T[32:64][0:32] = -T11 (A10 T00); 2x2 outputs per thread
  {
    const int rr = (tid >> 4) * 2, cc = (tid & 15) * 2;
    float s00 = 0.f, s01 = 0.f, s10 = 0.f, s11 = 0.f;
    for (int m = cc; m < 32; ++m) {
      const float a0 = sA[(32 + rr) * LDF + m], a1 = sA[(33 + rr) * LDF + m];
      const float t0 = sA[m * LDF + cc], t1 = sA[m * LDF + cc + 1];
      s00 = fmaf(a0, t0, s00); s01 = fmaf(a0, t1, s01);
      s10 = fmaf(a1, t0, s10); s11 = fmaf(a1, t1, s11);
    }
    sM[rr * 33 + cc] = s00; sM[rr * 33 + cc + 1] = s01;
    sM[(rr + 1) * 33 + cc] = s10; sM[(rr + 1) * 33 + cc + 1] = s11;
    __syncthreads();
    s00 = s01 = s10 = s11 = 0.f;
    for (int m = 0; m <= rr + 1; ++m) {
      const float u0 = sA[(32 + rr) * LDF + 32 + m];
      const float u1 = sA[(33 + rr) * LDF + 32 + m];
      const float q0 = sM[m * 33 + cc], q1 = sM[m * 33 + cc + 1];
      s00 = fmaf(u0, q0, s00); s01 = fmaf(u0, q1, s01);
      s10 = fmaf(u1, q0, s10); s11 = fmaf(u1, q1, s11);
    }
    sA[(32 + rr) * LDF + cc] = -s00; sA[(32 + rr) * LDF + cc + 1] = -s01;
    sA[(33 + rr) * LDF + cc] = -s10; sA[(33 + rr) * LDF + cc + 1] = -s11;
  }
  __syncthreads();
}

// Inclusive cumsum of g[0..63] (rows >= L zero) by warp 0 into sG; returns
// nothing, sG[L-1] is the chunk's last cumulative gate.
__device__ __forceinline__ void chunk_cumsum_warp(const float* __restrict__ graw, float* sG,
                                                  int lane) {
  const float a = graw[2 * lane], b = graw[2 * lane + 1];
  float pair = a + b, incl = pair;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float n = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += n;
  }
  const float excl = incl - pair;
  sG[2 * lane] = excl + a;
  sG[2 * lane + 1] = excl + a + b;
}

// (start, end) of sequence n.
__device__ __forceinline__ void seq_span(const int32_t* cu, int64_t n, int64_t T, int64_t& bos,
                                         int64_t& eos) {
  if (cu) {
    bos = cu[n];
    eos = cu[n + 1];
  } else {
    bos = n * T;
    eos = bos + T;
  }
}

// Maps a flattened chunk slot to (sequence, chunk start).  Returns false for
// slots past the last chunk.  One thread scans; the result is broadcast by
// the caller through shared memory.
__device__ __forceinline__ bool locate_chunk(const int32_t* cu, int64_t N, int64_t T, int64_t slot,
                                             int64_t& seq, int64_t& t0, int64_t& eos,
                                             int64_t& chunk_in_seq) {
  if (!cu) {
    const int64_t per = (T + BT - 1) / BT;
    if (per == 0) return false;
    seq = slot / per;
    if (seq >= N) return false;
    chunk_in_seq = slot - seq * per;
    t0 = seq * T + chunk_in_seq * BT;
    eos = seq * T + T;
    return true;
  }
  int64_t acc = 0;
  for (int64_t i = 0; i < N; ++i) {
    const int64_t s = cu[i], e = cu[i + 1];
    const int64_t nc = e > s ? (e - s + BT - 1) / BT : 0;
    if (slot < acc + nc) {
      seq = i;
      chunk_in_seq = slot - acc;
      t0 = s + chunk_in_seq * BT;
      eos = e;
      return true;
    }
    acc += nc;
  }
  return false;
}

// Chunk offset (number of chunks before sequence n).
__device__ __forceinline__ int64_t chunk_offset(const int32_t* cu, int64_t n, int64_t T) {
  if (!cu) return n * ((T + BT - 1) / BT);
  int64_t acc = 0;
  for (int64_t i = 0; i < n; ++i) {
    const int64_t len = (int64_t)cu[i + 1] - cu[i];
    acc += len > 0 ? (len + BT - 1) / BT : 0;
  }
  return acc;
}

// Opts a kernel into more than 48 KB of dynamic shared memory, once per
// device (the attribute is per device; every GPU a process uses needs it).
inline int ensure_smem_attr(const void* fn, size_t bytes, const char* what) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return set_error(XOPS_ERR_CUDA, "%s: cudaGetDevice: %s", what, cudaGetErrorString(e));
  e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
  if (e != cudaSuccess)
    return set_error(XOPS_ERR_CUDA, "%s: shared-memory attribute (%zu B): %s", what, bytes,
                     cudaGetErrorString(e));
  return XOPS_OK;
}

}  // namespace gdn
}  // namespace xops
