// Row-group normalisations: layer_norm_fwd (LayerNorm / RMSNorm with bias and
// SiLU gate), gemma_rms_norm and the last-axis L2 norm.
//
// All three are HBM-bound: one read of x (and z), one write of y.  A warp owns
// one (row, group) segment and keeps it in registers (EPL elements per lane,
// loaded as 8- or 16-byte vectors, fully coalesced across the warp); the
// statistics are warp-shuffle reductions, so there is no shared memory and no
// block-wide barrier.  Segments longer than 32*64 elements use a block per
// segment with a two-pass loop over global memory.
#include <algorithm>

#include "common.cuh"
#include "tcgen05.cuh"

namespace xops {
namespace {

// ----------------------------------------------------------------------------
// layer_norm_fwd: grouped LN/RMS, optional bias, optional gate z.
// Follows layer_norm_fwd_kernel (triton_npu/triton_src/test_layernorm_fwd.py:
// 1125-1187): mean/rstd at group*M + row; gate silu(z) = z*sigmoid(z) applied
// before the statistics (norm_before_gate == 0) or to the output (== 1).
// ----------------------------------------------------------------------------
template <typename TX, typename TW, int EPL, bool RMS, bool HAS_Z, bool HAS_B>
__global__ void __launch_bounds__(256) layer_norm_warp_kernel(
    const TX* __restrict__ x, const TW* __restrict__ w, const TW* __restrict__ b,
    const TX* __restrict__ z, TX* __restrict__ y, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int64_t M, int64_t ngroups, int64_t sx, int64_t sz,
    int64_t sy, float eps, bool norm_before_gate) {
  constexpr int G = EPL * 32;
  const int lane = threadIdx.x & 31;
  const int64_t seg = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (seg >= M * ngroups) return;
  const int64_t row = seg / ngroups;
  const int64_t grp = seg - row * ngroups;
  const int64_t col0 = grp * G + (int64_t)lane * EPL;

  float xv[EPL], zv[EPL];
  load_vec<TX, EPL>(x + row * sx + col0, xv);
  if constexpr (HAS_Z) {
    load_vec<TX, EPL>(z + row * sz + col0, zv);
#pragma unroll
    for (int i = 0; i < EPL; ++i) zv[i] = zv[i] * sigmoid_f(zv[i]);
    if (!norm_before_gate) {
#pragma unroll
      for (int i = 0; i < EPL; ++i) xv[i] *= zv[i];
    }
  }
  float mu = 0.f;
  if constexpr (!RMS) {
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < EPL; ++i) s += xv[i];
    mu = warp_sum(s) * (1.0f / G);
  }
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const float d = xv[i] - mu;
    ss += d * d;
  }
  const float var = warp_sum(ss) * (1.0f / G);
  const float rstd = rsqrtf(var + eps);
  if (lane == 0) {
    rstd_out[grp * M + row] = rstd;
    if constexpr (!RMS) mean_out[grp * M + row] = mu;
  }
  float wv[EPL], bv[EPL], out[EPL];
  load_vec<TW, EPL>(w + col0, wv);
  if constexpr (HAS_B) load_vec<TW, EPL>(b + col0, bv);
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    float t = (xv[i] - mu) * rstd * wv[i];
    if constexpr (HAS_B) t += bv[i];
    if constexpr (HAS_Z) {
      if (norm_before_gate) t *= zv[i];
    }
    out[i] = t;
  }
  store_vec<TX, EPL>(y + row * sy + col0, out);
}

// Short segments (G * sizeof(TX) <= 512 B, e.g. the gated RMSNorm's 128-wide
// groups): a lane owns one 16-byte vector, LPR = G / VEC lanes hold a
// segment, a warp covers 32 / LPR segments per pass and UNROLL passes are
// loaded before any is reduced, so every lane keeps 2 * UNROLL 16-byte loads
// (x and z) in flight.  Reductions are xor-shuffles inside the LPR-lane group.
template <typename TX, typename TW, int G, bool RMS, bool HAS_Z, bool HAS_B>
__global__ void __launch_bounds__(256) layer_norm_packed_kernel(
    const TX* __restrict__ x, const TW* __restrict__ w, const TW* __restrict__ b,
    const TX* __restrict__ z, TX* __restrict__ y, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int64_t M, int64_t ngroups, int64_t sx, int64_t sz,
    int64_t sy, float eps, bool norm_before_gate) {
  constexpr int VEC = 16 / (int)sizeof(TX);
  constexpr int LPR = G / VEC;
  static_assert(LPR >= 1 && LPR <= 32 && (LPR & (LPR - 1)) == 0, "bad packing");
  constexpr int SPW = 32 / LPR;  // segments per warp pass
  constexpr int UNROLL = 4;
  const int lane = threadIdx.x & 31;
  const int sub = lane / LPR, li = lane % LPR;
  const int64_t total = M * ngroups;
  const int64_t warp_global = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t seg0 = warp_global * (SPW * UNROLL);
  // x and z stay raw 16-byte words until their segment is processed
  uint4 xr[UNROLL], zr[UNROLL];
  int64_t row[UNROLL], grp[UNROLL];
  bool live[UNROLL];
#pragma unroll
  for (int u = 0; u < UNROLL; ++u) {
    const int64_t seg = seg0 + u * SPW + sub;
    live[u] = seg < total;
    row[u] = live[u] ? seg / ngroups : 0;
    grp[u] = live[u] ? seg - row[u] * ngroups : 0;
    if (live[u]) {
      xr[u] = __ldg(reinterpret_cast<const uint4*>(x + row[u] * sx + grp[u] * G + li * VEC));
      if constexpr (HAS_Z)
        zr[u] = __ldg(reinterpret_cast<const uint4*>(z + row[u] * sz + grp[u] * G + li * VEC));
    } else {
      xr[u] = make_uint4(0, 0, 0, 0);
      zr[u] = make_uint4(0, 0, 0, 0);
    }
  }
#pragma unroll
  for (int u = 0; u < UNROLL; ++u) {
    float xv[1][VEC], zv[1][VEC];
    {
      const TX* ex = reinterpret_cast<const TX*>(&xr[u]);
#pragma unroll
      for (int i = 0; i < VEC; ++i) xv[0][i] = to_f32<TX>(ex[i]);
      if constexpr (HAS_Z) {
        const TX* ez = reinterpret_cast<const TX*>(&zr[u]);
#pragma unroll
        for (int i = 0; i < VEC; ++i) zv[0][i] = to_f32<TX>(ez[i]);
      }
    }
    if constexpr (HAS_Z) {
#pragma unroll
      for (int i = 0; i < VEC; ++i) zv[0][i] = zv[0][i] * sigmoid_f(zv[0][i]);
      if (!norm_before_gate) {
#pragma unroll
        for (int i = 0; i < VEC; ++i) xv[0][i] *= zv[0][i];
      }
    }
    float mu = 0.f;
    if constexpr (!RMS) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < VEC; ++i) s += xv[0][i];
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      mu = s * (1.0f / G);
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      const float d = xv[0][i] - mu;
      ss += d * d;
    }
#pragma unroll
    for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = rsqrtf(ss * (1.0f / G) + eps);
    if (!live[u]) continue;
    if (li == 0) {
      rstd_out[grp[u] * M + row[u]] = rstd;
      if constexpr (!RMS) mean_out[grp[u] * M + row[u]] = mu;
    }
    float wv[VEC], bv[VEC], out[VEC];
    load_vec<TW, VEC>(w + grp[u] * G + li * VEC, wv);
    if constexpr (HAS_B) load_vec<TW, VEC>(b + grp[u] * G + li * VEC, bv);
#pragma unroll
    for (int i = 0; i < VEC; ++i) {
      float t = (xv[0][i] - mu) * rstd * wv[i];
      if constexpr (HAS_B) t += bv[i];
      if constexpr (HAS_Z) {
        if (norm_before_gate) t *= zv[0][i];
      }
      out[i] = t;
    }
    store_vec<TX, VEC>(y + row[u] * sy + grp[u] * G + li * VEC, out);
  }
}

// Long segments: one block per (row, group), two passes over global memory.
template <typename TX, typename TW, bool RMS, bool HAS_Z, bool HAS_B>
__global__ void __launch_bounds__(512) layer_norm_block_kernel(
    const TX* __restrict__ x, const TW* __restrict__ w, const TW* __restrict__ b,
    const TX* __restrict__ z, TX* __restrict__ y, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int64_t M, int64_t ngroups, int64_t G, int64_t sx,
    int64_t sz, int64_t sy, float eps, bool norm_before_gate) {
  __shared__ float red[2][32];
  const int64_t row = blockIdx.x / ngroups;
  const int64_t grp = blockIdx.x - row * ngroups;
  const TX* xr = x + row * sx + grp * G;
  const TX* zr = HAS_Z ? z + row * sz + grp * G : nullptr;
  auto load_x = [&](int64_t c) {
    float v = to_f32<TX>(xr[c]);
    if constexpr (HAS_Z) {
      if (!norm_before_gate) {
        const float zz = to_f32<TX>(zr[c]);
        v *= zz * sigmoid_f(zz);
      }
    }
    return v;
  };
  float s = 0.f, ss = 0.f;
  for (int64_t c = threadIdx.x; c < G; c += blockDim.x) {
    const float v = load_x(c);
    s += v;
    ss += v * v;
  }
  s = warp_sum(s);
  ss = warp_sum(ss);
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) { red[0][wid] = s; red[1][wid] = ss; }
  __syncthreads();
  if (wid == 0) {
    s = lane < nw ? red[0][lane] : 0.f;
    ss = lane < nw ? red[1][lane] : 0.f;
    s = warp_sum(s);
    ss = warp_sum(ss);
    if (lane == 0) { red[0][0] = s; red[1][0] = ss; }
  }
  __syncthreads();
  const float inv_g = 1.0f / (float)G;
  const float mu = RMS ? 0.f : red[0][0] * inv_g;
  // E[x^2] - mu^2 in fp32 is accurate for normalised activations; the
  // reference kernels compute the same two moments.
  const float var = fmaxf(red[1][0] * inv_g - mu * mu, 0.f);
  const float rstd = rsqrtf(var + eps);
  if (threadIdx.x == 0) {
    rstd_out[grp * M + row] = rstd;
    if constexpr (!RMS) mean_out[grp * M + row] = mu;
  }
  TX* yr = y + row * sy + grp * G;
  for (int64_t c = threadIdx.x; c < G; c += blockDim.x) {
    float t = (load_x(c) - mu) * rstd * to_f32<TW>(w[grp * G + c]);
    if constexpr (HAS_B) t += to_f32<TW>(b[grp * G + c]);
    if constexpr (HAS_Z) {
      if (norm_before_gate) {
        const float zz = to_f32<TX>(zr[c]);
        t *= zz * sigmoid_f(zz);
      }
    }
    yr[c] = from_f32<TX>(t);
  }
}

template <typename TX, typename TW, int EPL, bool RMS, bool HAS_Z, bool HAS_B>
int launch_ln_warp(const void* x, const void* w, const void* b, const void* z, void* y,
                   float* mean, float* rstd, int64_t M, int64_t ng, int64_t sx, int64_t sz,
                   int64_t sy, float eps, bool nbg, cudaStream_t st) {
  const int64_t segs = M * ng;
  const int64_t blocks = cdiv64(segs, 8);
  layer_norm_warp_kernel<TX, TW, EPL, RMS, HAS_Z, HAS_B><<<(unsigned)blocks, 256, 0, st>>>(
      (const TX*)x, (const TW*)w, (const TW*)b, (const TX*)z, (TX*)y, mean, rstd, M, ng, sx, sz,
      sy, eps, nbg);
  return check_launch("layer_norm_fwd");
}


// ----------------------------------------------------------------------------
// Short-group path for 16-bit tensors with contiguous rows (the gated
// RMSNorm's 128-wide groups of [tokens x heads*128]): the (row, group)
// segments are then contiguous in memory, so a tile of segments of x (and z)
// is one contiguous range.  A persistent CTA streams tiles of ~16 KB per
// tensor with 1-D bulk copies into a ring of RN_NS shared stages (warp 0),
// and 8 consumer warps normalise them: LPR = G / 8 lanes per segment, one
// 16-byte piece each, shuffle reductions inside the lane group, 16-byte
// stores of y.  Loads in flight per SM no longer depend on registers.
// ----------------------------------------------------------------------------
constexpr int RN_NS = 3, RN_TILE_BYTES = 16384, RN_NT = 32 + 256;
constexpr uint32_t RN_WAIT = 1u << 26;
__device__ int g_norm_error = 0;

template <typename TX, typename TW, int G, bool RMS, bool HAS_Z, bool HAS_B>
__global__ void __launch_bounds__(RN_NT, 2) layer_norm_stream_kernel(
    const TX* __restrict__ x, const TW* __restrict__ w, const TW* __restrict__ b,
    const TX* __restrict__ z, TX* __restrict__ y, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int64_t M, int64_t ngroups, float eps, bool norm_before_gate) {
  constexpr int SEGS = RN_TILE_BYTES / (G * 2);   // segments per tile
  constexpr int LPR = G / 8;                       // lanes per segment
  constexpr int SPW = 32 / LPR;                    // segments per warp pass
  constexpr int STAGE = (HAS_Z ? 2 : 1) * RN_TILE_BYTES;
  extern __shared__ unsigned char rn_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(rn_raw) + 127) & ~static_cast<uintptr_t>(127));
  __shared__ uint64_t full[RN_NS], empty[RN_NS];
  __shared__ int abort_sh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t total = M * ngroups;
  const int64_t tiles = (total + SEGS - 1) / SEGS;
  if (tid == 0) {
    for (int s = 0; s < RN_NS; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 8);
    }
    tc::mbar_fence_init();
    abort_sh = 0;
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      for (int64_t k = 0;; ++k) {
        const int64_t t = blockIdx.x + k * gridDim.x;
        if (t >= tiles) break;
        const int s = (int)(k % RN_NS);
        if (k >= RN_NS && !tc::mbar_wait(&empty[s], (uint32_t)((k / RN_NS - 1) & 1), RN_WAIT)) {
          atomicExch(&g_norm_error, 1);
          atomicExch(&abort_sh, 1);
          break;
        }
        if (*(volatile int*)&abort_sh) break;
        const int64_t s0 = t * SEGS;
        const int n = (int)(total - s0 < SEGS ? total - s0 : SEGS);
        const uint32_t bytes = (uint32_t)n * G * 2;
        unsigned char* st = sm + s * STAGE;
        tc::mbar_arrive_expect_tx(&full[s], (HAS_Z ? 2 : 1) * bytes);
        tc::bulk_load(st, x + s0 * G, bytes, &full[s]);
        if constexpr (HAS_Z) tc::bulk_load(st + RN_TILE_BYTES, z + s0 * G, bytes, &full[s]);
      }
    }
    return;
  }
  const int cw = warp - 1, sub = lane / LPR, li = lane % LPR;
  for (int64_t k = 0;; ++k) {
    const int64_t t = blockIdx.x + k * gridDim.x;
    if (t >= tiles) break;
    const int s = (int)(k % RN_NS);
    if (!tc::mbar_wait(&full[s], (uint32_t)((k / RN_NS) & 1), RN_WAIT)) {
      atomicExch(&g_norm_error, 1);
      break;
    }
    const unsigned char* st = sm + s * STAGE;
    const int64_t s0 = t * SEGS;
#pragma unroll
    for (int p = 0; p < SEGS / (8 * SPW); ++p) {
      const int si = (p * 8 + cw) * SPW + sub;  // segment in tile
      const int64_t seg = s0 + si;
      const bool live = seg < total;
      const uint4 xr = *reinterpret_cast<const uint4*>(st + si * (G * 2) + li * 16);
      float2 xv[4] = {unpack2<TX>(xr.x), unpack2<TX>(xr.y), unpack2<TX>(xr.z), unpack2<TX>(xr.w)};
      float2 gz[4];
      if constexpr (HAS_Z) {
        const uint4 zr =
            *reinterpret_cast<const uint4*>(st + RN_TILE_BYTES + si * (G * 2) + li * 16);
        gz[0] = silu2_lowp(unpack2<TX>(zr.x));
        gz[1] = silu2_lowp(unpack2<TX>(zr.y));
        gz[2] = silu2_lowp(unpack2<TX>(zr.z));
        gz[3] = silu2_lowp(unpack2<TX>(zr.w));
        if (!norm_before_gate) {
#pragma unroll
          for (int u = 0; u < 4; ++u) xv[u] = fmul2(xv[u], gz[u]);
        }
      }
      float mu = 0.f;
      if constexpr (!RMS) {
        float sum = 0.f;
#pragma unroll
        for (int u = 0; u < 4; ++u) sum += xv[u].x + xv[u].y;
#pragma unroll
        for (int o = LPR / 2; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
        mu = sum * (1.0f / G);
#pragma unroll
        for (int u = 0; u < 4; ++u) xv[u] = fsub2(xv[u], make_float2(mu, mu));
      }
      float2 ss2 = fmul2(xv[0], xv[0]);
#pragma unroll
      for (int u = 1; u < 4; ++u) ss2 = ffma2(xv[u], xv[u], ss2);
      float ss = ss2.x + ss2.y;
#pragma unroll
      for (int o = LPR / 2; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      const float rstd = rsqrtf(ss * (1.0f / G) + eps);
      if (live) {
        const uint32_t row = (uint32_t)(seg / ngroups), grp = (uint32_t)(seg - (int64_t)row * ngroups);
        if (li == 0) {
          rstd_out[(int64_t)grp * M + row] = rstd;
          if constexpr (!RMS) mean_out[(int64_t)grp * M + row] = mu;
        }
        float wv[8], bv[8];
        load_vec<TW, 8>(w + (int64_t)grp * G + li * 8, wv);
        if constexpr (HAS_B) load_vec<TW, 8>(b + (int64_t)grp * G + li * 8, bv);
        uint4 out;
        uint32_t* po = &out.x;
        const float2 r2 = make_float2(rstd, rstd);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          float2 v = fmul2(fmul2(xv[u], r2), make_float2(wv[2 * u], wv[2 * u + 1]));
          if constexpr (HAS_B) v = fadd2(v, make_float2(bv[2 * u], bv[2 * u + 1]));
          if constexpr (HAS_Z) {
            if (norm_before_gate) v = fmul2(v, gz[u]);
          }
          po[u] = pack2<TX>(v);
        }
        *reinterpret_cast<uint4*>(y + seg * G + li * 8) = out;
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[s]);
  }
}

template <typename TX, typename TW, int GG, bool RMS, bool HAS_Z, bool HAS_B>
int launch_ln_stream(const void* x, const void* w, const void* b, const void* z, void* y,
                     float* mean, float* rstd, int64_t M, int64_t ng, float eps, bool nbg,
                     cudaStream_t st) {
  constexpr int SEGS = RN_TILE_BYTES / (GG * 2);
  constexpr int SMEM = RN_NS * (HAS_Z ? 2 : 1) * RN_TILE_BYTES + 128;
  auto kern = layer_norm_stream_kernel<TX, TW, GG, RMS, HAS_Z, HAS_B>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
    return set_error(XOPS_ERR_CUDA, "layer_norm_fwd: shared-memory attribute failed");
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t tiles = cdiv64(M * ng, SEGS);
  const unsigned grid = (unsigned)std::min<int64_t>(tiles, 2 * (int64_t)sms);
  kern<<<grid, RN_NT, SMEM, st>>>((const TX*)x, (const TW*)w, (const TW*)b, (const TX*)z, (TX*)y,
                                  mean, rstd, M, ng, eps, nbg);
  return check_launch("layer_norm_fwd");
}

template <typename TX, typename TW, bool RMS, bool HAS_Z, bool HAS_B>
int dispatch_ln(const void* x, const void* w, const void* b, const void* z, void* y, float* mean,
                float* rstd, int64_t M, int64_t N, int64_t G, int64_t sx, int64_t sz, int64_t sy,
                float eps, bool nbg, cudaStream_t st) {
  const int64_t ng = N / G;
  // streaming path: 16-bit, contiguous rows (segments adjacent in memory),
  // enough segments to keep a grid of persistent CTAs busy
  if constexpr (sizeof(TX) == 2) {
    const bool contiguous = sx == N && sy == N && (!HAS_Z || sz == N);
    if (contiguous && M * ng >= 8192 && M * ng < (int64_t(1) << 31)) {
      if (G == 64) return launch_ln_stream<TX, TW, 64, RMS, HAS_Z, HAS_B>(x, w, b, z, y, mean, rstd, M, ng, eps, nbg, st);
      if (G == 128) return launch_ln_stream<TX, TW, 128, RMS, HAS_Z, HAS_B>(x, w, b, z, y, mean, rstd, M, ng, eps, nbg, st);
      if (G == 256) return launch_ln_stream<TX, TW, 256, RMS, HAS_Z, HAS_B>(x, w, b, z, y, mean, rstd, M, ng, eps, nbg, st);
    }
  }
  // packed path: 16-byte lanes, several short segments per warp
  constexpr int VEC = 16 / (int)sizeof(TX);
#define XOPS_LN_PACKED(GG)                                                                  \
  if (G == GG && GG % VEC == 0 && GG / VEC <= 32) {                                         \
    constexpr int SPW = 32 / (GG / VEC > 0 ? GG / VEC : 1);                                 \
    const int64_t warps = cdiv64(M * ng, (int64_t)SPW * 4);                                 \
    layer_norm_packed_kernel<TX, TW, GG, RMS, HAS_Z, HAS_B><<<(unsigned)cdiv64(warps, 8), 256, \
                                                              0, st>>>(                     \
        (const TX*)x, (const TW*)w, (const TW*)b, (const TX*)z, (TX*)y, mean, rstd, M, ng, sx, \
        sz, sy, eps, nbg);                                                                  \
    return check_launch("layer_norm_fwd");                                                  \
  }
  if constexpr (sizeof(TX) == 2) {
    XOPS_LN_PACKED(64)
    XOPS_LN_PACKED(128)
    XOPS_LN_PACKED(256)
  } else {
    XOPS_LN_PACKED(64)
    XOPS_LN_PACKED(128)
  }
#undef XOPS_LN_PACKED
  // warp path: G = 32 * EPL, vector width must divide each lane's slice
  switch (G) {
#define XOPS_LN_CASE(EPL)                                                                   \
  case 32 * EPL:                                                                            \
    return launch_ln_warp<TX, TW, EPL, RMS, HAS_Z, HAS_B>(x, w, b, z, y, mean, rstd, M, ng, \
                                                          sx, sz, sy, eps, nbg, st);
    XOPS_LN_CASE(1)
    XOPS_LN_CASE(2)
    XOPS_LN_CASE(4)
    XOPS_LN_CASE(8)
    XOPS_LN_CASE(16)
    XOPS_LN_CASE(32)
    XOPS_LN_CASE(64)
#undef XOPS_LN_CASE
    default:
      break;
  }
  const int threads = G >= 4096 ? 512 : 256;
  layer_norm_block_kernel<TX, TW, RMS, HAS_Z, HAS_B><<<(unsigned)(M * ng), threads, 0, st>>>(
      (const TX*)x, (const TW*)w, (const TW*)b, (const TX*)z, (TX*)y, mean, rstd, M, ng, G, sx,
      sz, sy, eps, nbg);
  return check_launch("layer_norm_fwd");
}

template <typename TX, typename TW>
int dispatch_ln_flags(const void* x, const void* w, const void* b, const void* z, void* y,
                      float* mean, float* rstd, int64_t M, int64_t N, int64_t G, int64_t sx,
                      int64_t sz, int64_t sy, float eps, bool nbg, bool rms, cudaStream_t st) {
  const bool hz = z != nullptr, hb = b != nullptr;
#define XOPS_LN_FLAGS(R, Z, B)                                                                \
  if (rms == R && hz == Z && hb == B)                                                         \
    return dispatch_ln<TX, TW, R, Z, B>(x, w, b, z, y, mean, rstd, M, N, G, sx, sz, sy, eps, \
                                        nbg, st);
  XOPS_LN_FLAGS(true, true, true)
  XOPS_LN_FLAGS(true, true, false)
  XOPS_LN_FLAGS(true, false, true)
  XOPS_LN_FLAGS(true, false, false)
  XOPS_LN_FLAGS(false, true, true)
  XOPS_LN_FLAGS(false, true, false)
  XOPS_LN_FLAGS(false, false, true)
  XOPS_LN_FLAGS(false, false, false)
#undef XOPS_LN_FLAGS
  return set_error(XOPS_ERR_UNSUPPORTED, "layer_norm_fwd: unreachable flag combination");
}

// ----------------------------------------------------------------------------
// gemma_rms_norm: y = x * rsqrt(mean(x^2)+eps) * (1 + gamma); rstd per row.
// ----------------------------------------------------------------------------
template <typename TX, typename TW, int EPL>
__global__ void __launch_bounds__(256) gemma_warp_kernel(const TX* __restrict__ x,
                                                         const TW* __restrict__ gamma,
                                                         TX* __restrict__ y,
                                                         float* __restrict__ rstd_out,
                                                         int64_t rows, float eps) {
  constexpr int N = EPL * 32;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  float xv[EPL], gv[EPL];
  load_vec<TX, EPL>(x + row * N + lane * EPL, xv);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) ss += xv[i] * xv[i];
  const float rstd = rsqrtf(warp_sum(ss) * (1.0f / N) + eps);
  if (lane == 0) rstd_out[row] = rstd;
  load_vec<TW, EPL>(gamma + lane * EPL, gv);
#pragma unroll
  for (int i = 0; i < EPL; ++i) xv[i] = xv[i] * rstd * (1.0f + gv[i]);
  store_vec<TX, EPL>(y + row * N + lane * EPL, xv);
}

template <typename TX, typename TW>
__global__ void __launch_bounds__(512) gemma_block_kernel(const TX* __restrict__ x,
                                                          const TW* __restrict__ gamma,
                                                          TX* __restrict__ y,
                                                          float* __restrict__ rstd_out,
                                                          int64_t N, float eps) {
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const TX* xr = x + row * N;
  float ss = 0.f;
  for (int64_t c = threadIdx.x; c < N; c += blockDim.x) {
    const float v = to_f32<TX>(xr[c]);
    ss += v * v;
  }
  ss = warp_sum(ss);
  const int wid = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  if (lane == 0) red[wid] = ss;
  __syncthreads();
  if (wid == 0) {
    ss = warp_sum(lane < nw ? red[lane] : 0.f);
    if (lane == 0) red[0] = ss;
  }
  __syncthreads();
  const float rstd = rsqrtf(red[0] / (float)N + eps);
  if (threadIdx.x == 0) rstd_out[row] = rstd;
  for (int64_t c = threadIdx.x; c < N; c += blockDim.x)
    y[row * N + c] = from_f32<TX>(to_f32<TX>(xr[c]) * rstd * (1.0f + to_f32<TW>(gamma[c])));
}

template <typename TX, typename TW>
int dispatch_gemma(const void* x, const void* g, void* y, float* rstd, int64_t rows, int64_t N,
                   float eps, cudaStream_t st) {
  const unsigned blocks = (unsigned)cdiv64(rows, 8);
  switch (N) {
#define XOPS_G_CASE(EPL)                                                                     \
  case 32 * EPL:                                                                             \
    gemma_warp_kernel<TX, TW, EPL><<<blocks, 256, 0, st>>>((const TX*)x, (const TW*)g, (TX*)y, \
                                                           rstd, rows, eps);                 \
    return check_launch("gemma_rms_norm");
    XOPS_G_CASE(2)
    XOPS_G_CASE(4)
    XOPS_G_CASE(8)
    XOPS_G_CASE(16)
    XOPS_G_CASE(32)
    XOPS_G_CASE(64)
#undef XOPS_G_CASE
    default:
      break;
  }
  gemma_block_kernel<TX, TW><<<(unsigned)rows, 512, 0, st>>>((const TX*)x, (const TW*)g, (TX*)y,
                                                             rstd, N, eps);
  return check_launch("gemma_rms_norm");
}

// ----------------------------------------------------------------------------
// l2norm over the last axis (l2norm_fwd_kernel2_loop semantics,
// triton_npu/triton_src/test_l2norm.py:17-60): y = x * rsqrt(sum x^2 + eps).
// ----------------------------------------------------------------------------
template <typename T, int EPL>
__global__ void __launch_bounds__(256) l2norm_warp_kernel(const T* __restrict__ x,
                                                          T* __restrict__ y, int64_t rows,
                                                          float eps) {
  constexpr int N = EPL * 32;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  float v[EPL];
  load_vec<T, EPL>(x + row * N + lane * EPL, v);
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) ss += v[i] * v[i];
  const float r = rsqrtf(warp_sum(ss) + eps);
#pragma unroll
  for (int i = 0; i < EPL; ++i) v[i] *= r;
  store_vec<T, EPL>(y + row * N + lane * EPL, v);
}

template <typename T>
__global__ void __launch_bounds__(256) l2norm_generic_kernel(const T* __restrict__ x,
                                                             T* __restrict__ y, int64_t rows,
                                                             int64_t N, float eps) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  float ss = 0.f;
  for (int64_t c = lane; c < N; c += 32) {
    const float v = to_f32<T>(x[row * N + c]);
    ss += v * v;
  }
  const float r = rsqrtf(warp_sum(ss) + eps);
  for (int64_t c = lane; c < N; c += 32) y[row * N + c] = from_f32<T>(to_f32<T>(x[row * N + c]) * r);
}

template <typename T>
int dispatch_l2(const void* x, void* y, int64_t rows, int64_t N, float eps, cudaStream_t st) {
  const unsigned blocks = (unsigned)cdiv64(rows, 8);
  switch (N) {
#define XOPS_L2_CASE(EPL)                                                                \
  case 32 * EPL:                                                                         \
    l2norm_warp_kernel<T, EPL><<<blocks, 256, 0, st>>>((const T*)x, (T*)y, rows, eps); \
    return check_launch("l2norm_last_dim");
    XOPS_L2_CASE(2)
    XOPS_L2_CASE(4)
    XOPS_L2_CASE(8)
#undef XOPS_L2_CASE
    default:
      break;
  }
  l2norm_generic_kernel<T><<<blocks, 256, 0, st>>>((const T*)x, (T*)y, rows, N, eps);
  return check_launch("l2norm_last_dim");
}

bool valid_dtype(int d) { return d == XOPS_F32 || d == XOPS_BF16 || d == XOPS_F16; }

}  // namespace
}  // namespace xops

using namespace xops;

extern "C" int xops_layer_norm_fwd(const void* x, const void* weight, const void* bias,
                                   const void* z, void* y, float* mean, float* rstd, int64_t M,
                                   int64_t N, int64_t group_size, int64_t stride_x_row,
                                   int64_t stride_z_row, int64_t stride_y_row, float eps,
                                   int norm_before_gate, int is_rms_norm, int x_dtype,
                                   int w_dtype, void* stream) {
  XOPS_REQUIRE(M >= 0 && N > 0, "layer_norm_fwd: bad shape M=%lld N=%lld", (long long)M,
               (long long)N);
  if (group_size <= 0) group_size = N;
  XOPS_REQUIRE(N % group_size == 0, "layer_norm_fwd: N=%lld not divisible by group_size=%lld",
               (long long)N, (long long)group_size);
  XOPS_REQUIRE(valid_dtype(x_dtype) && valid_dtype(w_dtype), "layer_norm_fwd: bad dtype");
  if (M == 0) return XOPS_OK;
  XOPS_REQUIRE(x && weight && y && rstd, "layer_norm_fwd: null pointer");
  XOPS_REQUIRE(is_rms_norm || mean, "layer_norm_fwd: LayerNorm needs a mean buffer");
  XOPS_REQUIRE(stride_x_row >= N && stride_y_row >= N && (!z || stride_z_row >= N),
               "layer_norm_fwd: row stride smaller than N");
  // vector loads need 16-byte aligned segments when the warp path is used
  const int xs = x_dtype == XOPS_F32 ? 4 : 2;
  const bool aligned = aligned16(x) && aligned16(y) && (!z || aligned16(z)) && aligned16(weight) &&
                       (!bias || aligned16(bias)) && (stride_x_row * xs) % 16 == 0 &&
                       (stride_y_row * xs) % 16 == 0 && (!z || (stride_z_row * xs) % 16 == 0);
  const int64_t G = aligned ? group_size : -1;  // -1 forces the scalar block path
  cudaStream_t st = (cudaStream_t)stream;
  const bool nbg = norm_before_gate != 0, rms = is_rms_norm != 0;
  auto run = [&](auto tx, auto tw) {
    using TX = decltype(tx);
    using TW = decltype(tw);
    if (G < 0) {
      // unaligned views: block kernel (scalar accesses)
      const int64_t ng = N / group_size;
      const bool hz = z != nullptr, hb = bias != nullptr;
#define XOPS_LNB(R, Z, B)                                                                    \
  if (rms == R && hz == Z && hb == B) {                                                      \
    layer_norm_block_kernel<TX, TW, R, Z, B><<<(unsigned)(M * ng), 256, 0, st>>>(            \
        (const TX*)x, (const TW*)weight, (const TW*)bias, (const TX*)z, (TX*)y, mean, rstd, M, \
        ng, group_size, stride_x_row, stride_z_row, stride_y_row, eps, nbg);                 \
    return check_launch("layer_norm_fwd");                                                   \
  }
      XOPS_LNB(true, true, true) XOPS_LNB(true, true, false) XOPS_LNB(true, false, true)
      XOPS_LNB(true, false, false) XOPS_LNB(false, true, true) XOPS_LNB(false, true, false)
      XOPS_LNB(false, false, true) XOPS_LNB(false, false, false)
#undef XOPS_LNB
      return (int)XOPS_ERR_UNSUPPORTED;
    }
    return dispatch_ln_flags<TX, TW>(x, weight, bias, z, y, mean, rstd, M, N, group_size,
                                     stride_x_row, stride_z_row, stride_y_row, eps, nbg, rms, st);
  };
  auto with_w = [&](auto tx) {
    switch (w_dtype) {
      case XOPS_F32: return run(tx, float{});
      case XOPS_BF16: return run(tx, __nv_bfloat16{});
      default: return run(tx, __half{});
    }
  };
  switch (x_dtype) {
    case XOPS_F32: return with_w(float{});
    case XOPS_BF16: return with_w(__nv_bfloat16{});
    default: return with_w(__half{});
  }
}

extern "C" int xops_gemma_rms_norm(const void* x, const void* gamma, void* y, float* rstd,
                                   int64_t rows, int64_t cols, float eps, int x_dtype,
                                   int gamma_dtype, void* stream) {
  XOPS_REQUIRE(rows >= 0 && cols > 0, "gemma_rms_norm: bad shape");
  XOPS_REQUIRE(valid_dtype(x_dtype) && valid_dtype(gamma_dtype), "gemma_rms_norm: bad dtype");
  if (rows == 0) return XOPS_OK;
  XOPS_REQUIRE(x && gamma && y && rstd, "gemma_rms_norm: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const bool aligned = aligned16(x) && aligned16(y) && aligned16(gamma);
  const int64_t n = aligned ? cols : -cols;
  auto run = [&](auto tx, auto tw) {
    using TX = decltype(tx);
    using TW = decltype(tw);
    if (n < 0) {
      gemma_block_kernel<TX, TW><<<(unsigned)rows, 512, 0, st>>>((const TX*)x, (const TW*)gamma,
                                                                 (TX*)y, rstd, cols, eps);
      return check_launch("gemma_rms_norm");
    }
    return dispatch_gemma<TX, TW>(x, gamma, y, rstd, rows, cols, eps, st);
  };
  auto with_w = [&](auto tx) {
    switch (gamma_dtype) {
      case XOPS_F32: return run(tx, float{});
      case XOPS_BF16: return run(tx, __nv_bfloat16{});
      default: return run(tx, __half{});
    }
  };
  switch (x_dtype) {
    case XOPS_F32: return with_w(float{});
    case XOPS_BF16: return with_w(__nv_bfloat16{});
    default: return with_w(__half{});
  }
}

extern "C" int xops_l2norm_last_dim(const void* x, void* y, int64_t rows, int64_t cols, float eps,
                                    int dtype, void* stream) {
  XOPS_REQUIRE(rows >= 0 && cols > 0, "l2norm_last_dim: bad shape");
  XOPS_REQUIRE(dtype == XOPS_F32 || dtype == XOPS_BF16, "l2norm_last_dim: dtype must be bf16/fp32");
  if (rows == 0) return XOPS_OK;
  XOPS_REQUIRE(x && y, "l2norm_last_dim: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const bool aligned = aligned16(x) && aligned16(y);
  const int64_t n = aligned ? cols : 1;  // 1 never matches a vector case
  if (dtype == XOPS_F32) {
    if (!aligned) {
      l2norm_generic_kernel<float><<<(unsigned)cdiv64(rows, 8), 256, 0, st>>>(
          (const float*)x, (float*)y, rows, cols, eps);
      return check_launch("l2norm_last_dim");
    }
    return dispatch_l2<float>(x, y, rows, cols, eps, st);
  }
  if (!aligned || n == 1) {
    l2norm_generic_kernel<__nv_bfloat16><<<(unsigned)cdiv64(rows, 8), 256, 0, st>>>(
        (const __nv_bfloat16*)x, (__nv_bfloat16*)y, rows, cols, eps);
    return check_launch("l2norm_last_dim");
  }
  return dispatch_l2<__nv_bfloat16>(x, y, rows, cols, eps, st);
}
