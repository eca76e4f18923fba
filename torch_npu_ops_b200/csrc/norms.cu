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
// Streaming path for 16-bit tensors with contiguous rows.  The (row, group)
// segments are then contiguous in memory, so a tile of whole segments of x
// (and z) is one contiguous range.  A persistent CTA streams tiles with 1-D
// bulk copies into a ring of RN_NS shared stages (warp 0 issues them) and 8
// consumer warps normalise from shared memory and store y with 16-byte
// stores, so the bytes in flight per SM do not depend on registers.
//
// One kernel family serves the three operators; KIND selects the statistics
// and the affine step:
//   LN     y = (x - mean) * rstd * w (+ b),  mean and rstd written
//   RMS    y = x * rstd * w (+ b),           rstd written
//   GEMMA  y = x * rstd * (1 + w),           rstd written (one group per row)
//   L2     y = x * rsqrt(sum x^2 + eps),     nothing else written
// with rstd = rsqrt(mean of squares (centred for LN) + eps) and the SiLU gate
// z * sigmoid(z) applied to x before the statistics or to y after them.
//
// Narrow segments (G <= 256): LPR = G / 8 lanes share one segment, one 16-byte
// piece each, shuffle reductions inside the lane group.
// Wide segments (256 < G <= 16384): one warp per segment, lane-strided 16-byte
// pieces, one pass over shared memory per statistic plus the output pass.
// ----------------------------------------------------------------------------
enum NormKind { K_LN = 0, K_RMS = 1, K_GEMMA = 2, K_L2 = 3 };
constexpr int RN_NS = 3, RN_TILE_BYTES = 16384, RN_NT = 32 + 256;
constexpr uint32_t RN_WAIT = 1u << 26;
__device__ int g_norm_error = 0;

// the affine step of one 8-element piece: v = xhat (already centred and
// scaled by rstd), w / b / gate per element
template <typename TW, int KIND, bool HAS_Z, bool HAS_B>
__device__ __forceinline__ void norm_affine(float2 (&v)[4], const TW* __restrict__ w,
                                            const TW* __restrict__ b, const float2 (&gz)[4],
                                            bool gate_after) {
  if constexpr (KIND == K_L2) return;
  float wv[8], bv[8];
  load_vec<TW, 8>(w, wv);
  if constexpr (HAS_B) load_vec<TW, 8>(b, bv);
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    float2 wu = make_float2(wv[2 * u], wv[2 * u + 1]);
    if constexpr (KIND == K_GEMMA) wu = fadd2(wu, make_float2(1.f, 1.f));
    v[u] = fmul2(v[u], wu);
    if constexpr (HAS_B) v[u] = fadd2(v[u], make_float2(bv[2 * u], bv[2 * u + 1]));
    if constexpr (HAS_Z) {
      if (gate_after) v[u] = fmul2(v[u], gz[u]);
    }
  }
}

template <typename TX>
__device__ __forceinline__ void unpack8(const uint4 r, float2 (&v)[4]) {
  v[0] = unpack2<TX>(r.x);
  v[1] = unpack2<TX>(r.y);
  v[2] = unpack2<TX>(r.z);
  v[3] = unpack2<TX>(r.w);
}
template <typename TX>
__device__ __forceinline__ uint4 pack8(const float2 (&v)[4]) {
  return make_uint4(pack2<TX>(v[0]), pack2<TX>(v[1]), pack2<TX>(v[2]), pack2<TX>(v[3]));
}
template <typename TX>
__device__ __forceinline__ void silu8(const uint4 r, float2 (&g)[4]) {
  g[0] = silu2_lowp(unpack2<TX>(r.x));
  g[1] = silu2_lowp(unpack2<TX>(r.y));
  g[2] = silu2_lowp(unpack2<TX>(r.z));
  g[3] = silu2_lowp(unpack2<TX>(r.w));
}

// Producer / ring bookkeeping shared by both widths.  Tiles hold SPT whole
// segments of G elements; tile t of the grid-strided sequence goes to stage
// k % RN_NS of the CTA that owns it.  x rows (ngroups segments each) are
// contiguous when sx == ngroups * G, which makes a tile one copy; otherwise
// each tile holds whole rows and takes one copy per row.
template <typename TX, bool HAS_Z>
__device__ __forceinline__ void norm_stream_produce(const TX* __restrict__ x,
                                                    const TX* __restrict__ z, unsigned char* sm,
                                                    uint64_t* full, uint64_t* empty,
                                                    int* abort_sh, int64_t total, int64_t G,
                                                    int64_t spt, int tile_bytes, int stage,
                                                    int64_t ngroups = 1, int64_t sx = -1,
                                                    int64_t sz = -1) {
  // strided rows (one copy per row of ngroups segments): x of the GDN q/k
  // L2 pre-pass, z of the gated norm read in place from the layer's
  // interleaved projection
  const bool strided = sx >= 0 && sx != ngroups * G;
  const bool zstrided = sz >= 0 && sz != ngroups * G;
  const int64_t tiles = (total + spt - 1) / spt;
  for (int64_t k = 0;; ++k) {
    const int64_t t = blockIdx.x + k * gridDim.x;
    if (t >= tiles) break;
    const int s = (int)(k % RN_NS);
    if (k >= RN_NS && !tc::mbar_wait(&empty[s], (uint32_t)((k / RN_NS - 1) & 1), RN_WAIT)) {
      atomicExch(&g_norm_error, 1);
      atomicExch(abort_sh, 1);
      break;
    }
    if (*(volatile int*)abort_sh) break;
    const int64_t s0 = t * spt;
    const int64_t n = total - s0 < spt ? total - s0 : spt;
    const uint32_t bytes = (uint32_t)(n * G * 2);
    unsigned char* st = sm + s * stage;
    tc::mbar_arrive_expect_tx(&full[s], (HAS_Z ? 2 : 1) * bytes);
    if (strided) {
      const uint32_t rb = (uint32_t)(ngroups * G * 2);
      for (int64_t r = 0; r < n / ngroups; ++r)
        tc::bulk_load(st + r * rb, x + (s0 / ngroups + r) * sx, rb, &full[s]);
    } else {
      tc::bulk_load(st, x + s0 * G, bytes, &full[s]);
    }
    if constexpr (HAS_Z) {
      if (zstrided) {
        const uint32_t rb = (uint32_t)(ngroups * G * 2);
        for (int64_t r = 0; r < n / ngroups; ++r)
          tc::bulk_load(st + tile_bytes + r * rb, z + (s0 / ngroups + r) * sz, rb, &full[s]);
      } else {
        tc::bulk_load(st + tile_bytes, z + s0 * G, bytes, &full[s]);
      }
    }
  }
}

template <typename TX, typename TW, int G, int KIND, bool HAS_Z, bool HAS_B>
__global__ void __launch_bounds__(RN_NT, 2) norm_stream_kernel(
    const TX* __restrict__ x, const TW* __restrict__ w, const TW* __restrict__ b,
    const TX* __restrict__ z, TX* __restrict__ y, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int64_t M, int64_t ngroups, int64_t sx, int64_t sz, float eps,
    bool norm_before_gate) {
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
    if (lane == 0)
      norm_stream_produce<TX, HAS_Z>(x, z, sm, full, empty, &abort_sh, total, G, SEGS,
                                     RN_TILE_BYTES, STAGE, ngroups, sx, sz);
    return;
  }
  const int cw = warp - 1, sub = lane / LPR, li = lane % LPR;
  constexpr float INV = KIND == K_L2 ? 1.0f : 1.0f / G;
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
      float2 xv[4], gz[4];
      unpack8<TX>(*reinterpret_cast<const uint4*>(st + si * (G * 2) + li * 16), xv);
      if constexpr (HAS_Z) {
        silu8<TX>(*reinterpret_cast<const uint4*>(st + RN_TILE_BYTES + si * (G * 2) + li * 16),
                  gz);
        if (!norm_before_gate) {
#pragma unroll
          for (int u = 0; u < 4; ++u) xv[u] = fmul2(xv[u], gz[u]);
        }
      }
      float mu = 0.f;
      if constexpr (KIND == K_LN) {
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
      const float rstd = rsqrtf(ss * INV + eps);
      if (live) {
        const uint32_t row = (uint32_t)(seg / ngroups), grp = (uint32_t)(seg - (int64_t)row * ngroups);
        if constexpr (KIND != K_L2) {
          if (li == 0) {
            rstd_out[(int64_t)grp * M + row] = rstd;
            if constexpr (KIND == K_LN) mean_out[(int64_t)grp * M + row] = mu;
          }
        }
        const float2 r2 = make_float2(rstd, rstd);
#pragma unroll
        for (int u = 0; u < 4; ++u) xv[u] = fmul2(xv[u], r2);
        norm_affine<TW, KIND, HAS_Z, HAS_B>(xv, KIND == K_L2 ? w : w + (int64_t)grp * G + li * 8,
                                            HAS_B ? b + (int64_t)grp * G + li * 8 : b, gz,
                                            norm_before_gate);
        *reinterpret_cast<uint4*>(y + seg * G + li * 8) = pack8<TX>(xv);
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[s]);
  }
}

// 8 weights (16 or 32 bytes) as fp32 pairs, from shared or global memory
template <typename TW>
__device__ __forceinline__ void lds_w8(const TW* p, float2 (&v)[4]) {
  if constexpr (sizeof(TW) == 2) {
    unpack8<TW>(*reinterpret_cast<const uint4*>(p), v);
  } else {
    const float4 a = reinterpret_cast<const float4*>(p)[0];
    const float4 c = reinterpret_cast<const float4*>(p)[1];
    v[0] = make_float2(a.x, a.y);
    v[1] = make_float2(a.z, a.w);
    v[2] = make_float2(c.x, c.y);
    v[3] = make_float2(c.z, c.w);
  }
}
template <typename TW>
__device__ __forceinline__ void ldg_w8(const TW* __restrict__ p, float2 (&v)[4]) {
  float f[8];
  load_vec<TW, 8>(p, f);
#pragma unroll
  for (int u = 0; u < 4; ++u) v[u] = make_float2(f[2 * u], f[2 * u + 1]);
}

// Wide segments: tiles of SPT = tile_bytes / (2G) whole segments; segment j
// of the CTA's stream (counted across its tiles) belongs to consumer warp
// j % 8, so every warp stays busy even when a tile holds fewer than 8
// segments.  A warp makes one pass over its segment in shared memory per
// statistic (mean for LN, the sum of squares) and one output pass; a gate
// applied before the statistics is recomputed in each pass rather than
// stored, which keeps the stage at 16-bit width.  The weight (and bias) rows,
// N = ngroups * G elements, are copied once per CTA into shared memory behind
// the ring when they fit (wsm), so the output pass never waits on L2 for them.
template <typename TX, typename TW, int KIND, bool HAS_Z, bool HAS_B>
__global__ void __launch_bounds__(RN_NT, 2) norm_wide_stream_kernel(
    const TX* __restrict__ x, const TW* __restrict__ w, const TW* __restrict__ b,
    const TX* __restrict__ z, TX* __restrict__ y, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int M, int ngroups, int G, int spt, int tile_bytes, bool wsm,
    float eps, bool norm_before_gate) {
  extern __shared__ unsigned char rn_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(rn_raw) + 127) & ~static_cast<uintptr_t>(127));
  __shared__ uint64_t full[RN_NS], empty[RN_NS];
  __shared__ int abort_sh;
  const int stage = (HAS_Z ? 2 : 1) * tile_bytes;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int N = ngroups * G;
  const int total = M * ngroups;
  const int tiles = (total + spt - 1) / spt;
  TW* sw = reinterpret_cast<TW*>(sm + RN_NS * stage);
  TW* sb = sw + N;
  if (tid == 0) {
    for (int s = 0; s < RN_NS; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 8);
    }
    tc::mbar_fence_init();
    abort_sh = 0;
  }
  if (KIND != K_L2 && wsm) {
    constexpr int VW = 16 / (int)sizeof(TW);
    for (int i = tid; i < N / VW; i += blockDim.x) {
      reinterpret_cast<uint4*>(sw)[i] = __ldg(reinterpret_cast<const uint4*>(w) + i);
      if constexpr (HAS_B) reinterpret_cast<uint4*>(sb)[i] = __ldg(reinterpret_cast<const uint4*>(b) + i);
    }
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0)
      norm_stream_produce<TX, HAS_Z>(x, z, sm, full, empty, &abort_sh, total, G, spt, tile_bytes,
                                     stage);
    return;
  }
  const int cw = warp - 1;
  const int nch = G >> 3;  // 16-byte pieces per segment
  const float inv = KIND == K_L2 ? 1.0f : 1.0f / (float)G;
  const bool gate_before = HAS_Z && !norm_before_gate;
  for (int k = 0;; ++k) {
    const int t = blockIdx.x + k * gridDim.x;
    if (t >= tiles) break;
    const int s = k % RN_NS;
    if (!tc::mbar_wait(&full[s], (uint32_t)((k / RN_NS) & 1), RN_WAIT)) {
      atomicExch(&g_norm_error, 1);
      break;
    }
    const unsigned char* st = sm + s * stage;
    const int s0 = t * spt;
    const int n = total - s0 < spt ? total - s0 : spt;
    // first segment of this tile that warp cw owns
    int i = (int)((cw - ((int64_t)k * spt) % 8 + 8) % 8);
    for (; i < n; i += 8) {
      const int seg = s0 + i;
      const uint4* xs = reinterpret_cast<const uint4*>(st + i * G * 2);
      const uint4* zs = reinterpret_cast<const uint4*>(st + tile_bytes + i * G * 2);
      auto load = [&](int c, float2 (&v)[4], float2 (&g)[4]) {
        unpack8<TX>(xs[c], v);
        if constexpr (HAS_Z) {
          silu8<TX>(zs[c], g);
          if (gate_before) {
#pragma unroll
            for (int u = 0; u < 4; ++u) v[u] = fmul2(v[u], g[u]);
          }
        }
      };
      float mu = 0.f;
      if constexpr (KIND == K_LN) {
        float2 a2 = make_float2(0.f, 0.f);
#pragma unroll 4
        for (int c = lane; c < nch; c += 32) {
          float2 v[4], g[4];
          load(c, v, g);
          a2 = fadd2(a2, fadd2(fadd2(v[0], v[1]), fadd2(v[2], v[3])));
        }
        mu = warp_sum(a2.x + a2.y) * inv;
      }
      const float2 m2 = make_float2(mu, mu);
      float2 q2 = make_float2(0.f, 0.f);
#pragma unroll 4
      for (int c = lane; c < nch; c += 32) {
        float2 v[4], g[4];
        load(c, v, g);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if constexpr (KIND == K_LN) v[u] = fsub2(v[u], m2);
          q2 = ffma2(v[u], v[u], q2);
        }
      }
      const float rstd = rsqrtf(warp_sum(q2.x + q2.y) * inv + eps);
      const int row = seg / ngroups, grp = seg - row * ngroups;
      if constexpr (KIND != K_L2) {
        if (lane == 0) {
          rstd_out[(int64_t)grp * M + row] = rstd;
          if constexpr (KIND == K_LN) mean_out[(int64_t)grp * M + row] = mu;
        }
      }
      const float2 r2 = make_float2(rstd, rstd);
      const TW* wg = (wsm ? sw : w) + grp * G;
      const TW* bg = (wsm ? sb : b) + (HAS_B ? grp * G : 0);
      uint4* yo = reinterpret_cast<uint4*>(y + (int64_t)seg * G);
#pragma unroll 2
      for (int c = lane; c < nch; c += 32) {
        float2 v[4], g[4], wv[4], bv[4];
        load(c, v, g);
        if constexpr (KIND != K_L2) {
          if (wsm) {
            lds_w8<TW>(wg + c * 8, wv);
            if constexpr (HAS_B) lds_w8<TW>(bg + c * 8, bv);
          } else {
            ldg_w8<TW>(wg + c * 8, wv);
            if constexpr (HAS_B) ldg_w8<TW>(bg + c * 8, bv);
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          if constexpr (KIND == K_LN) v[u] = fsub2(v[u], m2);
          v[u] = fmul2(v[u], r2);
          if constexpr (KIND == K_GEMMA) v[u] = ffma2(v[u], wv[u], v[u]);  // x (1 + w)
          if constexpr (KIND == K_LN || KIND == K_RMS) {
            if constexpr (HAS_B) v[u] = ffma2(v[u], wv[u], bv[u]);
            else v[u] = fmul2(v[u], wv[u]);
          }
          if constexpr (HAS_Z) {
            if (!gate_before) v[u] = fmul2(v[u], g[u]);
          }
        }
        yo[c] = pack8<TX>(v);
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[s]);
  }
}

// Few wide segments (decode-sized batches such as cfg4's [256, 2048]): one
// CTA per (row, group) segment, G / (8 VPT) threads each holding VPT 16-byte
// vectors, so every segment's bytes are in flight at once across the grid.
// Statistics are warp shuffles plus one shared-memory round per statistic.
// x and y rows may be strided (the segment is contiguous inside its row).
template <int NW>
__device__ __forceinline__ float block_sum(float v, float* red, int warp, int lane) {
  v = warp_sum(v);
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < NW ? red[lane] : 0.f;
  t = warp_sum(t);
  __syncthreads();  // red is reused by the next statistic
  return t;
}

template <typename TX, typename TW, int KIND, bool HAS_Z, bool HAS_B, int VPT, int NT>
__global__ void __launch_bounds__(NT) norm_rowblock_kernel(
    const TX* __restrict__ x, const TW* __restrict__ w, const TW* __restrict__ b,
    const TX* __restrict__ z, TX* __restrict__ y, float* __restrict__ mean_out,
    float* __restrict__ rstd_out, int64_t M, int64_t ngroups, int64_t sx, int64_t sz,
    int64_t sy, float eps, bool norm_before_gate) {
  constexpr int G = NT * VPT * 8;
  constexpr int NW = NT / 32;
  __shared__ float red[32];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t seg = blockIdx.x;
  const int64_t row = seg / ngroups, grp = seg - row * ngroups;
  const TX* xr = x + row * sx + grp * G;
  const TX* zr = HAS_Z ? z + row * sz + grp * G : nullptr;
  float2 v[VPT][4], gz[VPT][4];
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = (j * NT + tid) * 8;
    unpack8<TX>(__ldg(reinterpret_cast<const uint4*>(xr + c)), v[j]);
    if constexpr (HAS_Z) {
      silu8<TX>(__ldg(reinterpret_cast<const uint4*>(zr + c)), gz[j]);
      if (!norm_before_gate) {
#pragma unroll
        for (int u = 0; u < 4; ++u) v[j][u] = fmul2(v[j][u], gz[j][u]);
      }
    }
  }
  float mu = 0.f;
  if constexpr (KIND == K_LN) {
    float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
    for (int j = 0; j < VPT; ++j)
#pragma unroll
      for (int u = 0; u < 4; ++u) s2 = fadd2(s2, v[j][u]);
    mu = block_sum<NW>(s2.x + s2.y, red, warp, lane) * (1.0f / G);
#pragma unroll
    for (int j = 0; j < VPT; ++j)
#pragma unroll
      for (int u = 0; u < 4; ++u) v[j][u] = fsub2(v[j][u], make_float2(mu, mu));
  }
  float2 q2 = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < VPT; ++j)
#pragma unroll
    for (int u = 0; u < 4; ++u) q2 = ffma2(v[j][u], v[j][u], q2);
  const float ss = block_sum<NW>(q2.x + q2.y, red, warp, lane);
  const float rstd = rsqrtf(ss * (KIND == K_L2 ? 1.0f : 1.0f / G) + eps);
  if constexpr (KIND != K_L2) {
    if (tid == 0) {
      rstd_out[grp * M + row] = rstd;
      if constexpr (KIND == K_LN) mean_out[grp * M + row] = mu;
    }
  }
  const float2 r2 = make_float2(rstd, rstd);
  TX* yr = y + row * sy + grp * G;
#pragma unroll
  for (int j = 0; j < VPT; ++j) {
    const int c = (j * NT + tid) * 8;
    float2 wv[4], bv[4];
    if constexpr (KIND != K_L2) {
      ldg_w8<TW>(w + grp * G + c, wv);
      if constexpr (HAS_B) ldg_w8<TW>(b + grp * G + c, bv);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      float2 t = fmul2(v[j][u], r2);
      if constexpr (KIND == K_GEMMA) t = ffma2(t, wv[u], t);
      if constexpr (KIND == K_LN || KIND == K_RMS) {
        if constexpr (HAS_B) t = ffma2(t, wv[u], bv[u]);
        else t = fmul2(t, wv[u]);
      }
      if constexpr (HAS_Z) {
        if (norm_before_gate) t = fmul2(t, gz[j][u]);
      }
      v[j][u] = t;
    }
    *reinterpret_cast<uint4*>(yr + c) = pack8<TX>(v[j]);
  }
}

// G = 8 * VPT * NT for the (VPT, NT) pairs compiled: 512..8192
template <typename TX, typename TW, int KIND, bool HAS_Z, bool HAS_B>
int launch_norm_rowblock(const void* x, const void* w, const void* b, const void* z, void* y,
                         float* mean, float* rstd, int64_t M, int64_t ng, int64_t G, int64_t sx,
                         int64_t sz, int64_t sy, float eps, bool nbg, cudaStream_t st,
                         const char* what) {
#define XOPS_RB(VPT, NT)                                                                       \
  if (G == 8 * VPT * NT) {                                                                     \
    norm_rowblock_kernel<TX, TW, KIND, HAS_Z, HAS_B, VPT, NT><<<(unsigned)(M * ng), NT, 0, st>>>( \
        (const TX*)x, (const TW*)w, (const TW*)b, (const TX*)z, (TX*)y, mean, rstd, M, ng, sx,  \
        sz, sy, eps, nbg);                                                                     \
    return check_launch(what);                                                                 \
  }
  XOPS_RB(1, 64)
  XOPS_RB(1, 128)
  XOPS_RB(1, 256)
  XOPS_RB(2, 256)
  XOPS_RB(4, 256)
#undef XOPS_RB
  return -1;
}

int sm_count() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

template <typename TX, typename TW, int GG, int KIND, bool HAS_Z, bool HAS_B>
int launch_norm_stream(const void* x, const void* w, const void* b, const void* z, void* y,
                       float* mean, float* rstd, int64_t M, int64_t ng, float eps, bool nbg,
                       cudaStream_t st, const char* what, int64_t sx = -1, int64_t sz = -1) {
  constexpr int SEGS = RN_TILE_BYTES / (GG * 2);
  constexpr int SMEM = RN_NS * (HAS_Z ? 2 : 1) * RN_TILE_BYTES + 128;
  auto kern = norm_stream_kernel<TX, TW, GG, KIND, HAS_Z, HAS_B>;
  // two 96 KB CTAs fit the default carveout, which leaves L1 room for the
  // weight rows this kernel reads through it
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM) != cudaSuccess)
    return set_error(XOPS_ERR_CUDA, "%s: shared-memory attribute failed", what);
  const int64_t tiles = cdiv64(M * ng, SEGS);
  const unsigned grid = (unsigned)std::min<int64_t>(tiles, 2 * (int64_t)sm_count());
  kern<<<grid, RN_NT, SMEM, st>>>((const TX*)x, (const TW*)w, (const TW*)b, (const TX*)z, (TX*)y,
                                  mean, rstd, M, ng, sx, sz, eps, nbg);
  return check_launch(what);
}

// wide segments: 32 KB tiles per tensor (16 KB with a gate), three stages,
// two CTAs per SM; up to 16 KB of weight and bias rows staged behind the ring
constexpr int RN_WB_BYTES = 16384;
template <typename TX, typename TW, int KIND, bool HAS_Z, bool HAS_B>
int launch_norm_wide(const void* x, const void* w, const void* b, const void* z, void* y,
                     float* mean, float* rstd, int64_t M, int64_t ng, int64_t G, float eps,
                     bool nbg, cudaStream_t st, const char* what) {
  constexpr int TB = HAS_Z ? 16384 : 32768;
  const int64_t wb = KIND == K_L2 ? 0 : ng * G * (int64_t)sizeof(TW) * (HAS_B ? 2 : 1);
  const bool wsm = KIND != K_L2 && wb <= RN_WB_BYTES;
  const int smem = RN_NS * (HAS_Z ? 2 : 1) * TB + 128 + (wsm ? (int)wb : 0);
  const int spt = (int)(TB / (G * 2));
  auto kern = norm_wide_stream_kernel<TX, TW, KIND, HAS_Z, HAS_B>;
  if (!set_stream_smem(kern, RN_NS * (HAS_Z ? 2 : 1) * TB + 128 + RN_WB_BYTES))
    return set_error(XOPS_ERR_CUDA, "%s: shared-memory attribute failed", what);
  const int64_t tiles = cdiv64(M * ng, spt);
  const unsigned grid = (unsigned)std::min<int64_t>(tiles, 2 * (int64_t)sm_count());
  kern<<<grid, RN_NT, smem, st>>>((const TX*)x, (const TW*)w, (const TW*)b, (const TX*)z, (TX*)y,
                                  mean, rstd, (int)M, (int)ng, (int)G, spt, TB, wsm, eps, nbg);
  return check_launch(what);
}

// Streaming dispatch shared by the three operators.  Returns -1 when the
// shape is not a streaming shape (the caller then uses the register paths).
// Streaming needs 16-bit data, contiguous rows, 16-byte-aligned bases,
// G % 8 == 0 and enough bytes to fill a persistent grid.
template <typename TX, typename TW, int KIND, bool HAS_Z, bool HAS_B>
int dispatch_stream(const void* x, const void* w, const void* b, const void* z, void* y,
                    float* mean, float* rstd, int64_t M, int64_t N, int64_t G, float eps,
                    bool nbg, cudaStream_t st, const char* what, int64_t sz = -1) {
  if constexpr (sizeof(TX) != 2) {
    return -1;
  } else {
    const int64_t ng = N / G;
    const int64_t segs = M * ng;
    const bool zstr = HAS_Z && sz >= 0 && sz != N;  // z rows sz elements apart
    if (segs >= (int64_t(1) << 31) || G % 8 != 0) return -1;
    if (!aligned16(x) || !aligned16(y) || (HAS_Z && !aligned16(z))) return -1;
    if (KIND != K_L2 && !aligned16(w)) return -1;
    if (HAS_B && !aligned16(b)) return -1;
    // strided z: each tile must hold whole rows, and each row copy starts on 16 bytes
    if (zstr && (G > 256 || (RN_TILE_BYTES / (G * 2)) % ng != 0 || (sz * 2) % 16 != 0)) return -1;
    if (G <= 256) {
      if (segs < 8192) return -1;
      if (G == 64) return launch_norm_stream<TX, TW, 64, KIND, HAS_Z, HAS_B>(x, w, b, z, y, mean, rstd, M, ng, eps, nbg, st, what, -1, sz);
      if (G == 128) return launch_norm_stream<TX, TW, 128, KIND, HAS_Z, HAS_B>(x, w, b, z, y, mean, rstd, M, ng, eps, nbg, st, what, -1, sz);
      if (G == 256) return launch_norm_stream<TX, TW, 256, KIND, HAS_Z, HAS_B>(x, w, b, z, y, mean, rstd, M, ng, eps, nbg, st, what, -1, sz);
      return -1;
    }
    if (G > (HAS_Z ? 8192 : 16384)) return -1;
    if (segs * G * 2 < (int64_t(4) << 20))  // too small to fill a persistent grid
      return launch_norm_rowblock<TX, TW, KIND, HAS_Z, HAS_B>(x, w, b, z, y, mean, rstd, M, ng, G,
                                                              N, N, N, eps, nbg, st, what);
    return launch_norm_wide<TX, TW, KIND, HAS_Z, HAS_B>(x, w, b, z, y, mean, rstd, M, ng, G, eps,
                                                        nbg, st, what);
  }
}

template <typename TX, typename TW, bool RMS, bool HAS_Z, bool HAS_B>
int dispatch_ln(const void* x, const void* w, const void* b, const void* z, void* y, float* mean,
                float* rstd, int64_t M, int64_t N, int64_t G, int64_t sx, int64_t sz, int64_t sy,
                float eps, bool nbg, cudaStream_t st) {
  const int64_t ng = N / G;
  // streaming path: 16-bit, contiguous x and y rows (segments adjacent in
  // memory); z rows contiguous or strided
  if (sx == N && sy == N && (!HAS_Z || sz >= N)) {
    const int rc = dispatch_stream<TX, TW, RMS ? K_RMS : K_LN, HAS_Z, HAS_B>(
        x, w, b, z, y, mean, rstd, M, N, G, eps, nbg, st, "layer_norm_fwd", HAS_Z ? sz : -1);
    if (rc >= 0) return rc;
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

}  // namespace

int l2norm_rows_stream(const void* x, void* y, int64_t rows, int64_t heads, int64_t x_stride,
                       float eps, cudaStream_t st) {
  // rows of `heads` 128-element bf16 segments; a 16 KB tile holds 64
  // segments, which must be whole rows for the per-row copies
  constexpr int SEGS = RN_TILE_BYTES / (128 * 2);
  if (rows * heads < 8192 || rows * heads >= (int64_t(1) << 31) || SEGS % heads != 0) return -1;
  if (!aligned16(x) || !aligned16(y) || (x_stride * 2) % 16 != 0 || x_stride < heads * 128)
    return -1;
  return launch_norm_stream<__nv_bfloat16, __nv_bfloat16, 128, K_L2, false, false>(
      x, nullptr, nullptr, nullptr, y, nullptr, nullptr, rows, heads, eps, true, st,
      "l2norm(q/k)", x_stride);
}

int take_norm_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_norm_error, sizeof(int)) != cudaSuccess) return -1;
  const int zero = 0;
  cudaMemcpyToSymbol(g_norm_error, &zero, sizeof(int));
  return v;
}

namespace {
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
    const int rc = dispatch_stream<TX, TW, K_GEMMA, false, false>(
        x, gamma, nullptr, nullptr, y, nullptr, rstd, rows, cols, cols, eps, true, st,
        "gemma_rms_norm");
    if (rc >= 0) return rc;
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
  const int rc = dispatch_stream<__nv_bfloat16, __nv_bfloat16, K_L2, false, false>(
      x, nullptr, nullptr, nullptr, y, nullptr, nullptr, rows, cols, cols, eps, true, st,
      "l2norm_last_dim");
  if (rc >= 0) return rc;
  if (!aligned || n == 1) {
    l2norm_generic_kernel<__nv_bfloat16><<<(unsigned)cdiv64(rows, 8), 256, 0, st>>>(
        (const __nv_bfloat16*)x, (__nv_bfloat16*)y, rows, cols, eps);
    return check_launch("l2norm_last_dim");
  }
  return dispatch_l2<__nv_bfloat16>(x, y, rows, cols, eps, st);
}
