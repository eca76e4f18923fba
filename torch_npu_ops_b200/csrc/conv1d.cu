// Depthwise causal conv1d with SiLU: varlen prefill and decode update.
//
// Both are HBM-bound streaming kernels.  A thread owns VEC = 8 adjacent
// channels (one 16-byte bf16 vector per token), so consecutive threads read
// consecutive 16-byte pieces of a token row and every access is coalesced.
//
// Prefill (causal_conv1d_update_v2 with query_start_loc semantics,
// triton_npu/triton_src/test_causal_conv1d_update_v2.py:260-339, one
// sequence at a time): a CTA takes one tile of TILE_T consecutive tokens of
// one sequence; each thread slides its window of width-1 previous inputs
// down the tile in registers, so x is read once (plus width-1 halo rows per
// tile, which hit L2) and out written once.  The history before a
// sequence's first token comes from conv_state; the CTA that owns a
// sequence's first tile is the only one that reads or writes that state
// line, and it writes the final state straight from x, so no two CTAs race
// on a state line.
//
// Decode (causal_conv1d_update_ref, test_causal_conv1d_update.py:1158-1210;
// continuous-batching slot lookup and pad-slot skip as the decode kernels,
// :783-792): per (row, channel vector) read state + x, write out + state.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace xops {
namespace {

constexpr int VEC = 8;
constexpr int TILE_T = 64;
constexpr int MAXW = 8;

// Finds the sequence that owns flattened tile `tile` given per-sequence tile
// counts, by a linear scan over query_start_loc done cooperatively by the
// block (sequences are few; this is cheap next to the tile's traffic).
__device__ __forceinline__ void locate_tile(const int32_t* __restrict__ qsl, int nseq,
                                            int64_t tile, int* s_seq, int64_t* s_t0) {
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    int seq = -1;
    int64_t t0 = 0;
    for (int i = 0; i < nseq; ++i) {
      const int64_t s = qsl[i], e = qsl[i + 1];
      const int64_t n = e > s ? (e - s + TILE_T - 1) / TILE_T : 0;
      if (tile < acc + n) {
        seq = i;
        t0 = s + (tile - acc) * TILE_T;
        break;
      }
      acc += n;
    }
    *s_seq = seq;
    *s_t0 = t0;
  }
  __syncthreads();
}

template <typename T, int W>
__global__ void __launch_bounds__(128, 3) conv1d_varlen_kernel(
    const T* __restrict__ x, T* __restrict__ state, const T* __restrict__ weight,
    const T* __restrict__ bias, const int32_t* __restrict__ qsl,
    const int32_t* __restrict__ slots, T* __restrict__ out, int nseq, int64_t dim, bool silu,
    int32_t pad_slot) {
  __shared__ int s_seq;
  __shared__ int64_t s_t0;
  locate_tile(qsl, nseq, blockIdx.y, &s_seq, &s_t0);
  const int seq = s_seq;
  if (seq < 0) return;
  const int64_t c0 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * VEC;
  if (c0 >= dim) return;
  const int64_t sstart = qsl[seq], send = qsl[seq + 1];
  const int64_t t0 = s_t0;
  const int64_t t1 = min(t0 + (int64_t)TILE_T, send);
  const int line = slots ? slots[seq] : seq;
  if (slots && line == pad_slot) return;
  constexpr int H = W - 1;  // history length == state_len

  float w[VEC][W], b[VEC];
#pragma unroll
  for (int c = 0; c < VEC; ++c) {
#pragma unroll
    for (int j = 0; j < W; ++j) w[c][j] = to_f32<T>(weight[(c0 + c) * W + j]);
    b[c] = bias ? to_f32<T>(bias[c0 + c]) : 0.f;
  }
  // window: hist[j][c] = input at position t-H+j (j = 0 oldest)
  float hist[H > 0 ? H : 1][VEC];
  const bool first_tile = (t0 == sstart);
  T* st_line = state + ((int64_t)line * dim + c0) * H;
  float st_old[H > 0 ? H : 1][VEC];
  if (first_tile) {
#pragma unroll
    for (int c = 0; c < VEC; ++c)
#pragma unroll
      for (int j = 0; j < H; ++j) st_old[j][c] = to_f32<T>(st_line[c * H + j]);
#pragma unroll
    for (int j = 0; j < H; ++j)
#pragma unroll
      for (int c = 0; c < VEC; ++c) hist[j][c] = st_old[j][c];
  } else {
#pragma unroll
    for (int j = 0; j < H; ++j) {
      float tmp[VEC];
      load_vec<T, VEC>(x + (t0 - H + j) * dim + c0, tmp);
#pragma unroll
      for (int c = 0; c < VEC; ++c) hist[j][c] = tmp[c];
    }
  }
  // UNROLL token rows are loaded before any is consumed, so each thread keeps
  // UNROLL independent 16-byte loads in flight.
  // (kept as raw 16-byte words until used, so the batch costs 4 registers
  // per bf16 row instead of 8).
  constexpr int UNROLL = 8;
  constexpr int RW = VEC * (int)sizeof(T) / 16;
  for (int64_t tb = t0; tb < t1; tb += UNROLL) {
    uint4 raw[UNROLL][RW];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u)
      if (tb + u < t1) {
        const uint4* src = reinterpret_cast<const uint4*>(x + (tb + u) * dim + c0);
#pragma unroll
        for (int r = 0; r < RW; ++r) raw[u][r] = __ldg(src + r);
      }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      if (tb + u >= t1) break;
      float cur_u[VEC];
      {
        const T* e = reinterpret_cast<const T*>(raw[u]);
#pragma unroll
        for (int c = 0; c < VEC; ++c) cur_u[c] = to_f32<T>(e[c]);
      }
      float o[VEC];
#pragma unroll
      for (int c = 0; c < VEC; ++c) {
        float acc = b[c];
#pragma unroll
        for (int j = 0; j < H; ++j) acc = fmaf(hist[j][c], w[c][j], acc);
        acc = fmaf(cur_u[c], w[c][H], acc);
        o[c] = silu ? silu_f(acc) : acc;
      }
      store_vec<T, VEC>(out + (tb + u) * dim + c0, o);
#pragma unroll
      for (int j = 0; j + 1 < H; ++j)
#pragma unroll
        for (int c = 0; c < VEC; ++c) hist[j][c] = hist[j + 1][c];
      if constexpr (H > 0) {
#pragma unroll
        for (int c = 0; c < VEC; ++c) hist[H - 1][c] = cur_u[c];
      }
    }
  }
  if (first_tile) {
    // final state = last H entries of cat(old_state, x_seq), read from x
    const int64_t len = send - sstart;
    float nst[H > 0 ? H : 1][VEC];
#pragma unroll
    for (int j = 0; j < H; ++j) {
      const int64_t pos = len - H + j;  // position in cat coords relative to seq start
      if (pos >= 0) {
        float tmp[VEC];
        load_vec<T, VEC>(x + (sstart + pos) * dim + c0, tmp);
#pragma unroll
        for (int c = 0; c < VEC; ++c) nst[j][c] = tmp[c];
      } else {
#pragma unroll
        for (int c = 0; c < VEC; ++c) nst[j][c] = st_old[H + pos][c];
      }
    }
#pragma unroll
    for (int c = 0; c < VEC; ++c)
#pragma unroll
      for (int j = 0; j < H; ++j) st_line[c * H + j] = from_f32<T>(nst[j][c]);
  }
}

// Decode: one thread per (row, channel vector); general seqlen/state_len.
template <typename T, int W>
__global__ void __launch_bounds__(256) conv1d_update_kernel(
    const T* __restrict__ x, T* __restrict__ state, const T* __restrict__ weight,
    const T* __restrict__ bias, const int32_t* __restrict__ slots, T* __restrict__ out,
    int64_t batch, int64_t dim, int64_t seqlen, int64_t state_len, int64_t sxb, int64_t sxd,
    int64_t sxt, bool silu, int32_t pad_slot) {
  const int64_t nvec = dim / VEC;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= batch * nvec) return;
  const int64_t row = gid / nvec;
  const int64_t c0 = (gid - row * nvec) * VEC;
  const int line = slots ? slots[row] : (int)row;
  if (slots && line == pad_slot) return;
  T* st = state + ((int64_t)line * dim + c0) * state_len;
  for (int c = 0; c < VEC; ++c) {
    const int64_t ch = c0 + c;
    float wv[W];
#pragma unroll
    for (int j = 0; j < W; ++j) wv[j] = to_f32<T>(weight[ch * W + j]);
    const float bv = bias ? to_f32<T>(bias[ch]) : 0.f;
    T* s = st + (int64_t)c * state_len;
    // cat = [s_0 .. s_{L-1}, x_0 .. x_{n-1}]; out_t uses cat[L + t - (W-1) .. L + t]
    for (int64_t t = 0; t < seqlen; ++t) {
      float acc = bv;
#pragma unroll
      for (int j = 0; j < W; ++j) {
        const int64_t p = state_len + t - (W - 1) + j;
        const float val = p < state_len ? to_f32<T>(s[p])
                                        : to_f32<T>(x[row * sxb + ch * sxd + (p - state_len) * sxt]);
        acc = fmaf(val, wv[j], acc);
      }
      out[(row * dim + ch) * seqlen + t] = from_f32<T>(silu ? silu_f(acc) : acc);
    }
    // state <- last state_len entries of cat
    const int64_t total = state_len + seqlen;
    for (int64_t j = 0; j < state_len; ++j) {
      const int64_t p = total - state_len + j;
      const float val = p < state_len ? to_f32<T>(s[p])
                                      : to_f32<T>(x[row * sxb + ch * sxd + (p - state_len) * sxt]);
      s[j] = from_f32<T>(val);
    }
  }
}

// Decode fast path (width 4, state_len 3, seqlen 1): vectorised state/x/w.
template <typename T>
__global__ void __launch_bounds__(256) conv1d_decode_w4_kernel(
    const T* __restrict__ x, T* __restrict__ state, const T* __restrict__ weight,
    const T* __restrict__ bias, const int32_t* __restrict__ slots, T* __restrict__ out,
    int64_t batch, int64_t dim, int64_t sxb, bool silu, int32_t pad_slot) {
  const int64_t nvec = dim / VEC;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (gid >= batch * nvec) return;
  const int64_t row = gid / nvec;
  const int64_t c0 = (gid - row * nvec) * VEC;
  const int line = slots ? slots[row] : (int)row;
  if (slots && line == pad_slot) return;
  float xs[VEC], st[3 * VEC], w[4 * VEC], o[VEC];
  load_vec<T, VEC>(x + row * sxb + c0, xs);
  T* sp = state + ((int64_t)line * dim + c0) * 3;
  load_vec<T, 3 * VEC>(sp, st);
  load_vec<T, 4 * VEC>(weight + c0 * 4, w);
#pragma unroll
  for (int c = 0; c < VEC; ++c) {
    float acc = bias ? to_f32<T>(bias[c0 + c]) : 0.f;
    acc = fmaf(st[3 * c + 0], w[4 * c + 0], acc);
    acc = fmaf(st[3 * c + 1], w[4 * c + 1], acc);
    acc = fmaf(st[3 * c + 2], w[4 * c + 2], acc);
    acc = fmaf(xs[c], w[4 * c + 3], acc);
    o[c] = silu ? silu_f(acc) : acc;
  }
  store_vec<T, VEC>(out + row * dim + c0, o);
  float ns[3 * VEC];
#pragma unroll
  for (int c = 0; c < VEC; ++c) {
    ns[3 * c + 0] = st[3 * c + 1];
    ns[3 * c + 1] = st[3 * c + 2];
    ns[3 * c + 2] = xs[c];
  }
  store_vec<T, 3 * VEC>(sp, ns);
}

// The same for 16-bit types, two batch rows per thread: the weights and bias
// of the thread's 8 channels are read once and held packed, and both rows'
// x and state loads are issued before any arithmetic, so each thread keeps
// 128 bytes in flight (three CTAs per SM, twice the per-row kernel's).  The
// arithmetic is the per-row kernel's, in the same order.
template <typename T>
__global__ void __launch_bounds__(256, 3) conv1d_decode_w4_rows_kernel(
    const T* __restrict__ x, T* __restrict__ state, const T* __restrict__ weight,
    const T* __restrict__ bias, const int32_t* __restrict__ slots, T* __restrict__ out,
    int64_t batch, int64_t dim, int64_t sxb, bool silu, int32_t pad_slot) {
  static_assert(sizeof(T) == 2, "16-bit types only");
  constexpr int R = 2;
  const int64_t nvec = dim / VEC;
  const int64_t gid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int64_t rb = gid / nvec;
  if (rb * R >= batch) return;
  const int64_t c0 = (gid - rb * nvec) * VEC;
  uint4 wv[4];
#pragma unroll
  for (int q = 0; q < 4; ++q) wv[q] = __ldg(reinterpret_cast<const uint4*>(weight + c0 * 4) + q);
  const uint4 bv = bias ? __ldg(reinterpret_cast<const uint4*>(bias + c0)) : make_uint4(0, 0, 0, 0);
  uint4 xv[R], sv[R][3];
  T* sp[R];
  bool on[R];
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const int64_t row = rb * R + r;
    const int line = row < batch ? (slots ? slots[row] : (int)row) : pad_slot;
    on[r] = row < batch && !(slots && line == pad_slot);
    sp[r] = state + ((int64_t)(on[r] ? line : 0) * dim + c0) * 3;
    if (on[r]) {
      xv[r] = *reinterpret_cast<const uint4*>(x + row * sxb + c0);
#pragma unroll
      for (int q = 0; q < 3; ++q) sv[r][q] = reinterpret_cast<const uint4*>(sp[r])[q];
    }
  }
  auto word = [](const uint4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; };
  // element e of a packed vector array (8 bf16 per uint4)
  auto elem = [&](const uint4* v, int e) {
    const float2 p = unpack2<T>(word(v[e >> 3], (e >> 1) & 3));
    return (e & 1) ? p.y : p.x;
  };
#pragma unroll
  for (int r = 0; r < R; ++r) {
    if (!on[r]) continue;
    // outputs and the shifted state are packed as they are formed
    uint32_t ow[VEC / 2];
#pragma unroll
    for (int m = 0; m < VEC / 2; ++m) {
      float oo[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int c = 2 * m + hh;
        float acc = bias ? elem(&bv, c) : 0.f;
        acc = fmaf(elem(sv[r], 3 * c + 0), elem(wv, 4 * c + 0), acc);
        acc = fmaf(elem(sv[r], 3 * c + 1), elem(wv, 4 * c + 1), acc);
        acc = fmaf(elem(sv[r], 3 * c + 2), elem(wv, 4 * c + 2), acc);
        acc = fmaf(elem(&xv[r], c), elem(wv, 4 * c + 3), acc);
        oo[hh] = silu ? silu_f(acc) : acc;
      }
      ow[m] = pack2<T>(make_float2(oo[0], oo[1]));
    }
    *reinterpret_cast<uint4*>(out + (rb * R + r) * dim + c0) = make_uint4(ow[0], ow[1], ow[2], ow[3]);
    // new state element e: the old element e + 1, or x for the last tap
    uint32_t nw[3 * VEC / 2];
#pragma unroll
    for (int k = 0; k < 3 * VEC / 2; ++k) {
      float a[2];
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int e = 2 * k + hh;
        a[hh] = (e % 3 == 2) ? elem(&xv[r], e / 3) : elem(sv[r], e + 1);
      }
      nw[k] = pack2<T>(make_float2(a[0], a[1]));
    }
#pragma unroll
    for (int q = 0; q < 3; ++q)
      reinterpret_cast<uint4*>(sp[r])[q] =
          make_uint4(nw[4 * q], nw[4 * q + 1], nw[4 * q + 2], nw[4 * q + 3]);
  }
}

// ----------------------------------------------------------------------------
// Prefill for 16-bit inputs, TMA-fed.  A persistent CTA walks tiles of
// RB_T = 64 tokens x RB_C = 256 channels (one sequence per tile).  Warp 0
// streams each tile plus its W-1 halo rows into a ring of RB_NS shared
// stages with one TMA box per tile, so the loads in flight per SM do not
// depend on registers (three CTAs per SM keep six tiles in flight); warps
// 1-8 slide the window over 16 of the tile's tokens for 4 channels per lane
// (8-byte shared reads, coalesced 8-byte global writes; a warp covers 128
// channels).  The halo of a sequence's first tile comes from conv_state,
// and the lanes that read a state line are the ones that write its final
// value, as in the per-thread kernel above.
// ----------------------------------------------------------------------------
// A slab of RB_C channels arrives as one box of a plain input, or as two
// boxes of RB_B channels, each at its 128-channel block's place in the GDN
// layer's interleaved projection mixed_qkvz (QkvzMap): the conv then reads
// the projection output directly and the de-interleave pass disappears.
constexpr int RB_T = 64, RB_C = 256, RB_B = 128, RB_NS = 2, RB_STAGE = 35840;  // (64 + 5) rows x 512 B, rounded
constexpr int RB_NT = 32 + 256;
constexpr int RB_CV = 4;  // channels per consumer lane
constexpr int RB_SMEM = RB_NS * RB_STAGE + 1024;
constexpr uint32_t RB_WAIT = 1u << 26;

// Source column of conv channel c.  nqk == 0: c.  Otherwise the input is
// mixed_qkvz [T, nqk * group] with, per key head i, q (128) | k (128) |
// v (r value heads x 128) | z (r x 128) (fused_qkvzba_split_reshape_cat,
// triton_npu/triton_src/test_fused_qkvzba_split_reshape.py:463-507), and
// the conv channels are all q heads, then all k heads, then all v heads.
struct QkvzMap {
  int nqk, r;
  int64_t group;
};
__device__ __forceinline__ int64_t qkvz_col(const QkvzMap& m, int64_t c) {
  if (m.nqk == 0) return c;
  const int64_t blk = c >> 7, in = c & 127;
  if (blk < m.nqk) return blk * m.group + in;
  if (blk < 2 * m.nqk) return (blk - m.nqk) * m.group + 128 + in;
  const int64_t j = blk - 2 * m.nqk;
  return (j / m.r) * m.group + 256 + (j % m.r) * 128 + in;
}

struct RbTile {
  int64_t t0, sstart, send;
  int seq, line, slab;
};

__device__ __forceinline__ void rb_mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(bar)), "r"(count));
}
__device__ __forceinline__ bool rb_mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = (uint32_t)__cvta_generic_to_shared(bar);
  for (uint32_t i = 0; i < RB_WAIT; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok) : "r"(a), "r"(parity) : "memory");
    if (ok) return true;
  }
  return false;
}
__device__ __forceinline__ void rb_mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];\n" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(bar)) : "memory");
}
__device__ __forceinline__ void rb_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;\n" ::"r"(
                   (uint32_t)__cvta_generic_to_shared(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void rb_tma_load(void* dst, const void* tmap, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"((uint32_t)__cvta_generic_to_shared(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(x), "r"(y),
      "r"((uint32_t)__cvta_generic_to_shared(bar)) : "memory");
}

__device__ int g_conv_error = 0;

template <typename T, int W, bool MAP>
__global__ void __launch_bounds__(RB_NT, 3) conv1d_varlen_tma_kernel(
    const __grid_constant__ CUtensorMap xmap, const T* __restrict__ x, T* __restrict__ state,
    const T* __restrict__ weight, const T* __restrict__ bias, const int32_t* __restrict__ qsl,
    const int32_t* __restrict__ slots, T* __restrict__ out, int nseq, int64_t dim,
    int64_t tiles_per_slab, int64_t total_tiles, int box_c, bool silu, int32_t pad_slot,
    int64_t l2_channels, float l2_eps, int64_t x_ld, QkvzMap cm) {
  constexpr int H = W - 1;
  extern __shared__ unsigned char rb_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(rb_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ uint64_t full[RB_NS], empty[RB_NS];
  __shared__ RbTile info[RB_NS];
  __shared__ int abort_sh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < RB_NS; ++s) {
      rb_mbar_init(&full[s], 1);
      rb_mbar_init(&empty[s], 8);
    }
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
    abort_sh = 0;
  }
  __syncthreads();
  auto fail = [&]() {
    atomicExch(&g_conv_error, 1);
    atomicExch(&abort_sh, 1);
  };
  if (warp == 0) {
    if (lane == 0) {
      for (int64_t k = 0;; ++k) {
        const int64_t idx = blockIdx.x + k * gridDim.x;
        if (idx >= total_tiles) break;
        const int s = (int)(k % RB_NS);
        if (k >= RB_NS && !rb_mbar_wait(&empty[s], (uint32_t)((k / RB_NS - 1) & 1))) {
          fail();
          break;
        }
        if (*(volatile int*)&abort_sh) break;
        RbTile ti;
        ti.slab = (int)(idx / tiles_per_slab);
        int64_t r = idx - (int64_t)ti.slab * tiles_per_slab, acc = 0;
        ti.seq = -1;
        ti.t0 = ti.sstart = ti.send = 0;
        for (int i = 0; i < nseq; ++i) {
          const int64_t a = qsl[i], e = qsl[i + 1];
          const int64_t n = e > a ? (e - a + RB_T - 1) / RB_T : 0;
          if (r < acc + n) {
            ti.seq = i;
            ti.sstart = a;
            ti.send = e;
            ti.t0 = a + (r - acc) * RB_T;
            break;
          }
          acc += n;
        }
        ti.line = ti.seq >= 0 ? (slots ? slots[ti.seq] : ti.seq) : 0;
        info[s] = ti;
        if (ti.seq < 0) {  // past the slab's last tile (the count is an upper bound)
          rb_mbar_arrive(&full[s]);
          continue;
        }
        const int64_t ch0 = (int64_t)ti.slab * RB_C;
        if constexpr (MAP) {
          // two 128-channel boxes, one per head block, at their projection columns
          const int nb = ch0 + box_c < dim ? 2 : 1;
          rb_expect_tx(&full[s], (uint32_t)(nb * (RB_T + H) * box_c * sizeof(T)));
          for (int bb = 0; bb < nb; ++bb)
            rb_tma_load(sm + s * RB_STAGE + bb * (RB_T + H) * box_c * (int)sizeof(T), &xmap,
                        (int)qkvz_col(cm, ch0 + bb * box_c), (int)(ti.t0 - H), &full[s]);
        } else {
          rb_expect_tx(&full[s], (uint32_t)((RB_T + H) * box_c * sizeof(T)));
          rb_tma_load(sm + s * RB_STAGE, &xmap, (int)ch0, (int)(ti.t0 - H), &full[s]);
        }
      }
    }
    return;
  }
  // consumers: warp pair = 16-token group; lane = 4 channels as two fp32
  // pairs, so the taps and the SiLU run as packed f32x2 instructions
  const int cw = warp - 1, tg = cw >> 1, quad = (cw & 1) * 32 + lane;
  int cur_slab = -1;
  float2 w[2][W], b[2];
  for (int64_t k = 0;; ++k) {
    const int64_t idx = blockIdx.x + k * gridDim.x;
    if (idx >= total_tiles) break;
    const int s = (int)(k % RB_NS);
    if (!rb_mbar_wait(&full[s], (uint32_t)((k / RB_NS) & 1))) {
      fail();
      break;
    }
    const RbTile ti = info[s];
    const int64_t c0 = (int64_t)ti.slab * RB_C + quad * RB_CV;
    const bool live = ti.seq >= 0 && c0 < dim && !(slots && ti.line == pad_slot);
    if (live) {
      if (ti.slab != cur_slab) {
        cur_slab = ti.slab;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
#pragma unroll
          for (int j = 0; j < W; ++j)
            w[p][j] = make_float2(to_f32<T>(weight[(c0 + 2 * p) * W + j]),
                                  to_f32<T>(weight[(c0 + 2 * p + 1) * W + j]));
          b[p] = bias ? make_float2(to_f32<T>(bias[c0 + 2 * p]), to_f32<T>(bias[c0 + 2 * p + 1]))
                      : make_float2(0.f, 0.f);
        }
      }
      // channel quad * 4 of the slab: with the map, in box quad * 4 / 128
      const int rstride = box_c * 2;
      const int qb = MAP ? quad * RB_CV / RB_B : 0, qin = quad * RB_CV - qb * RB_B;
      const unsigned char* stg = sm + s * RB_STAGE + qb * (RB_T + H) * rstride + qin * 2 +
                                 tg * 16 * rstride;
      float2 hist[H > 0 ? H : 1][2];
      const bool first = ti.t0 == ti.sstart && tg == 0;
      T* st_line = state + ((int64_t)ti.line * dim + c0) * H;
      if (first) {
#pragma unroll
        for (int j = 0; j < H; ++j)
#pragma unroll
          for (int p = 0; p < 2; ++p)
            hist[j][p] = make_float2(to_f32<T>(st_line[(2 * p) * H + j]),
                                     to_f32<T>(st_line[(2 * p + 1) * H + j]));
      } else {
#pragma unroll
        for (int j = 0; j < H; ++j) {
          const uint2 raw = *reinterpret_cast<const uint2*>(stg + j * rstride);
          hist[j][0] = unpack2<T>(raw.x);
          hist[j][1] = unpack2<T>(raw.y);
        }
      }
      const int64_t tb = ti.t0 + tg * 16;
      const int64_t nvalid = ti.send - tb;  // tokens of this group inside the sequence
      T* dst = out + tb * dim + c0;
      // the warp's 128 channels are one q or k head of the GDN layer: its
      // output row is L2-normalised (x / sqrt(sum x^2 + eps) over the head,
      // from the rounded conv output, as the separate l2norm pass would do)
      const bool l2 = c0 < l2_channels;
      // tokens in pairs: the two rows' sums of squares reduce across the
      // warp together, so their shuffle latencies overlap
#pragma unroll
      for (int ug = 0; ug < 16; ug += 2) {
        uint2 packed[2];
#pragma unroll
        for (int du = 0; du < 2; ++du) {
          const int u = ug + du;
          const uint2 raw = *reinterpret_cast<const uint2*>(stg + (H + u) * rstride);
          float2 cur[2] = {unpack2<T>(raw.x), unpack2<T>(raw.y)};
          uint32_t* pk = &packed[du].x;
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            float2 a = b[p];
#pragma unroll
            for (int j = 0; j < H; ++j) a = ffma2(hist[j][p], w[p][j], a);
            a = ffma2(cur[p], w[p][H], a);
            pk[p] = pack2<T>(silu ? silu2_lowp(a) : a);
          }
#pragma unroll
          for (int j = 0; j + 1 < H; ++j) {
            hist[j][0] = hist[j + 1][0];
            hist[j][1] = hist[j + 1][1];
          }
          if constexpr (H > 0) {
            hist[H - 1][0] = cur[0];
            hist[H - 1][1] = cur[1];
          }
        }
        if (l2) {
          float ss[2];
#pragma unroll
          for (int du = 0; du < 2; ++du) {
            const float2 r0 = unpack2<T>(packed[du].x), r1 = unpack2<T>(packed[du].y);
            ss[du] = r0.x * r0.x + r0.y * r0.y + r1.x * r1.x + r1.y * r1.y;
          }
          // two sums in six shuffles: the first exchange leaves token 0's
          // partial sums in lanes 0-15 and token 1's in lanes 16-31, each
          // half reduces its own, and one exchange hands every lane both
          const bool hi = lane & 16;
          float keep = hi ? ss[1] : ss[0];
          keep += __shfl_xor_sync(0xffffffffu, hi ? ss[0] : ss[1], 16);
#pragma unroll
          for (int o = 8; o > 0; o >>= 1) keep += __shfl_xor_sync(0xffffffffu, keep, o);
          const float other = __shfl_xor_sync(0xffffffffu, keep, 16);
          ss[0] = hi ? other : keep;
          ss[1] = hi ? keep : other;
#pragma unroll
          for (int du = 0; du < 2; ++du) {
            const float rn = rsqrtf(ss[du] + l2_eps);
            const float2 r0 = unpack2<T>(packed[du].x), r1 = unpack2<T>(packed[du].y);
            packed[du].x = pack2<T>(make_float2(r0.x * rn, r0.y * rn));
            packed[du].y = pack2<T>(make_float2(r1.x * rn, r1.y * rn));
          }
        }
#pragma unroll
        for (int du = 0; du < 2; ++du)
          if (ug + du < nvalid) *reinterpret_cast<uint2*>(dst + (int64_t)(ug + du) * dim) = packed[du];
      }
      if (first) {
        // final state = last H entries of cat(old_state, x_seq).  Entry j
        // reads old-state index len + j > j when it comes from the old state,
        // so writing index j in increasing order never clobbers a later read.
        const int64_t len = ti.send - ti.sstart;
#pragma unroll
        for (int j = 0; j < H; ++j) {
          const int64_t pos = len - H + j;
          float v[RB_CV];
          if (pos >= 0) {
            load_vec<T, RB_CV>(x + (ti.sstart + pos) * x_ld + (MAP ? qkvz_col(cm, c0) : c0), v);
          } else {
#pragma unroll
            for (int c = 0; c < RB_CV; ++c) v[c] = to_f32<T>(st_line[c * H + H + pos]);
          }
#pragma unroll
          for (int c = 0; c < RB_CV; ++c) st_line[c * H + j] = from_f32<T>(v[c]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) rb_mbar_arrive(&empty[s]);
  }
}

// cuTensorMapEncodeTiled through the runtime's driver entry point.
static PFN_cuTensorMapEncodeTiled_v12000 conv_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      p = nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

template <typename T>
int launch_varlen_tma(int W, const void* x, void* state, const void* w, const void* b,
                      const int32_t* qsl, const int32_t* slots, void* out, int nseq,
                      int64_t total, int64_t dim, bool silu, int32_t pad, cudaStream_t st,
                      int64_t l2_channels = 0, float l2_eps = 0.f, int64_t x_ld = 0,
                      QkvzMap cm = QkvzMap{0, 1, 0}) {
  auto enc = conv_map_encoder();
  if (!enc) return set_error(XOPS_ERR_CUDA, "causal_conv1d_varlen: cuTensorMapEncodeTiled is unavailable");
  if (x_ld == 0) x_ld = dim;
  CUtensorMap m;
  // the map spans the source rows: the channels, or the projection's columns
  const int64_t src_cols = cm.nqk ? cm.nqk * cm.group : dim;
  cuuint64_t dims[2] = {(cuuint64_t)src_cols, (cuuint64_t)total};
  cuuint64_t strides[1] = {(cuuint64_t)(x_ld * (int64_t)sizeof(T))};
  // box width: a slab (plain input) or a 128-channel head block; dim is a multiple of 8
  const int box_c = (int)std::min<int64_t>(dim, cm.nqk ? RB_B : RB_C);
  cuuint32_t box[2] = {(cuuint32_t)box_c, (cuuint32_t)(RB_T + W - 1)};
  cuuint32_t es[2] = {1, 1};
  const CUresult r = enc(&m, sizeof(T) == 2 ? (std::is_same<T, __half>::value
                                                   ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16
                                                   : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16)
                                              : CU_TENSOR_MAP_DATA_TYPE_FLOAT32,
                         2, const_cast<void*>(x), dims, strides, box, es,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(XOPS_ERR_CUDA, "causal_conv1d_varlen: tensor map encoding failed (%d)", (int)r);
  // exact tile count per channel slab: sum over sequences of ceil(len / RB_T)
  // is bounded by total / RB_T + nseq; the kernel maps tiles exactly from
  // query_start_loc, so the bound only sizes the slab stride
  const int64_t tiles_per_slab = total / RB_T + nseq;
  const int64_t slabs = (dim + RB_C - 1) / RB_C;
  const int64_t total_tiles = slabs * tiles_per_slab;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // three persistent CTAs per SM (72 KB each): the consumer warps are
  // latency-bound, so the third CTA's warps fill issue slots (cfg5: 0.50 ->
  // 0.44 ms against two per SM)
  const unsigned grid = (unsigned)std::min<int64_t>(total_tiles, 3 * (int64_t)sms);
  switch (W) {
#define XOPS_CT(WW)                                                                            \
  case WW: {                                                                                   \
    auto kern = cm.nqk ? conv1d_varlen_tma_kernel<T, WW, true>                                 \
                       : conv1d_varlen_tma_kernel<T, WW, false>;                               \
    if (!set_stream_smem(kern, RB_SMEM))                                                        \
      return set_error(XOPS_ERR_CUDA, "causal_conv1d_varlen: shared-memory attribute failed"); \
    kern<<<grid, RB_NT, RB_SMEM, st>>>(m, (const T*)x, (T*)state, (const T*)w, (const T*)b,    \
                                       qsl, slots, (T*)out, nseq, dim, tiles_per_slab,          \
                                       total_tiles, box_c, silu, pad, l2_channels, l2_eps,      \
                                       x_ld, cm);                                               \
    return check_launch("causal_conv1d_varlen");                                               \
  }
    XOPS_CT(2) XOPS_CT(3) XOPS_CT(4) XOPS_CT(5) XOPS_CT(6)
#undef XOPS_CT
    default:
      return set_error(XOPS_ERR_UNSUPPORTED, "causal_conv1d_varlen: width %d not in [2, 6]", W);
  }
}

template <typename T>
int launch_varlen_w(int W, const void* x, void* state, const void* w, const void* b,
                    const int32_t* qsl, const int32_t* slots, void* out, int nseq,
                    int64_t tiles, int64_t dim, bool silu, int32_t pad, cudaStream_t st) {
  const int threads = 128;
  dim3 grid((unsigned)cdiv64(dim / VEC, threads), (unsigned)tiles);
  switch (W) {
#define XOPS_CV(WW)                                                                           \
  case WW:                                                                                    \
    conv1d_varlen_kernel<T, WW><<<grid, threads, 0, st>>>((const T*)x, (T*)state, (const T*)w, \
                                                         (const T*)b, qsl, slots, (T*)out,    \
                                                         nseq, dim, silu, pad);               \
    return check_launch("causal_conv1d_varlen");
    XOPS_CV(2) XOPS_CV(3) XOPS_CV(4) XOPS_CV(5) XOPS_CV(6)
#undef XOPS_CV
    default:
      return set_error(XOPS_ERR_UNSUPPORTED, "causal_conv1d_varlen: width %d not in [2, 6]", W);
  }
}

// ----------------------------------------------------------------------------
// Slot-table path of npu_causal_conv1d_update_v2: speculative decoding and
// prefix-cache (APC) block tables (_causal_conv1d_update_kernel_npu_tiled_v2,
// triton_npu/triton_src/test_causal_conv1d_update_v2.py:34-233, torch
// reference :260-345).  Per sequence b:
//   in  = idx[b, initial_state_idx[b]]   out = idx[b, block_idx_last[b]]
//         (a [B] table: idx[b] for both; no table: b); in == pad_slot_id skips
//   off = num_accepted_tokens[b] - 1 (speculative) or 0
//   L   = width - 1 + (speculative ? len - 1 : 0)   state columns rewritten
// outputs convolve cat(state[in, :, off : off + width - 1], x_seq); the new
// state[out, :, 0:L] is the last L of cat(state[in, :, off + shift :], x_seq)
// with shift = 1 (speculative) or len.  L is per sequence: the reference
// derives it from max_query_len, which for sequences shorter than that
// rewrites only part of the window.
// One thread per (sequence, channel); everything read from the input line is
// read before the output line is written, so in == out is safe.
template <typename T, int W>
__global__ void __launch_bounds__(256) conv1d_v2_slots_kernel(
    const T* __restrict__ x, T* conv_state, const T* __restrict__ w, const T* __restrict__ bias,
    const int32_t* __restrict__ idx, int64_t idx_stride, const int32_t* __restrict__ accepted,
    const int32_t* __restrict__ init_idx, const int32_t* __restrict__ last_idx,
    const int32_t* __restrict__ qsl, T* __restrict__ out, int64_t dim, int64_t state_len,
    int64_t num_lines, bool silu, int32_t pad_slot_id) {
  const int64_t b = blockIdx.y;
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t in_line = b, out_line = b;
  if (idx) {
    const int64_t i0 = init_idx ? init_idx[b] : 0, i1 = last_idx ? last_idx[b] : 0;
    in_line = idx[b * idx_stride + i0];
    out_line = idx[b * idx_stride + i1];
  }
  // a padded row, or a line outside the cache: nothing is read or written
  if (in_line == pad_slot_id || in_line < 0 || in_line >= num_lines || out_line < 0 ||
      out_line >= num_lines)
    return;
  const int64_t qs = qsl[b], len = (int64_t)qsl[b + 1] - qs;
  if (len <= 0 || c >= dim) return;
  const bool spec = accepted != nullptr;
  const int64_t off = spec ? (int64_t)accepted[b] - 1 : 0;
  const int64_t L = (W - 1) + (spec ? len - 1 : 0);
  const T* src = conv_state + (in_line * dim + c) * state_len;
  T* dst = conv_state + (out_line * dim + c) * state_len;
  auto st = [&](int64_t j) { return j >= 0 && j < state_len ? to_f32<T>(src[j]) : 0.f; };
  float wv[W], hist[W > 1 ? W - 1 : 1], keepv[W > 2 ? W - 2 : 1];
#pragma unroll
  for (int j = 0; j < W; ++j) wv[j] = to_f32<T>(w[c * W + j]);
#pragma unroll
  for (int j = 0; j < W - 1; ++j) hist[j] = st(off + j);
  const int64_t shift = spec ? 1 : len;
  const int64_t keep = len < L ? L - len : 0;  // <= W - 2
#pragma unroll
  for (int j = 0; j < W - 2; ++j) keepv[j] = j < keep ? st(off + shift + j) : 0.f;
  const float bsum = bias ? to_f32<T>(bias[c]) : 0.f;
  for (int64_t t = 0; t < len; ++t) {
    const float xv = to_f32<T>(x[(qs + t) * dim + c]);
    float acc = bsum + xv * wv[W - 1];
#pragma unroll
    for (int j = 0; j < W - 1; ++j) acc = fmaf(hist[j], wv[j], acc);
#pragma unroll
    for (int j = 0; j + 1 < W - 1; ++j) hist[j] = hist[j + 1];
    if (W > 1) hist[W > 1 ? W - 2 : 0] = xv;
    out[(qs + t) * dim + c] = from_f32<T>(silu ? silu_f(acc) : acc);
  }
  // new window: keep carried columns, then the sequence's last tokens
  for (int64_t j = 0; j < L && j < state_len; ++j) {
    float v;
    if (j < keep) {
      v = 0.f;
#pragma unroll
      for (int u = 0; u < W - 2; ++u)
        if (u == j) v = keepv[u];
    } else {
      v = to_f32<T>(x[(qs + len - L + j) * dim + c]);
    }
    dst[j] = from_f32<T>(v);
  }
}

int launch_v2_slots(int W, const void* x, void* state, const void* w, const void* b,
                    const int32_t* idx, int64_t idx_stride, const int32_t* accepted,
                    const int32_t* init_idx, const int32_t* last_idx, const int32_t* qsl,
                    void* out, int64_t batch, int64_t dim, int64_t state_len,
                    int64_t num_lines, bool silu, int32_t pad, int dtype, cudaStream_t st) {
  const dim3 grid((unsigned)cdiv64(dim, 256), (unsigned)batch);
  auto run = [&](auto t) {
    using T = decltype(t);
    switch (W) {
#define XOPS_V2S(WW)                                                                              \
  case WW:                                                                                        \
    conv1d_v2_slots_kernel<T, WW><<<grid, 256, 0, st>>>(                                          \
        (const T*)x, (T*)state, (const T*)w, (const T*)b, idx, idx_stride, accepted, init_idx,   \
        last_idx, qsl, (T*)out, dim, state_len, num_lines, silu, pad);                            \
    return check_launch("causal_conv1d_update_v2(slots)");
      XOPS_V2S(1) XOPS_V2S(2) XOPS_V2S(3) XOPS_V2S(4) XOPS_V2S(5) XOPS_V2S(6)
#undef XOPS_V2S
      default:
        return set_error(XOPS_ERR_UNSUPPORTED, "causal_conv1d_update_v2: width %d", W);
    }
  };
  switch (dtype) {
    case XOPS_F32: return run(float{});
    case XOPS_BF16: return run(__nv_bfloat16{});
    default: return run(__half{});
  }
}

}  // namespace

int take_conv_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_conv_error, sizeof(int)) != cudaSuccess) return -1;
  const int zero = 0;
  cudaMemcpyToSymbol(g_conv_error, &zero, sizeof(int));
  return v;
}
}  // namespace xops

using namespace xops;

extern "C" int xops_causal_conv1d_varlen(const void* x, void* conv_state, const void* weight,
                                         const void* bias, const int32_t* query_start_loc,
                                         const int32_t* conv_state_indices, void* out,
                                         int64_t batch, int64_t total_tokens, int64_t dim,
                                         int64_t width, int64_t num_cache_lines, int silu,
                                         int32_t pad_slot_id, int dtype, void* stream) {
  XOPS_REQUIRE(batch >= 0 && total_tokens >= 0 && dim > 0, "causal_conv1d_varlen: bad shape");
  XOPS_REQUIRE(width >= 2 && width <= 6, "causal_conv1d_varlen expects width in [2, 6], got %lld",
               (long long)width);
  XOPS_REQUIRE(dim % VEC == 0, "causal_conv1d_varlen: dim must be a multiple of %d", VEC);
  XOPS_REQUIRE(dtype == XOPS_BF16 || dtype == XOPS_F32 || dtype == XOPS_F16,
               "causal_conv1d_varlen: bad dtype");
  XOPS_REQUIRE(conv_state_indices || num_cache_lines >= batch,
               "causal_conv1d_varlen: conv_state has fewer lines than sequences");
  if (batch == 0 || total_tokens == 0) return XOPS_OK;
  XOPS_REQUIRE(x && conv_state && weight && query_start_loc && out,
               "causal_conv1d_varlen: null pointer");
  XOPS_REQUIRE(aligned16(x) && aligned16(out), "causal_conv1d_varlen: x/out must be 16-byte aligned");
  // upper bound on tiles: sum ceil(len/TILE) <= total/TILE + batch
  const int64_t tiles = total_tokens / TILE_T + batch;
  cudaStream_t st = (cudaStream_t)stream;
  switch (dtype) {
    case XOPS_BF16:
      return launch_varlen_tma<__nv_bfloat16>((int)width, x, conv_state, weight, bias,
                                              query_start_loc, conv_state_indices, out,
                                              (int)batch, total_tokens, dim, silu != 0,
                                              pad_slot_id, st);
    case XOPS_F16:
      return launch_varlen_tma<__half>((int)width, x, conv_state, weight, bias, query_start_loc,
                                       conv_state_indices, out, (int)batch, total_tokens, dim,
                                       silu != 0, pad_slot_id, st);
    default:
      return launch_varlen_w<float>((int)width, x, conv_state, weight, bias, query_start_loc,
                                    conv_state_indices, out, (int)batch, tiles, dim, silu != 0,
                                    pad_slot_id, st);
  }
}

extern "C" int xops_causal_conv1d_varlen_qk_l2norm(
    const void* x, void* conv_state, const void* weight, const void* bias,
    const int32_t* query_start_loc, const int32_t* conv_state_indices, void* out, int64_t batch,
    int64_t total_tokens, int64_t dim, int64_t width, int64_t num_cache_lines, int silu,
    int32_t pad_slot_id, int dtype, int64_t l2_channels, float l2_eps, void* stream) {
  XOPS_REQUIRE(batch >= 0 && total_tokens >= 0 && dim > 0, "causal_conv1d_varlen_qk_l2norm: bad shape");
  XOPS_REQUIRE(width >= 2 && width <= 6,
               "causal_conv1d_varlen_qk_l2norm expects width in [2, 6], got %lld", (long long)width);
  XOPS_REQUIRE(l2_channels >= 0 && l2_channels % 128 == 0 && l2_channels <= dim && dim % 128 == 0,
               "causal_conv1d_varlen_qk_l2norm: the normalised channels must be whole 128-channel "
               "heads at the front of a dim that is a multiple of 128 (got %lld of %lld)",
               (long long)l2_channels, (long long)dim);
  XOPS_UNSUPPORTED(dtype == XOPS_BF16 || dtype == XOPS_F16,
                   "causal_conv1d_varlen_qk_l2norm: 16-bit activations only");
  XOPS_REQUIRE(conv_state_indices || num_cache_lines >= batch,
               "causal_conv1d_varlen_qk_l2norm: conv_state has fewer lines than sequences");
  if (batch == 0 || total_tokens == 0) return XOPS_OK;
  XOPS_REQUIRE(x && conv_state && weight && query_start_loc && out,
               "causal_conv1d_varlen_qk_l2norm: null pointer");
  XOPS_REQUIRE(aligned16(x) && aligned16(out),
               "causal_conv1d_varlen_qk_l2norm: x/out must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == XOPS_BF16)
    return launch_varlen_tma<__nv_bfloat16>((int)width, x, conv_state, weight, bias,
                                            query_start_loc, conv_state_indices, out, (int)batch,
                                            total_tokens, dim, silu != 0, pad_slot_id, st,
                                            l2_channels, l2_eps);
  return launch_varlen_tma<__half>((int)width, x, conv_state, weight, bias, query_start_loc,
                                   conv_state_indices, out, (int)batch, total_tokens, dim,
                                   silu != 0, pad_slot_id, st, l2_channels, l2_eps);
}

extern "C" int xops_causal_conv1d_varlen_qkvz(
    const void* mixed_qkvz, int64_t x_ld, int64_t num_k_heads, int64_t num_v_heads,
    void* conv_state, const void* weight, const void* bias, const int32_t* query_start_loc,
    const int32_t* conv_state_indices, void* out, int64_t batch, int64_t total_tokens,
    int64_t width, int64_t num_cache_lines, int silu, int32_t pad_slot_id, int dtype,
    int qk_l2norm, float l2_eps, void* stream) {
  XOPS_REQUIRE(batch >= 0 && total_tokens >= 0 && num_k_heads >= 1 && num_v_heads >= 1 &&
                   num_v_heads % num_k_heads == 0,
               "causal_conv1d_varlen_qkvz: bad shape (num_v_heads must be a multiple of "
               "num_k_heads)");
  XOPS_REQUIRE(width >= 2 && width <= 6,
               "causal_conv1d_varlen_qkvz expects width in [2, 6], got %lld", (long long)width);
  XOPS_UNSUPPORTED(dtype == XOPS_BF16 || dtype == XOPS_F16,
                   "causal_conv1d_varlen_qkvz: 16-bit activations only");
  const int64_t r = num_v_heads / num_k_heads, group = 128 * (2 + 2 * r);
  const int64_t dim = 128 * (2 * num_k_heads + num_v_heads);
  XOPS_REQUIRE(x_ld >= num_k_heads * group && x_ld % 8 == 0,
               "causal_conv1d_varlen_qkvz: the projection's row stride must cover its %lld "
               "columns and be a multiple of 8", (long long)(num_k_heads * group));
  XOPS_REQUIRE(conv_state_indices || num_cache_lines >= batch,
               "causal_conv1d_varlen_qkvz: conv_state has fewer lines than sequences");
  if (batch == 0 || total_tokens == 0) return XOPS_OK;
  XOPS_REQUIRE(mixed_qkvz && conv_state && weight && query_start_loc && out,
               "causal_conv1d_varlen_qkvz: null pointer");
  XOPS_REQUIRE(aligned16(mixed_qkvz) && aligned16(out),
               "causal_conv1d_varlen_qkvz: mixed_qkvz/out must be 16-byte aligned");
  cudaStream_t st = (cudaStream_t)stream;
  const QkvzMap cm{(int)num_k_heads, (int)r, group};
  const int64_t l2c = qk_l2norm ? 2 * 128 * num_k_heads : 0;
  if (dtype == XOPS_BF16)
    return launch_varlen_tma<__nv_bfloat16>((int)width, mixed_qkvz, conv_state, weight, bias,
                                            query_start_loc, conv_state_indices, out, (int)batch,
                                            total_tokens, dim, silu != 0, pad_slot_id, st, l2c,
                                            l2_eps, x_ld, cm);
  return launch_varlen_tma<__half>((int)width, mixed_qkvz, conv_state, weight, bias,
                                   query_start_loc, conv_state_indices, out, (int)batch,
                                   total_tokens, dim, silu != 0, pad_slot_id, st, l2c, l2_eps, x_ld,
                                   cm);
}

extern "C" int xops_causal_conv1d_update(const void* x, void* conv_state, const void* weight,
                                         const void* bias, const int32_t* conv_state_indices,
                                         void* out, int64_t batch, int64_t dim, int64_t seqlen,
                                         int64_t width, int64_t state_len,
                                         int64_t num_cache_lines, int64_t x_stride_b,
                                         int64_t x_stride_d, int64_t x_stride_t, int silu,
                                         int32_t pad_slot_id, int dtype, void* stream) {
  XOPS_REQUIRE(batch >= 0 && dim > 0 && seqlen >= 1, "causal_conv1d_update: bad shape");
  XOPS_REQUIRE(width >= 1 && width <= MAXW, "causal_conv1d_update: width must be in [1, %d]", MAXW);
  XOPS_REQUIRE(state_len >= width - 1, "causal_conv1d_update: state_len < width - 1");
  XOPS_REQUIRE(dim % VEC == 0, "causal_conv1d_update: dim must be a multiple of %d", VEC);
  XOPS_REQUIRE(dtype == XOPS_BF16 || dtype == XOPS_F32 || dtype == XOPS_F16,
               "causal_conv1d_update: bad dtype");
  XOPS_REQUIRE(conv_state_indices || num_cache_lines >= batch,
               "causal_conv1d_update: conv_state has fewer lines than batch rows");
  if (batch == 0) return XOPS_OK;
  XOPS_REQUIRE(x && conv_state && weight && out, "causal_conv1d_update: null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t n = batch * (dim / VEC);
  const unsigned blocks = (unsigned)cdiv64(n, 256);
  const bool fast = width == 4 && state_len == 3 && seqlen == 1 && x_stride_d == 1 &&
                    aligned16(x) && aligned16(out) && aligned16(conv_state) &&
                    aligned16(weight) && (x_stride_b % VEC) == 0;
  auto run = [&](auto tag) {
    using T = decltype(tag);
    if (fast) {
      if constexpr (sizeof(T) == 2) {
        if (!bias || aligned16(bias)) {
          const unsigned b2 = (unsigned)cdiv64(cdiv64(batch, 2) * (dim / VEC), 256);
          conv1d_decode_w4_rows_kernel<T><<<b2, 256, 0, st>>>(
              (const T*)x, (T*)conv_state, (const T*)weight, (const T*)bias, conv_state_indices,
              (T*)out, batch, dim, x_stride_b, silu != 0, pad_slot_id);
          return check_launch("causal_conv1d_update");
        }
      }
      conv1d_decode_w4_kernel<T><<<blocks, 256, 0, st>>>(
          (const T*)x, (T*)conv_state, (const T*)weight, (const T*)bias, conv_state_indices,
          (T*)out, batch, dim, x_stride_b, silu != 0, pad_slot_id);
      return check_launch("causal_conv1d_update");
    }
    switch (width) {
#define XOPS_CU(WW)                                                                             \
  case WW:                                                                                      \
    conv1d_update_kernel<T, WW><<<blocks, 256, 0, st>>>(                                        \
        (const T*)x, (T*)conv_state, (const T*)weight, (const T*)bias, conv_state_indices,     \
        (T*)out, batch, dim, seqlen, state_len, x_stride_b, x_stride_d, x_stride_t, silu != 0, \
        pad_slot_id);                                                                           \
    return check_launch("causal_conv1d_update");
      XOPS_CU(1) XOPS_CU(2) XOPS_CU(3) XOPS_CU(4) XOPS_CU(5) XOPS_CU(6) XOPS_CU(7) XOPS_CU(8)
#undef XOPS_CU
      default:
        return (int)XOPS_ERR_UNSUPPORTED;
    }
  };
  switch (dtype) {
    case XOPS_BF16: return run(__nv_bfloat16{});
    case XOPS_F16: return run(__half{});
    default: return run(float{});
  }
}

extern "C" int xops_causal_conv1d_update_v2_slots(
    const void* x, void* conv_state, const void* weight, const void* bias,
    const int32_t* conv_state_indices, int64_t indices_stride, const int32_t* num_accepted_tokens,
    const int32_t* initial_state_idx, const int32_t* block_idx_last_scheduled_token,
    const int32_t* query_start_loc, void* out, int64_t batch, int64_t dim, int64_t width,
    int64_t state_len, int64_t num_cache_lines, int silu, int32_t pad_slot_id, int dtype,
    void* stream) {
  const char* what = "causal_conv1d_update_v2";
  XOPS_REQUIRE(batch >= 0 && batch < 65536 && dim >= 1, "%s: bad shape", what);
  XOPS_REQUIRE(width >= 1 && width <= 6, "%s expects width in [1, 6], got %lld", what,
               (long long)width);
  XOPS_REQUIRE(state_len >= width - 1, "%s: conv_state holds %lld columns, width %lld needs %lld",
               what, (long long)state_len, (long long)width, (long long)(width - 1));
  XOPS_REQUIRE((initial_state_idx == nullptr) == (block_idx_last_scheduled_token == nullptr),
               "%s expects both APC tensors or neither.", what);
  XOPS_REQUIRE(!initial_state_idx || conv_state_indices,
               "%s: APC block tables need a 2D conv_state_indices", what);
  XOPS_REQUIRE(dtype == XOPS_F32 || dtype == XOPS_BF16 || dtype == XOPS_F16, "%s: bad dtype",
               what);
  if (batch == 0) return XOPS_OK;
  XOPS_REQUIRE(x && conv_state && weight && query_start_loc && out, "%s: null pointer", what);
  return launch_v2_slots((int)width, x, conv_state, weight, bias, conv_state_indices,
                         indices_stride, num_accepted_tokens, initial_state_idx,
                         block_idx_last_scheduled_token, query_start_loc, out, batch, dim,
                         state_len, num_cache_lines, silu != 0, pad_slot_id, dtype,
                         (cudaStream_t)stream);
}
