// The reference's chunk pipeline as separate operators (drop-in for callers
// that run the stages themselves): chunk_local_cumsum, chunk_scaled_dot_kkt,
// solve_tril, recompute_w_u, chunk_gated_delta_rule_fwd_h and chunk_fwd_o
// (triton_npu/torch_api/npu_triton_chunk_gated_delta_rule.cpp:151-802).
// Each follows the layouts of the reference's Triton kernels
// (triton_npu/triton_src/chunk_gated_delta_rule/*.py) and computes in fp32
// with bf16 operands on the tcgen05 tensor cores: SW128 shared-memory tiles,
// fp32 accumulators in TMEM, one thread issuing, a bounded mbarrier wait
// (a timeout sets the device error flag and the CTA leaves).  The fused
// xops_chunk_gated_delta_rule is the production path; these exist so every
// stage can also be called alone.
//
// Varlen chunk addressing is derived on the device from cu_seqlens (no host
// copy of the offsets, unlike prepare_chunk_indices_like_python at :38-75):
// chunk-parallel kernels launch an upper bound of T/64 + N chunk slots and
// the CTAs past the last chunk exit.
#include "gdn_common.cuh"
#include "gdn_tc.cuh"
#include "tcgen05.cuh"

namespace xops {
namespace gdn {
namespace {

struct ChunkPos {
  int64_t seq, t0, eos, cis;
  int L;
  bool valid;
};

// Resolves blockIdx.x to a chunk; thread 0 scans, everyone reads the result.
__device__ __forceinline__ ChunkPos resolve_chunk(const int32_t* cu, int64_t N, int64_t T) {
  __shared__ int64_t s_pos[4];
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    int64_t seq = 0, t0 = 0, eos = 0, cis = 0;
    const bool ok = locate_chunk(cu, N, T, blockIdx.x, seq, t0, eos, cis);
    s_pos[0] = seq; s_pos[1] = t0; s_pos[2] = eos; s_pos[3] = cis;
    s_ok = ok ? 1 : 0;
  }
  __syncthreads();
  ChunkPos p;
  p.valid = s_ok != 0;
  p.seq = s_pos[0]; p.t0 = s_pos[1]; p.eos = s_pos[2]; p.cis = s_pos[3];
  p.L = (int)((p.eos - p.t0) < BT ? (p.eos - p.t0) : BT);
  return p;
}

constexpr uint32_t SO_WAIT = 1u << 26;
__device__ int g_subop_error = 0;

// TMEM columns for one CTA (a power of two >= 32), allocated by warp 0
struct TmemBlock {
  uint32_t base;
};
__device__ __forceinline__ bool so_wait(uint64_t* bar, uint32_t& phase) {
  const bool ok = tc::mbar_wait(bar, phase, SO_WAIT);
  phase ^= 1u;
  if (!ok) atomicExch(&g_subop_error, 1);
  tc::fence_after();
  return ok;
}

// Values t = 0..63 of TMEM lane row (this thread's lane of warp quarter q),
// 16 columns at a time, into v (64 floats)
__device__ __forceinline__ void tmem_row64(uint32_t tm, int q, uint32_t col, float (&v)[64]) {
  tc::tmem_ld32(tm_addr(tm, q, col), *reinterpret_cast<float(*)[32]>(v));
  tc::tmem_ld32(tm_addr(tm, q, col + 32), *reinterpret_cast<float(*)[32]>(v + 32));
  tc::tmem_wait_ld();
}

// Two accumulators D1[c][t], D2[c][t] (TMEM lane c = 32 q + lane, columns
// col1 + t, col2 + t) of warp quarter q, combined per element by f(t, d1,
// d2), stored as bf16 out[(t0 + t) * row_stride + c] for t < L.  Sixteen
// tokens at a time: the 16-lane TMEM loads give the mma fragment layout
// (register pairs 0 / 1 of a load: values l / 4 and l / 4 + 8, tokens
// 2 (l % 4) + {0, 1}; pairs 2 / 3: the same 8 tokens further on), and two
// transposing stmatrix stores write 16 tokens x 32 values into the warp's
// 1 KB buffer, from which each lane stores two 16-byte pieces.
template <typename F>
__device__ __forceinline__ void store_ct(uint32_t tm, int q, uint32_t col1, uint32_t col2,
                                         unsigned char* buf, bf16* out, int64_t row_stride,
                                         int64_t t0, int L, int lane, F f) {
  const int mi = lane >> 3, tok = ((mi >> 1) << 3) + (lane & 7), vb = (mi & 1) << 3;
  const int tr = 2 * (lane & 3);
  for (int tb = 0; tb < 64; tb += 16) {
    uint32_t a1[8], b1[8], a2[8], b2[8];
    tc::tmem_ld16x256b_x2(tm_addr(tm, q, col1 + tb), a1);
    tc::tmem_ld16x256b_x2(tm_addr(tm, q, col1 + tb) + (16u << 16), b1);
    tc::tmem_ld16x256b_x2(tm_addr(tm, q, col2 + tb), a2);
    tc::tmem_ld16x256b_x2(tm_addr(tm, q, col2 + tb) + (16u << 16), b2);
    tc::tmem_wait_ld();
    auto pk = [&](const uint32_t(&x)[8], const uint32_t(&y)[8], int e, int t) {
      return pack2<bf16>(make_float2(f(t, __uint_as_float(x[e]), __uint_as_float(y[e])),
                                     f(t + 1, __uint_as_float(x[e + 1]), __uint_as_float(y[e + 1]))));
    };
    const int ta = tb + tr, tc8 = tb + tr + 8;
    __syncwarp();
    stmatrix_x4_trans(buf + tok * 64 + vb * 2, pk(a1, a2, 0, ta), pk(a1, a2, 2, ta),
                      pk(a1, a2, 4, tc8), pk(a1, a2, 6, tc8));
    stmatrix_x4_trans(buf + tok * 64 + (16 + vb) * 2, pk(b1, b2, 0, ta), pk(b1, b2, 2, ta),
                      pk(b1, b2, 4, tc8), pk(b1, b2, 6, tc8));
    __syncwarp();
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int r = (lane >> 2) + 8 * j, m = lane & 3;  // token row, 8-value piece
      if (tb + r < L)
        *reinterpret_cast<uint4*>(out + (t0 + tb + r) * row_stride + q * 32 + m * 8) =
            *reinterpret_cast<const uint4*>(buf + r * 64 + m * 16);
    }
  }
}

// ---- chunk_local_cumsum (cumsum.py:25-73) ----------------------------------
__global__ void __launch_bounds__(256) cumsum_kernel(const float* __restrict__ g,
                                                     float* __restrict__ out,
                                                     const int32_t* __restrict__ cu, int64_t N,
                                                     int64_t T, int64_t H) {
  const ChunkPos p = resolve_chunk(cu, N, T);
  if (!p.valid) return;
  for (int64_t h = threadIdx.x; h < H; h += blockDim.x) {
    float acc = 0.f;
    for (int i = 0; i < p.L; ++i) {
      acc += g[(p.t0 + i) * H + h];
      out[(p.t0 + i) * H + h] = acc;
    }
  }
}

// ---- chunk_scaled_dot_kkt (chunk_scaled_dot_kkt.py:25-84) ------------------
// One CTA per (chunk, key head): the Gram matrix k kᵀ is one M = 128 product
// (rows 64..127 of the A operand are don't-care and their results unused),
// shared by every value head of the key head; the epilogue applies each
// head's beta_i e^{gc_i - gc_j} on the strict lower triangle.
constexpr int KK_NT = 128, KK_SMEM = 32768 + 1024 + 8192;  // k tile (128-row extent), gates
__global__ void __launch_bounds__(KK_NT) kkt_kernel(const bf16* __restrict__ k,
                                                    const float* __restrict__ beta,
                                                    const float* __restrict__ gc,
                                                    float* __restrict__ A,
                                                    const int32_t* __restrict__ cu, int64_t N,
                                                    int64_t T, int64_t Hg, int64_t H) {
  extern __shared__ unsigned char kk_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(kk_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* sgb = reinterpret_cast<float*>(sm + 32768);  // [grp][64] gc, then [grp][64] beta
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_sh;
  const ChunkPos p = resolve_chunk(cu, N, T);
  if (!p.valid) return;
  const int hk = blockIdx.y, grp = (int)(H / Hg);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (warp == 0) {
    tc::tmem_alloc(&tmem_sh, 64);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::mbar_fence_init();
  }
  // k rows as the first 64 rows of a 128-row SW128 tile (halves 16 KB apart)
  cp_tile128(sm, 16384, k + p.t0 * Hg * 128 + (int64_t)hk * 128, Hg * 128, p.L, tid, KK_NT);
  cp_async_commit();
  for (int e = tid; e < grp * 64; e += KK_NT) {
    const int hh = e >> 6, t = e & 63;
    const int64_t gi = (p.t0 + t) * H + hk * grp + hh;
    sgb[e] = (gc && t < p.L) ? gc[gi] : 0.f;
    sgb[grp * 64 + e] = t < p.L ? beta[gi] : 0.f;
  }
  cp_async_wait_all();
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = tmem_sh, sb = tc::smem_addr(sm);
  uint32_t phase = 0;
  if (tid == 0) {
    const uint32_t id = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      tc::mma_bf16(tm, kdesc(sb, 16384, j), kdesc(sb, 16384, j), id, j > 0);
    tc::commit(&bar);
  }
  const bool ok = so_wait(&bar, phase);
  if (ok && warp < 2) {  // lanes 0..63: Gram rows i
    const int i = warp * 32 + lane;
    float gr[64];
    tmem_row64(tm, warp, 0, gr);
    if (i < p.L) {
      for (int hh = 0; hh < grp; ++hh) {
        const float* sg = sgb + hh * 64;
        const float bi = sgb[grp * 64 + hh * 64 + i], gi = sg[i];
        float4* dst = reinterpret_cast<float4*>(A + ((p.t0 + i) * H + hk * grp + hh) * BT);
#pragma unroll
        for (int c = 0; c < 64; c += 4) {
          float v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int j = c + u;
            v[u] = j < i ? gr[j] * bi * __expf(fminf(gi - sg[j], 0.f)) : 0.f;
          }
          dst[c >> 2] = make_float4(v[0], v[1], v[2], v[3]);
        }
      }
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, 64);
}

// ---- solve_tril (solve_tril.py:32-330) --------------------------------------
template <typename TO>
__global__ void __launch_bounds__(256) solve_tril_kernel(const float* __restrict__ A,
                                                         TO* __restrict__ Ai,
                                                         const int32_t* __restrict__ cu,
                                                         int64_t N, int64_t T, int64_t H) {
  __shared__ float sA[BT * LDF], sT[BT * LDF], sM[32 * 33];
  const ChunkPos p = resolve_chunk(cu, N, T);
  if (!p.valid) return;
  const int h = blockIdx.y, tid = threadIdx.x;
  for (int e = tid; e < BT * BT; e += 256) {
    const int i = e >> 6, j = e & 63;
    sA[i * LDF + j] = (i < p.L && j < i) ? A[((p.t0 + i) * H + h) * BT + j] : 0.f;
  }
  __syncthreads();
  tri_inverse_64(sA, sT, sM, tid);
  for (int e = tid; e < BT * BT; e += 256) {
    const int i = e >> 6, j = e & 63;
    if (i < p.L) Ai[((p.t0 + i) * H + h) * BT + j] = from_f32<TO>(j < p.L ? sT[i * LDF + j] : 0.f);
  }
}

// ---- recompute_w_u (wy_fast.py:23-85) ----------------------------------------
// One CTA per (chunk, value head).  With V (or K) as the M = 128 dimension:
//   uᵀ[c][t] = sum_j v[j][c] T'[t][j] + v[t][c] (d_t - bf16(d_t)),
//   wᵀ[kk][t] = sum_j k[j][kk] T''[t][j],
// T' = Ai diag(beta) with its diagonal d_t = Ai_tt beta_t in bf16 and the
// rounding of d_t restored by a diagonal correction product, T'' = Ai
// diag(beta e^{gc}); v and k are MN-major A operands straight from their
// token-row tiles.  Results leave TMEM transposed through stmatrix.
constexpr int WU_NT = 128;
constexpr int WU_K = 0, WU_V = 16384, WU_TP = 32768, WU_TPP = 40960, WU_TPL = 49152,
              WU_BUF = 57344, WU_SMEM = WU_BUF + 4 * 1024 + 1024;
template <typename TA>
__global__ void __launch_bounds__(WU_NT) recompute_wu_kernel(
    const bf16* __restrict__ k, const bf16* __restrict__ v, const float* __restrict__ beta,
    const float* __restrict__ gc, const TA* __restrict__ Ai, bf16* __restrict__ w,
    bf16* __restrict__ u, const int32_t* __restrict__ cu, int64_t N, int64_t T, int64_t Hg,
    int64_t H) {
  extern __shared__ unsigned char wu_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(wu_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_sh;
  const ChunkPos p = resolve_chunk(cu, N, T);
  if (!p.valid) return;
  const int h = blockIdx.y, hk = (int)(h / (H / Hg));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (warp == 0) {
    tc::tmem_alloc(&tmem_sh, 128);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::mbar_fence_init();
  }
  cp_tile128(sm + WU_K, 8192, k + p.t0 * Hg * 128 + (int64_t)hk * 128, Hg * 128, p.L, tid, WU_NT);
  cp_tile128(sm + WU_V, 8192, v + p.t0 * H * 128 + (int64_t)h * 128, H * 128, p.L, tid, WU_NT);
  cp_async_commit();
  // T' (diagonal in bf16), T'' and the diagonal correction as K-major [64 x 64]
  // tiles: 16-byte chunk (t, c8) of each
  for (int e = tid; e < 64 * 8; e += WU_NT) {
    const int t = e >> 3, c8 = e & 7;
    float tp[8], tq[8], tl[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      const int j = c8 * 8 + m;
      float tv = 0.f, eg = 0.f;
      if (t < p.L && j < p.L) {
        tv = to_f32<TA>(Ai[((p.t0 + t) * H + h) * BT + j]) * beta[(p.t0 + j) * H + h];
        eg = __expf(gc[(p.t0 + j) * H + h]);
      }
      tp[m] = tv;
      tq[m] = tv * eg;
      tl[m] = j == t ? tv - __bfloat162float(__float2bfloat16_rn(tv)) : 0.f;
    }
    uint4 a, b2, c;
    a.x = pack_bf16(tp[0], tp[1]); a.y = pack_bf16(tp[2], tp[3]);
    a.z = pack_bf16(tp[4], tp[5]); a.w = pack_bf16(tp[6], tp[7]);
    b2.x = pack_bf16(tq[0], tq[1]); b2.y = pack_bf16(tq[2], tq[3]);
    b2.z = pack_bf16(tq[4], tq[5]); b2.w = pack_bf16(tq[6], tq[7]);
    c.x = pack_bf16(tl[0], tl[1]); c.y = pack_bf16(tl[2], tl[3]);
    c.z = pack_bf16(tl[4], tl[5]); c.w = pack_bf16(tl[6], tl[7]);
    const uint32_t off = chunk_off(t, c8, 0);
    *reinterpret_cast<uint4*>(sm + WU_TP + off) = a;
    *reinterpret_cast<uint4*>(sm + WU_TPP + off) = b2;
    *reinterpret_cast<uint4*>(sm + WU_TPL + off) = c;
  }
  cp_async_wait_all();
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = tmem_sh, sb = tc::smem_addr(sm);
  uint32_t phase = 0;
  if (tid == 0) {
    const uint32_t id = tc::idesc_bf16(128, 64, true, false);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      tc::mma_bf16(tm, mndesc(sb + WU_V, 8192, j), kdesc64(sb + WU_TP, j), id, j > 0);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      tc::mma_bf16(tm, mndesc(sb + WU_V, 8192, j), kdesc64(sb + WU_TPL, j), id, true);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      tc::mma_bf16(tm + 64, mndesc(sb + WU_K, 8192, j), kdesc64(sb + WU_TPP, j), id, j > 0);
    tc::commit(&bar);
  }
  if (so_wait(&bar, phase)) {
    unsigned char* buf = sm + WU_BUF + warp * 1024;
    auto first = [](int, float x, float) { return x; };
    store_ct(tm, warp, 0, 0, buf, u + (int64_t)h * 128, H * 128, p.t0, p.L, lane, first);
    store_ct(tm, warp, 64, 64, buf, w + (int64_t)h * 128, H * 128, p.t0, p.L, lane, first);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, 128);
}

// ---- chunk_gated_delta_rule_fwd_h (chunk_delta_h.py:30-199) ------------------
// One CTA per (sequence, value head), serial over its chunks.  The fp32 state
// lives in registers as Sᵀ[c][kk] (thread: value row c = TMEM lane, 32 key
// columns), and per chunk, with V as the M = 128 dimension:
//   store h_c = bf16(S) and Sᵀ as the bf16 A operand (TMEM);
//   D[c][t]  = sum_kk Sᵀ[c][kk] w[t][kk];   v_new = u - Dᵀ  (stored if asked);
//   vt = v_new e^{gl - gc} as bf16 hi + lo (TMEM);
//   dS[c][kk] = sum_t vt[t][c] k[t][kk];     S = e^{gl} S + dS.
constexpr int FH_NT = 512;
constexpr int FH_W = 0, FH_K = 16384, FH_U = 32768, FH_G = 49152, FH_SMEM = FH_G + 256 + 1024;
constexpr uint32_t FH_TM_D = 0, FH_TM_S = 64, FH_TM_VH = 128, FH_TM_VL = 160, FH_TM_DS = 256;
__global__ void __launch_bounds__(FH_NT, 1) fwd_h_kernel(
    const bf16* __restrict__ k, const bf16* __restrict__ w, const bf16* __restrict__ u,
    const float* __restrict__ gc, const float* __restrict__ h0, bf16* __restrict__ hout,
    bf16* __restrict__ vnew, float* __restrict__ ht, const int32_t* __restrict__ cu, int64_t N,
    int64_t T, int64_t Hg, int64_t H) {
  extern __shared__ unsigned char fh_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(fh_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* sg = reinterpret_cast<float*>(sm + FH_G);
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_sh;
  __shared__ int abort_sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quarter = warp & 3, colq = warp >> 2;
  const int c = quarter * 32 + lane;          // value row (TMEM lane)
  const int kc0 = colq * 32, tc0 = colq * 16;  // key columns / token columns owned
  const int64_t n = blockIdx.x / H;
  const int h = (int)(blockIdx.x - n * H), hk = (int)(h / (H / Hg));
  int64_t bos, eos;
  seq_span(cu, n, T, bos, eos);
  const int64_t boh = chunk_offset(cu, n, T);
  if (warp == 0) {
    tc::tmem_alloc(&tmem_sh, 512);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::mbar_fence_init();
    abort_sh = 0;
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = tmem_sh, sb = tc::smem_addr(sm);
  uint32_t phase = 0;
  float2 S[16];  // Sᵀ[c][kc0 + 2m], Sᵀ[c][kc0 + 2m + 1]
  {
    const float* src = h0 ? h0 + ((int64_t)n * H + h) * 128 * 128 : nullptr;
#pragma unroll
    for (int m = 0; m < 16; ++m)
      S[m] = src ? make_float2(src[(kc0 + 2 * m) * 128 + c], src[(kc0 + 2 * m + 1) * 128 + c])
                 : make_float2(0.f, 0.f);
  }
  int64_t ci = 0;
  for (int64_t t0 = bos; t0 < eos; t0 += BT, ++ci) {
    const int L = (int)((eos - t0) < BT ? (eos - t0) : BT);
    cp_tile128(sm + FH_W, 8192, w + t0 * H * 128 + (int64_t)h * 128, H * 128, L, tid, FH_NT);
    cp_tile128(sm + FH_K, 8192, k + t0 * Hg * 128 + (int64_t)hk * 128, Hg * 128, L, tid, FH_NT);
    cp_tile128(sm + FH_U, 8192, u + t0 * H * 128 + (int64_t)h * 128, H * 128, L, tid, FH_NT);
    cp_async_commit();
    if (tid < BT) sg[tid] = (gc && tid < L) ? gc[(t0 + tid) * H + h] : 0.f;
    // h_c = the state before this chunk: bf16 to the output and as the A operand
    bf16* hdst = hout + ((boh + ci) * H + h) * 128 * 128;
    uint32_t pk[16];
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      pk[m] = pack2<bf16>(S[m]);
      const __nv_bfloat162 b2 = *reinterpret_cast<const __nv_bfloat162*>(&pk[m]);
      hdst[(int64_t)(kc0 + 2 * m) * 128 + c] = b2.x;
      hdst[(int64_t)(kc0 + 2 * m + 1) * 128 + c] = b2.y;
    }
    tc::tmem_st16u(tm_addr(tm, quarter, FH_TM_S + kc0 / 2), pk);
    tc::tmem_wait_st();
    cp_async_wait_all();
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (*(volatile int*)&abort_sh) break;
    const float gl = gc ? sg[L - 1] : 0.f;
    if (tid == 0) {
      const uint32_t id_w = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        tc::mma_bf16_ts(tm + FH_TM_D, tm + FH_TM_S + 8 * j, kdesc(sb + FH_W, 8192, j), id_w, j > 0);
      tc::commit(&bar);
    }
    if (!so_wait(&bar, phase)) atomicExch(&abort_sh, 1);
    // v_new = u - D for this thread's 16 tokens; vt = v_new e^{gl - gc} (hi + lo)
    float d[16];
    tc::tmem_ld16(tm_addr(tm, quarter, FH_TM_D + tc0), d);
    tc::tmem_wait_ld();
    uint32_t hi[8], lo[8];
#pragma unroll
    for (int m = 0; m < 8; ++m) {
      float vv[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = tc0 + 2 * m + e;
        const float uu = __bfloat162float(*reinterpret_cast<const bf16*>(sm + FH_U + elem_off(t, c, 8192)));
        vv[e] = uu - d[2 * m + e];
        if (vnew && t < L) vnew[((t0 + t) * H + h) * 128 + c] = __float2bfloat16_rn(vv[e]);
        if (gc) vv[e] *= __expf(fminf(gl - sg[t], 0.f));
      }
      const float2 sc = make_float2(vv[0], vv[1]);
      hi[m] = pack2<bf16>(sc);
      lo[m] = pack2<bf16>(fsub2(sc, unpack2<bf16>(hi[m])));
    }
    tc::tmem_st8u(tm_addr(tm, quarter, FH_TM_VH + tc0 / 2), hi);
    tc::tmem_st8u(tm_addr(tm, quarter, FH_TM_VL + tc0 / 2), lo);
    tc::tmem_wait_st();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (*(volatile int*)&abort_sh) break;
    if (tid == 0) {
      const uint32_t id_s = tc::idesc_bf16(128, 128, false, true);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        tc::mma_bf16_ts(tm + FH_TM_DS, tm + FH_TM_VH + 8 * j, mndesc(sb + FH_K, 8192, j), id_s, j > 0);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        tc::mma_bf16_ts(tm + FH_TM_DS, tm + FH_TM_VL + 8 * j, mndesc(sb + FH_K, 8192, j), id_s, true);
      tc::commit(&bar);
    }
    if (!so_wait(&bar, phase)) atomicExch(&abort_sh, 1);
    const float dl = gc ? __expf(gl) : 1.f;
    const float2 dl2 = make_float2(dl, dl);
#pragma unroll
    for (int cb = 0; cb < 2; ++cb) {
      float ds[16];
      tc::tmem_ld16(tm_addr(tm, quarter, FH_TM_DS + kc0 + cb * 16), ds);
      tc::tmem_wait_ld();
#pragma unroll
      for (int m = 0; m < 8; ++m)
        S[cb * 8 + m] = ffma2(S[cb * 8 + m], dl2, make_float2(ds[2 * m], ds[2 * m + 1]));
    }
    tc::fence_before();
    __syncthreads();  // the tiles and TMEM operands of this chunk are done with
    tc::fence_after();
    if (*(volatile int*)&abort_sh) break;
  }
  if (ht && !*(volatile int*)&abort_sh) {
    float* dst = ht + ((int64_t)n * H + h) * 128 * 128;
#pragma unroll
    for (int m = 0; m < 16; ++m) {
      dst[(kc0 + 2 * m) * 128 + c] = S[m].x;
      dst[(kc0 + 2 * m + 1) * 128 + c] = S[m].y;
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, 512);
}

// ---- chunk_fwd_o (chunk_o.py:26-116) -----------------------------------------
// One CTA per (chunk, value head), three tcgen05 products:
//   G[t][j]   = q_t . k_j                      (M = 128 with don't-care rows 64..127)
//   D1[c][t]  = sum_kk h[kk][c] q[t][kk]       (h as an MN-major A operand)
//   D2[c][t]  = sum_j v_new[j][c] Aqk[t][j],   Aqk = tril(G e^{gc_t - gc_j}) in bf16
// and o[t][c] = scale (e^{gc_t} D1 + D2), stored transposed through stmatrix.
constexpr int FO_NT = 128;
constexpr int FO_Q = 0, FO_K = 16384, FO_V = 32768, FO_H = 49152, FO_AQK = 81920,
              FO_BUF = 90112, FO_G = FO_BUF + 4096, FO_SMEM = FO_G + 256 + 1024;
__global__ void __launch_bounds__(FO_NT) fwd_o_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ vnew,
    const bf16* __restrict__ hs, const float* __restrict__ gc, bf16* __restrict__ o,
    const int32_t* __restrict__ cu, int64_t N, int64_t T, int64_t Hg, int64_t H, float scale) {
  extern __shared__ unsigned char fo_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(fo_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* sg = reinterpret_cast<float*>(sm + FO_G);
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_sh;
  const ChunkPos p = resolve_chunk(cu, N, T);
  if (!p.valid) return;
  const int h = blockIdx.y, hk = (int)(h / (H / Hg));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t gidx = chunk_offset(cu, p.seq, T) + p.cis;
  if (warp == 0) {
    tc::tmem_alloc(&tmem_sh, 256);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::mbar_fence_init();
  }
  // q, k, v_new: 64 token rows (halves 8 KB apart; q's A-operand use reads
  // on into k's rows, whose products land in unused TMEM lanes); h: 128 rows
  cp_tile128(sm + FO_Q, 8192, q + p.t0 * Hg * 128 + (int64_t)hk * 128, Hg * 128, p.L, tid, FO_NT);
  cp_tile128(sm + FO_K, 8192, k + p.t0 * Hg * 128 + (int64_t)hk * 128, Hg * 128, p.L, tid, FO_NT);
  cp_tile128(sm + FO_V, 8192, vnew + p.t0 * H * 128 + (int64_t)h * 128, H * 128, p.L, tid, FO_NT);
  const bf16* hsrc = hs + (gidx * H + h) * 128 * 128;
  cp_tile128(sm + FO_H, 16384, hsrc, 128, 64, tid, FO_NT);
  cp_tile128(sm + FO_H + 64 * 128, 16384, hsrc + 64 * 128, 128, 64, tid, FO_NT);
  cp_async_commit();
  if (tid < BT) sg[tid] = (gc && tid < p.L) ? gc[(p.t0 + tid) * H + h] : 0.f;
  cp_async_wait_all();
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = tmem_sh, sb = tc::smem_addr(sm);
  uint32_t phase = 0;
  if (tid == 0) {
    const uint32_t id_g = tc::idesc_bf16(128, 64, false, false);
    const uint32_t id_o = tc::idesc_bf16(128, 64, true, false);
#pragma unroll
    for (int j = 0; j < 8; ++j)  // G: q rows x k rows over kk
      tc::mma_bf16(tm, kdesc(sb + FO_Q, 8192, j), kdesc(sb + FO_K, 8192, j), id_g, j > 0);
#pragma unroll
    for (int j = 0; j < 8; ++j)  // D1: h (kk rows, MN = c) x q (K-major over kk)
      tc::mma_bf16(tm + 64, mndesc(sb + FO_H, 16384, j), kdesc(sb + FO_Q, 8192, j), id_o, j > 0);
    tc::commit(&bar);
  }
  bool ok = so_wait(&bar, phase);
  if (ok && warp < 2) {  // Aqk rows t = lanes 0..63, bf16 K-major [64 x 64] tile
    const int t = warp * 32 + lane;
    float gr[64];
    tmem_row64(tm, warp, 0, gr);
    const float gt = sg[t];
#pragma unroll
    for (int c8 = 0; c8 < 8; ++c8) {
      float e[8];
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int j = c8 * 8 + m;
        const float d = gc ? __expf(fminf(gt - sg[j], 0.f)) : 1.f;
        e[m] = j <= t ? gr[j] * d : 0.f;
      }
      uint4 pk;
      pk.x = pack_bf16(e[0], e[1]); pk.y = pack_bf16(e[2], e[3]);
      pk.z = pack_bf16(e[4], e[5]); pk.w = pack_bf16(e[6], e[7]);
      *reinterpret_cast<uint4*>(sm + FO_AQK + chunk_off(t, c8, 0)) = pk;
    }
  }
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  if (tid == 0 && ok) {
    const uint32_t id_o = tc::idesc_bf16(128, 64, true, false);
#pragma unroll
    for (int j = 0; j < 4; ++j)  // D2: v_new (token rows, MN = c) x Aqk (K-major over j)
      tc::mma_bf16(tm + 128, mndesc(sb + FO_V, 8192, j), kdesc64(sb + FO_AQK, j), id_o, j > 0);
    tc::commit(&bar);
  }
  if (ok) ok = so_wait(&bar, phase);
  if (ok) {
    unsigned char* buf = sm + FO_BUF + warp * 1024;
    const bool gated = gc != nullptr;
    auto comb = [&](int t, float d1, float d2) {
      return scale * ((gated ? __expf(sg[t]) : 1.f) * d1 + d2);
    };
    store_ct(tm, warp, 64, 128, buf, o + (int64_t)h * 128, H * 128, p.t0, p.L, lane, comb);
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, 256);
}

int common_checks(const char* what, const int32_t* cu, int64_t B, int64_t T, int64_t N) {
  XOPS_REQUIRE(B >= 1 && T >= 0 && N >= 0, "%s: bad shape", what);
  XOPS_REQUIRE(cu || N == B, "%s: without cu_seqlens N must equal B", what);
  XOPS_REQUIRE(!cu || B == 1, "%s: cu_seqlens requires B == 1", what);
  return XOPS_OK;
}

unsigned chunk_slots(const int32_t* cu, int64_t B, int64_t T, int64_t N) {
  return (unsigned)(cu ? T / BT + N : B * ((T + BT - 1) / BT));
}

}  // namespace
}  // namespace gdn
}  // namespace xops

using namespace xops;
using namespace xops::gdn;

namespace xops {
int take_subop_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gdn::g_subop_error, sizeof(int)) != cudaSuccess) return -1;
  const int zero = 0;
  cudaMemcpyToSymbol(gdn::g_subop_error, &zero, sizeof(int));
  return v;
}
}  // namespace xops

extern "C" int64_t xops_total_chunks(const int32_t* cu_seqlens_host, int64_t B, int64_t T,
                                     int64_t N, int64_t chunk_size) {
  if (chunk_size <= 0) return -1;
  if (!cu_seqlens_host) return B * ((T + chunk_size - 1) / chunk_size);
  int64_t acc = 0;
  for (int64_t i = 0; i < N; ++i) {
    const int64_t len = (int64_t)cu_seqlens_host[i + 1] - cu_seqlens_host[i];
    if (len > 0) acc += (len + chunk_size - 1) / chunk_size;
  }
  return acc;
}

extern "C" int xops_chunk_local_cumsum(const float* g, float* g_cumsum, const int32_t* cu_seqlens,
                                       int64_t B, int64_t T, int64_t N, int64_t H,
                                       int64_t chunk_size, void* stream) {
  if (int rc = common_checks("chunk_local_cumsum", cu_seqlens, B, T, N)) return rc;
  XOPS_UNSUPPORTED(chunk_size == BT, "chunk_local_cumsum: only chunk_size 64 is compiled");
  XOPS_REQUIRE(H >= 1, "chunk_local_cumsum: bad H");
  if (N == 0 || T == 0) return XOPS_OK;
  XOPS_REQUIRE(g && g_cumsum, "chunk_local_cumsum: null pointer");
  cumsum_kernel<<<chunk_slots(cu_seqlens, B, T, N), 256, 0, (cudaStream_t)stream>>>(
      g, g_cumsum, cu_seqlens, N, T, H);
  return check_launch("chunk_local_cumsum");
}

extern "C" int xops_chunk_scaled_dot_kkt_fwd(const void* k, const float* beta,
                                             const float* g_cumsum, float* A,
                                             const int32_t* cu_seqlens, int64_t B, int64_t T,
                                             int64_t N, int64_t Hg, int64_t H, int64_t K,
                                             int64_t chunk_size, void* stream) {
  if (int rc = common_checks("chunk_scaled_dot_kkt_fwd", cu_seqlens, B, T, N)) return rc;
  XOPS_UNSUPPORTED(chunk_size == BT && K == 128, "chunk_scaled_dot_kkt_fwd: needs chunk 64, K 128");
  XOPS_REQUIRE(Hg >= 1 && H % Hg == 0, "chunk_scaled_dot_kkt_fwd: H must be a multiple of Hg");
  XOPS_UNSUPPORTED(H / Hg <= 16, "chunk_scaled_dot_kkt_fwd: at most 16 value heads per key head");
  if (N == 0 || T == 0) return XOPS_OK;
  XOPS_REQUIRE(k && beta && A && aligned16(k), "chunk_scaled_dot_kkt_fwd: bad pointer");
  if (int rc = ensure_smem_attr((const void*)kkt_kernel, KK_SMEM, "chunk_scaled_dot_kkt_fwd"))
    return rc;
  dim3 grid(chunk_slots(cu_seqlens, B, T, N), (unsigned)Hg);
  kkt_kernel<<<grid, KK_NT, KK_SMEM, (cudaStream_t)stream>>>((const bf16*)k, beta, g_cumsum, A,
                                                             cu_seqlens, N, T, Hg, H);
  return check_launch("chunk_scaled_dot_kkt_fwd");
}

extern "C" int xops_solve_tril(const float* A, void* Ai, const int32_t* cu_seqlens, int64_t B,
                               int64_t T, int64_t N, int64_t H, int64_t chunk_size, int out_dtype,
                               void* stream) {
  if (int rc = common_checks("solve_tril", cu_seqlens, B, T, N)) return rc;
  XOPS_UNSUPPORTED(chunk_size == BT, "solve_tril: only chunk_size 64 is compiled");
  if (N == 0 || T == 0) return XOPS_OK;
  XOPS_REQUIRE(A && Ai, "solve_tril: null pointer");
  dim3 grid(chunk_slots(cu_seqlens, B, T, N), (unsigned)H);
  cudaStream_t st = (cudaStream_t)stream;
  switch (out_dtype) {
    case XOPS_F32: solve_tril_kernel<float><<<grid, 256, 0, st>>>(A, (float*)Ai, cu_seqlens, N, T, H); break;
    case XOPS_BF16: solve_tril_kernel<bf16><<<grid, 256, 0, st>>>(A, (bf16*)Ai, cu_seqlens, N, T, H); break;
    case XOPS_F16: solve_tril_kernel<__half><<<grid, 256, 0, st>>>(A, (__half*)Ai, cu_seqlens, N, T, H); break;
    default: return set_error(XOPS_ERR_INVALID_ARGUMENT, "solve_tril: bad out_dtype");
  }
  return check_launch("solve_tril");
}

extern "C" int xops_recompute_w_u_fwd(const void* k, const void* v, const float* beta,
                                      const float* g_cumsum, const void* Ai, int ai_dtype, void* w,
                                      void* u, const int32_t* cu_seqlens, int64_t B, int64_t T,
                                      int64_t N, int64_t Hg, int64_t H, int64_t K, int64_t V,
                                      void* stream) {
  if (int rc = common_checks("recompute_w_u_fwd", cu_seqlens, B, T, N)) return rc;
  XOPS_UNSUPPORTED(K == 128 && V == 128, "recompute_w_u_fwd: only K == V == 128 is compiled");
  XOPS_REQUIRE(Hg >= 1 && H % Hg == 0, "recompute_w_u_fwd: H must be a multiple of Hg");
  if (N == 0 || T == 0) return XOPS_OK;
  XOPS_REQUIRE(k && v && beta && g_cumsum && Ai && w && u, "recompute_w_u_fwd: null pointer");
  XOPS_REQUIRE(aligned16(k) && aligned16(v), "recompute_w_u_fwd: k/v must be 16-byte aligned");
  const size_t smem = WU_SMEM;
  dim3 grid(chunk_slots(cu_seqlens, B, T, N), (unsigned)H);
  cudaStream_t st = (cudaStream_t)stream;
#define XOPS_WU(TA)                                                                                \
  {                                                                                                \
    if (int rc = ensure_smem_attr((const void*)recompute_wu_kernel<TA>, smem, "recompute_w_u_fwd")) \
      return rc;                                                                                   \
    recompute_wu_kernel<TA><<<grid, WU_NT, smem, st>>>((const bf16*)k, (const bf16*)v, beta,       \
                                                     g_cumsum, (const TA*)Ai, (bf16*)w, (bf16*)u,  \
                                                     cu_seqlens, N, T, Hg, H);                     \
  }
  switch (ai_dtype) {
    case XOPS_F32: XOPS_WU(float) break;
    case XOPS_BF16: XOPS_WU(bf16) break;
    case XOPS_F16: XOPS_WU(__half) break;
    default: return set_error(XOPS_ERR_INVALID_ARGUMENT, "recompute_w_u_fwd: bad Ai dtype");
  }
#undef XOPS_WU
  return check_launch("recompute_w_u_fwd");
}

extern "C" int xops_chunk_gated_delta_rule_fwd_h(const void* k, const void* w, const void* u,
                                                 const float* g_cumsum, const float* h0, void* h,
                                                 void* v_new, float* ht,
                                                 const int32_t* cu_seqlens, int64_t B, int64_t T,
                                                 int64_t N, int64_t Hg, int64_t H, int64_t K,
                                                 int64_t V, int64_t NT, void* stream) {
  if (int rc = common_checks("chunk_gated_delta_rule_fwd_h", cu_seqlens, B, T, N)) return rc;
  XOPS_UNSUPPORTED(K == 128 && V == 128, "chunk_gated_delta_rule_fwd_h: only K == V == 128");
  XOPS_REQUIRE(Hg >= 1 && H % Hg == 0, "chunk_gated_delta_rule_fwd_h: H must be a multiple of Hg");
  XOPS_REQUIRE(NT >= 0, "chunk_gated_delta_rule_fwd_h: bad NT");
  if (N == 0) return XOPS_OK;
  XOPS_REQUIRE(k && w && u && (h || NT == 0), "chunk_gated_delta_rule_fwd_h: null pointer");
  XOPS_REQUIRE(aligned16(k) && aligned16(w) && aligned16(u),
               "chunk_gated_delta_rule_fwd_h: k/w/u must be 16-byte aligned");
  const size_t smem = FH_SMEM;
  if (int rc = ensure_smem_attr((const void*)fwd_h_kernel, smem, "chunk_gated_delta_rule_fwd_h"))
    return rc;
  fwd_h_kernel<<<(unsigned)(N * H), FH_NT, smem, (cudaStream_t)stream>>>(
      (const bf16*)k, (const bf16*)w, (const bf16*)u, g_cumsum, h0, (bf16*)h, (bf16*)v_new, ht,
      cu_seqlens, N, T, Hg, H);
  return check_launch("chunk_gated_delta_rule_fwd_h");
}

extern "C" int xops_chunk_fwd_o(const void* q, const void* k, const void* v_new, const void* h,
                                const float* g_cumsum, void* o, const int32_t* cu_seqlens,
                                int64_t B, int64_t T, int64_t N, int64_t Hg, int64_t H, int64_t K,
                                int64_t V, int64_t NT, float scale, void* stream) {
  if (int rc = common_checks("chunk_fwd_o", cu_seqlens, B, T, N)) return rc;
  XOPS_UNSUPPORTED(K == 128 && V == 128, "chunk_fwd_o: only K == V == 128 is compiled");
  XOPS_REQUIRE(Hg >= 1 && H % Hg == 0, "chunk_fwd_o: H must be a multiple of Hg");
  (void)NT;
  if (N == 0 || T == 0) return XOPS_OK;
  XOPS_REQUIRE(q && k && v_new && h && o, "chunk_fwd_o: null pointer");
  XOPS_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v_new) && aligned16(h),
               "chunk_fwd_o: tensors must be 16-byte aligned");
  const size_t smem = FO_SMEM;
  if (int rc = ensure_smem_attr((const void*)fwd_o_kernel, smem, "chunk_fwd_o")) return rc;
  dim3 grid(chunk_slots(cu_seqlens, B, T, N), (unsigned)H);
  fwd_o_kernel<<<grid, FO_NT, smem, (cudaStream_t)stream>>>(
      (const bf16*)q, (const bf16*)k, (const bf16*)v_new, (const bf16*)h, g_cumsum, (bf16*)o,
      cu_seqlens, N, T, Hg, H, scale);
  return check_launch("chunk_fwd_o");
}
