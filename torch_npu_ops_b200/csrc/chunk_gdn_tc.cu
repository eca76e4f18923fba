// Chunked gated delta rule prefill on the sm_100a tensor cores (tcgen05 +
// TMEM), fully fused: one CTA per (sequence, value head) walks the
// sequence's 64-token chunks in order and keeps the fp32 state in TMEM for
// the whole sequence.  None of the reference's intermediates -- g cumsum,
// A, (I+A)^-1, w, u, per-chunk h, v_new (npu_triton_chunk_gated_delta_rule.cpp:
// 556-642 writes each to HBM) -- leaves the SM; HBM sees q, k, v, g, beta,
// h0 once and o, ht once.
//
// All products are issued as tcgen05.mma (M = 128, bf16 operands from
// 128-byte-swizzled shared tiles, fp32 accumulators in TMEM).  The state is
// kept transposed, S^T[v][kk] (TMEM lane = value column v), so every product
// that touches it has M = 128:
//   G    = [k; q] k^T                 (M 128 = 64 k rows + 64 q rows, N 64)
//   u^T  = v^T T'^T,  w^T = k^T T''^T (A = v / k tiles read MN-major)
//   D_u += S^T (-w)^T                 (v_new^T = beta*v + D_u, B negated)
//   D_qh = S^T q^T                    (o inter-chunk term)
//   S^T += vt_hi^T k + vt_lo^T k      (k tile read MN-major as B)
//   D_o += v_new^T Aqk^T              (o intra-chunk term)
// with gc = in-chunk cumsum of g, D_ij = e^{gc_i - gc_j} (i >= j),
// T = (I + strict_tril(beta_i D_ij k_i.k_j))^-1, T' = (T - I) diag(beta),
// T'' = T diag(beta e^{gc}), vt = v_new e^{gc_last - gc} split into bf16 hi +
// lo, o = scale (e^{gc} (q S) + tril(q k^T D) v_new).  The diagonal beta_i v_i
// term and the hi/lo split keep the fp32 state within ~1e-5 of the fp32
// recurrence (a bf16 u or beta-on-diagonal costs ~2e-3).
//
// Phases are separated by CTA barriers; one thread issues the MMAs and
// tcgen05.commit arrives on an mbarrier that every thread waits on with a
// bounded poll (a timeout records an error and the CTA bails out).
#include "gdn_common.cuh"
#include "tcgen05.cuh"

namespace xops {
namespace gdn {

__device__ int g_tc_error = 0;  // set by a CTA whose mbarrier wait timed out

namespace {

constexpr int NT = 256;  // 8 warps
constexpr uint32_t WAIT_LIMIT = 1u << 26;

// ---- shared memory layout (byte offsets from a 1024-aligned base) ----------
// SW128 tiles: [rows x 128] bf16 as two [rows x 64] halves.
constexpr int OFF_KQ = 0;           // [K h0 | Q h0 | K h1 | Q h1], 8 KB each
constexpr int KQ_HALF = 16384;      // distance between the two column halves
constexpr int OFF_Q = 8192;         // Q h0 (Q h1 at OFF_Q + KQ_HALF)
constexpr int OFF_V = 32768;        // [64 x 128], halves 8 KB apart
constexpr int OFF_HT = 49152;       // S^T bf16 [128 v x 128 kk], halves 16 KB apart
constexpr int OFF_W = 81920;        // w bf16 [64 t x 128 kk], halves 8 KB apart
constexpr int OFF_VN = 98304;       // v_new^T bf16 [128 v x 64 t]
constexpr int OFF_VTH = 114688;     // vt hi [128 x 64]
constexpr int OFF_VTL = 131072;     // vt lo [128 x 64]
constexpr int OFF_TP = 147456;      // T'  [64 i x 64 j]
constexpr int OFF_TPP = 155648;     // T'' [64 x 64]
constexpr int OFF_AQK = 163840;     // Aqk [64 x 64]
constexpr int OFF_FA = 172032;      // fp32 A  [64 x LDF]
constexpr int OFF_FT = OFF_FA + 64 * LDF * 4;   // fp32 T
constexpr int OFF_FM = OFF_FT + 64 * LDF * 4;   // fp32 scratch 32 x 33
constexpr int OFF_G = OFF_FM + 32 * 33 * 4;     // graw[64], gc[64], beta[64]
constexpr int SMEM_USED = OFF_G + 3 * 64 * 4;
constexpr int SMEM_BYTES = SMEM_USED + 1024;    // + alignment slack

// TMEM columns
constexpr uint32_t TM_S = 0, TM_G = 128, TM_U = 192, TM_QH = 256, TM_W = 320, TM_O = 384;
constexpr uint32_t TM_COLS = 512;

__device__ __forceinline__ uint64_t kdesc(uint32_t tile, uint32_t half_stride, int kstep) {
  return tc::smem_desc(tile + (uint32_t)((kstep >> 2) * half_stride + (kstep & 3) * 32), 16, 1024);
}
__device__ __forceinline__ uint64_t kdesc64(uint32_t tile, int kstep) {
  return tc::smem_desc(tile + (uint32_t)(kstep * 32), 16, 1024);
}
// MN-major: tile rows = K index (16 per k-step), LBO = distance between MN halves
__device__ __forceinline__ uint64_t mndesc(uint32_t tile, uint32_t half_stride, int kstep) {
  return tc::smem_desc(tile + (uint32_t)(kstep * 2048), half_stride, 1024);
}

// 16-byte chunk c (0..15) of row r of a [rows x 128] SW128 tile
__device__ __forceinline__ uint32_t chunk_off(int r, int c, uint32_t half_stride) {
  return (uint32_t)((c >> 3) * half_stride + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}
// element (r, col) of a SW128 tile
__device__ __forceinline__ uint32_t elem_off(int r, int col, uint32_t half_stride) {
  return (uint32_t)((col >> 6) * half_stride + r * 128 + ((((col & 63) >> 3) ^ (r & 7)) << 4) +
                    (col & 7) * 2);
}

__device__ __forceinline__ void load_tile_sw128(unsigned char* base, uint32_t half_stride,
                                                const bf16* src, int64_t stride, int L, int tid) {
  for (int e = tid; e < 64 * 16; e += NT) {
    const int r = e >> 4, c = e & 15;
    const bool ok = r < L;
    cp_async16(base + chunk_off(r, c, half_stride), src + (int64_t)(ok ? r : 0) * stride + c * 8,
               ok ? 16 : 0);
  }
}

// L2-normalise rows [r0, r0+16) of a [64 x 128] SW128 tile in place (one warp)
__device__ __forceinline__ void l2norm_rows(unsigned char* base, uint32_t half_stride, int r0,
                                            int lane) {
  for (int r = r0; r < r0 + 16; ++r) {
    // lane owns elements 4*lane .. 4*lane+3 (column order does not matter)
    const int col = 4 * lane;
    __nv_bfloat162* p = reinterpret_cast<__nv_bfloat162*>(base + elem_off(r, col, half_stride));
    float2 a = __bfloat1622float2(p[0]), b = __bfloat1622float2(p[1]);
    const float ss = warp_sum(a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y);
    const float rn = rsqrtf(ss + 1e-6f);
    p[0] = __floats2bfloat162_rn(a.x * rn, a.y * rn);
    p[1] = __floats2bfloat162_rn(b.x * rn, b.y * rn);
  }
}

__device__ __forceinline__ uint32_t tm_addr(uint32_t base, int lane_quarter, uint32_t col) {
  return base + ((uint32_t)(lane_quarter * 32) << 16) + col;
}

__global__ void __launch_bounds__(NT, 1) chunk_gdn_tc_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v,
    const float* __restrict__ g, const float* __restrict__ beta, const float* __restrict__ h0,
    bf16* __restrict__ o, float* __restrict__ ht, const int32_t* __restrict__ cu, int64_t T,
    int64_t Hg, int64_t H, int64_t q_stride, int64_t k_stride, int64_t v_stride, float scale,
    bool l2norm) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_base_sh;
  __shared__ int abort_flag;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quarter = warp & 3;      // TMEM lane quarter this warp may access
  const int colhalf = warp >> 2;     // which 32-column half of a 64-column region
  const int64_t n = blockIdx.x / H;
  const int h = (int)(blockIdx.x - n * H);
  const int hk = (int)(h / (H / Hg));
  int64_t bos, eos;
  seq_span(cu, n, T, bos, eos);
  constexpr int K = 128, V = 128;

  float* graw = reinterpret_cast<float*>(sm + OFF_G);
  float* gcs = graw + 64;
  float* bet = gcs + 64;
  const uint32_t s_base = tc::smem_addr(sm);

  if (warp == 0) {
    tc::tmem_alloc(&tmem_base_sh, TM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::mbar_fence_init();
    abort_flag = 0;
  }
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = tmem_base_sh;
  uint32_t phase = 0;

  // wait for the MMAs committed so far; returns false after a timeout
  auto mma_wait = [&]() -> bool {
    const bool ok = tc::mbar_wait(&bar, phase, WAIT_LIMIT);
    phase ^= 1u;
    if (!ok) {
      atomicExch(&abort_flag, 1);
      atomicExch(&g_tc_error, 1);
    }
    tc::fence_after();
    __syncthreads();
    return abort_flag == 0;
  };

  // ---- initial state into TMEM: S^T[v][kk] = h0[kk][v] ---------------------
  {
    const int vrow = quarter * 32 + lane;
    const float* src = h0 ? h0 + ((int64_t)n * H + h) * K * V : nullptr;
#pragma unroll
    for (int cb = 0; cb < 2; ++cb) {
      const int c0 = colhalf * 64 + cb * 32;
      float vals[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) vals[i] = src ? src[(c0 + i) * V + vrow] : 0.f;
      tc::tmem_st32(tm_addr(tm, quarter, TM_S + c0), vals);
    }
    tc::tmem_wait_st();
  }

  const int64_t o_stride = H * V;
  bool ok = true;
  for (int64_t t0 = bos; t0 < eos && ok; t0 += BT) {
    const int L = (int)((eos - t0) < BT ? (eos - t0) : BT);
    // ---- P0: tiles, gates, cumsum -------------------------------------------
    load_tile_sw128(sm + OFF_KQ, KQ_HALF, k + t0 * k_stride + (int64_t)hk * K, k_stride, L, tid);
    load_tile_sw128(sm + OFF_Q, KQ_HALF, q + t0 * q_stride + (int64_t)hk * K, q_stride, L, tid);
    load_tile_sw128(sm + OFF_V, 8192, v + t0 * v_stride + (int64_t)h * V, v_stride, L, tid);
    cp_async_commit();
    if (tid < BT) {
      graw[tid] = tid < L ? g[(t0 + tid) * H + h] : 0.f;
      bet[tid] = tid < L ? beta[(t0 + tid) * H + h] : 0.f;
    }
    __syncthreads();
    if (warp == 0) chunk_cumsum_warp(graw, gcs, lane);
    cp_async_wait_all();
    __syncthreads();
    const float gl = gcs[L - 1];
    if (l2norm) l2norm_rows(sm + (warp < 4 ? OFF_KQ : OFF_Q), KQ_HALF, 16 * (warp & 3), lane);
    // state -> bf16 S^T tile (A operand) and rescale the fp32 state by e^{gl}
    {
      const int vrow = quarter * 32 + lane;
      const float dl = __expf(gl);
#pragma unroll
      for (int cb = 0; cb < 2; ++cb) {
        const int c0 = colhalf * 64 + cb * 32;
        float vals[32];
        tc::tmem_ld32(tm_addr(tm, quarter, TM_S + c0), vals);
        tc::tmem_wait_ld();
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          uint4 pk;
          pk.x = pack_bf16(vals[c], vals[c + 1]);
          pk.y = pack_bf16(vals[c + 2], vals[c + 3]);
          pk.z = pack_bf16(vals[c + 4], vals[c + 5]);
          pk.w = pack_bf16(vals[c + 6], vals[c + 7]);
          *reinterpret_cast<uint4*>(sm + OFF_HT + chunk_off(vrow, (c0 + c) >> 3, 16384)) = pk;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) vals[i] *= dl;
        tc::tmem_st32(tm_addr(tm, quarter, TM_S + c0), vals);
      }
      tc::tmem_wait_st();
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();

    // ---- P1: Gram [k;q] k^T and q-state product ------------------------------
    if (tid == 0) {
      const uint32_t idG = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        tc::mma_bf16(tm + TM_G, kdesc(s_base + OFF_KQ, KQ_HALF, j),
                     kdesc(s_base + OFF_KQ, KQ_HALF, j), idG, j > 0);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        tc::mma_bf16(tm + TM_QH, kdesc(s_base + OFF_HT, 16384, j),
                     kdesc(s_base + OFF_Q, KQ_HALF, j), idG, j > 0);
      tc::commit(&bar);
    }
    if (!(ok = mma_wait())) break;

    // ---- P2: Gram epilogue: A (fp32, strictly lower) and Aqk (bf16) ----------
    {
      const int row = quarter * 32 + lane;  // 0..63 k rows, 64..127 q rows
      const int c0 = colhalf * 32;
      float vals[32];
      tc::tmem_ld32(tm_addr(tm, quarter, TM_G + c0), vals);
      tc::tmem_wait_ld();
      if (row < 64) {
        float* fa = reinterpret_cast<float*>(sm + OFF_FA);
        const float bi = bet[row], gi = gcs[row];
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          const int j = c0 + c;
          fa[row * LDF + j] = (j < row) ? vals[c] * bi * __expf(fminf(gi - gcs[j], 0.f)) : 0.f;
        }
      } else {
        const int i = row - 64;
        const float gi = gcs[i];
#pragma unroll
        for (int c = 0; c < 32; c += 8) {
          float e[8];
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            const int j = c0 + c + u;
            e[u] = (j <= i) ? vals[c + u] * __expf(fminf(gi - gcs[j], 0.f)) : 0.f;
          }
          uint4 pk;
          pk.x = pack_bf16(e[0], e[1]); pk.y = pack_bf16(e[2], e[3]);
          pk.z = pack_bf16(e[4], e[5]); pk.w = pack_bf16(e[6], e[7]);
          *reinterpret_cast<uint4*>(sm + OFF_AQK + (uint32_t)(i * 128 + ((((c0 + c) >> 3) ^ (i & 7)) << 4))) = pk;
        }
      }
    }
    __syncthreads();

    // ---- P3: T = (I + A)^-1; T' = (T - I) diag(beta), T'' = T diag(beta e^gc) --
    {
      float* fa = reinterpret_cast<float*>(sm + OFF_FA);
      float* ft = reinterpret_cast<float*>(sm + OFF_FT);
      float* fm = reinterpret_cast<float*>(sm + OFF_FM);
      tri_inverse_64(fa, ft, fm, tid);
      for (int e = tid; e < 64 * 8; e += NT) {
        const int i = e >> 3, cchunk = e & 7;
        float tp[8], tpp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = cchunk * 8 + u;
          const float tv = ft[i * LDF + j] * bet[j];
          tp[u] = (i == j) ? 0.f : tv;
          tpp[u] = tv * __expf(gcs[j]);
        }
        const uint32_t off = (uint32_t)(i * 128 + ((cchunk ^ (i & 7)) << 4));
        uint4 a, b;
        a.x = pack_bf16(tp[0], tp[1]); a.y = pack_bf16(tp[2], tp[3]);
        a.z = pack_bf16(tp[4], tp[5]); a.w = pack_bf16(tp[6], tp[7]);
        b.x = pack_bf16(tpp[0], tpp[1]); b.y = pack_bf16(tpp[2], tpp[3]);
        b.z = pack_bf16(tpp[4], tpp[5]); b.w = pack_bf16(tpp[6], tpp[7]);
        *reinterpret_cast<uint4*>(sm + OFF_TP + off) = a;
        *reinterpret_cast<uint4*>(sm + OFF_TPP + off) = b;
      }
    }
    tc::fence_proxy_async();
    __syncthreads();

    // ---- P4: u^T = v^T T'^T, w^T = k^T T''^T ---------------------------------
    if (tid == 0) {
      const uint32_t idMN = tc::idesc_bf16(128, 64, true, false);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        tc::mma_bf16(tm + TM_U, mndesc(s_base + OFF_V, 8192, j), kdesc64(s_base + OFF_TP, j), idMN,
                     j > 0);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        tc::mma_bf16(tm + TM_W, mndesc(s_base + OFF_KQ, KQ_HALF, j), kdesc64(s_base + OFF_TPP, j),
                     idMN, j > 0);
      tc::commit(&bar);
    }
    if (!(ok = mma_wait())) break;

    // ---- P5: w (bf16, [t][kk]) from w^T in TMEM ------------------------------
    {
      const int kk = quarter * 32 + lane;
      const int c0 = colhalf * 32;
      float vals[32];
      tc::tmem_ld32(tm_addr(tm, quarter, TM_W + c0), vals);
      tc::tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c)
        *reinterpret_cast<bf16*>(sm + OFF_W + elem_off(c0 + c, kk, 8192)) = __float2bfloat16_rn(vals[c]);
    }
    tc::fence_proxy_async();
    __syncthreads();

    // ---- P6: D_u += S^T (-w)^T ------------------------------------------------
    if (tid == 0) {
      const uint32_t idN = tc::idesc_bf16(128, 64, false, false, /*neg_b=*/true);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        tc::mma_bf16(tm + TM_U, kdesc(s_base + OFF_HT, 16384, j), kdesc(s_base + OFF_W, 8192, j),
                     idN, true);
      tc::commit(&bar);
    }
    if (!(ok = mma_wait())) break;

    // ---- P7: v_new, vt hi/lo, o_inter -> TMEM ---------------------------------
    {
      const int vrow = quarter * 32 + lane;
      const int c0 = colhalf * 32;  // tokens c0 .. c0+31
      float du[32], qh[32];
      tc::tmem_ld32(tm_addr(tm, quarter, TM_U + c0), du);
      tc::tmem_ld32(tm_addr(tm, quarter, TM_QH + c0), qh);
      tc::tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        float vn[8], th[8], tl[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int i = c0 + c + u;
          const float vi = __bfloat162float(
              *reinterpret_cast<const bf16*>(sm + OFF_V + elem_off(i, vrow, 8192)));
          vn[u] = du[c + u] + bet[i] * vi;
          const float s = vn[u] * __expf(fminf(gl - gcs[i], 0.f));
          th[u] = __bfloat162float(__float2bfloat16_rn(s));
          tl[u] = s - th[u];
          qh[c + u] *= __expf(gcs[i]);
        }
        const uint32_t off = (uint32_t)(vrow * 128 + ((((c0 + c) >> 3) ^ (vrow & 7)) << 4));
        uint4 a, b2, d;
        a.x = pack_bf16(vn[0], vn[1]); a.y = pack_bf16(vn[2], vn[3]);
        a.z = pack_bf16(vn[4], vn[5]); a.w = pack_bf16(vn[6], vn[7]);
        b2.x = pack_bf16(th[0], th[1]); b2.y = pack_bf16(th[2], th[3]);
        b2.z = pack_bf16(th[4], th[5]); b2.w = pack_bf16(th[6], th[7]);
        d.x = pack_bf16(tl[0], tl[1]); d.y = pack_bf16(tl[2], tl[3]);
        d.z = pack_bf16(tl[4], tl[5]); d.w = pack_bf16(tl[6], tl[7]);
        *reinterpret_cast<uint4*>(sm + OFF_VN + off) = a;
        *reinterpret_cast<uint4*>(sm + OFF_VTH + off) = b2;
        *reinterpret_cast<uint4*>(sm + OFF_VTL + off) = d;
      }
      tc::tmem_st32(tm_addr(tm, quarter, TM_O + c0), qh);
      tc::tmem_wait_st();
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();

    // ---- P8: S^T += vt^T k ; D_o += v_new^T Aqk^T ------------------------------
    if (tid == 0) {
      const uint32_t idS = tc::idesc_bf16(128, 128, false, true);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        tc::mma_bf16(tm + TM_S, kdesc64(s_base + OFF_VTH, j), mndesc(s_base + OFF_KQ, KQ_HALF, j),
                     idS, true);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        tc::mma_bf16(tm + TM_S, kdesc64(s_base + OFF_VTL, j), mndesc(s_base + OFF_KQ, KQ_HALF, j),
                     idS, true);
      const uint32_t idO = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        tc::mma_bf16(tm + TM_O, kdesc64(s_base + OFF_VN, j), kdesc64(s_base + OFF_AQK, j), idO,
                     true);
      tc::commit(&bar);
    }
    if (!(ok = mma_wait())) break;

    // ---- P9: o = scale * D_o ----------------------------------------------------
    {
      const int vrow = quarter * 32 + lane;
      const int c0 = colhalf * 32;
      float ov[32];
      tc::tmem_ld32(tm_addr(tm, quarter, TM_O + c0), ov);
      tc::tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) {
        const int i = c0 + c;
        if (i < L) o[(t0 + i) * o_stride + (int64_t)h * V + vrow] = __float2bfloat16_rn(ov[c] * scale);
      }
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
  }

  if (ok && ht) {
    const int vrow = quarter * 32 + lane;
    float* dst = ht + ((int64_t)n * H + h) * K * V;
#pragma unroll
    for (int cb = 0; cb < 2; ++cb) {
      const int c0 = colhalf * 64 + cb * 32;
      float vals[32];
      tc::tmem_ld32(tm_addr(tm, quarter, TM_S + c0), vals);
      tc::tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) dst[(c0 + i) * V + vrow] = vals[i];
    }
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, TM_COLS);
}

}  // namespace
}  // namespace gdn
}  // namespace xops

using namespace xops;

extern "C" int xops_chunk_gated_delta_rule(const void* q, const void* k, const void* v,
                                           const float* g, const float* beta, const float* h0,
                                           void* o, float* ht, const int32_t* cu_seqlens,
                                           int64_t B, int64_t T, int64_t N, int64_t Hg,
                                           int64_t H, int64_t K, int64_t V,
                                           int64_t q_token_stride, int64_t k_token_stride,
                                           int64_t v_token_stride, float scale,
                                           int use_qk_l2norm_in_kernel, void* stream) {
  XOPS_REQUIRE(B >= 1 && T >= 0 && N >= 0 && Hg >= 1 && H >= 1,
               "chunk_gated_delta_rule: bad shape");
  XOPS_REQUIRE(H % Hg == 0,
               "chunk_gated_delta_rule expects num_heads_v to be divisible by num_heads_qk, got "
               "%lld and %lld", (long long)H, (long long)Hg);
  XOPS_REQUIRE(cu_seqlens || N == B, "chunk_gated_delta_rule: without cu_seqlens N must equal B");
  XOPS_REQUIRE(!cu_seqlens || B == 1, "chunk_gated_delta_rule: cu_seqlens requires B == 1");
  XOPS_UNSUPPORTED(K == 128 && V == 128,
                   "chunk_gated_delta_rule: only K == V == 128 is compiled (got %lld, %lld)",
                   (long long)K, (long long)V);
  if (q_token_stride == 0) q_token_stride = Hg * K;
  if (k_token_stride == 0) k_token_stride = Hg * K;
  if (v_token_stride == 0) v_token_stride = H * V;
  XOPS_REQUIRE(q_token_stride >= Hg * K && k_token_stride >= Hg * K && v_token_stride >= H * V &&
                   q_token_stride % 8 == 0 && k_token_stride % 8 == 0 && v_token_stride % 8 == 0,
               "chunk_gated_delta_rule: token strides must cover the heads and be multiples of 8");
  if (N == 0 || T == 0) return XOPS_OK;
  XOPS_REQUIRE(q && k && v && g && beta && o, "chunk_gated_delta_rule: null pointer");
  XOPS_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o),
               "chunk_gated_delta_rule: tensors must be 16-byte aligned");
  const size_t smem = gdn::SMEM_BYTES;
  if (int rc = gdn::ensure_smem_attr((const void*)gdn::chunk_gdn_tc_kernel, smem,
                                     "chunk_gated_delta_rule"))
    return rc;
  gdn::chunk_gdn_tc_kernel<<<(unsigned)(N * H), gdn::NT, smem, (cudaStream_t)stream>>>(
      (const gdn::bf16*)q, (const gdn::bf16*)k, (const gdn::bf16*)v, g, beta, h0, (gdn::bf16*)o,
      ht, cu_seqlens, T, Hg, H, q_token_stride, k_token_stride, v_token_stride, scale,
      use_qk_l2norm_in_kernel != 0);
  return check_launch("chunk_gated_delta_rule");
}

extern "C" int xops_device_error_count(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gdn::g_tc_error, sizeof(int)) != cudaSuccess) return -1;
  const int zero = 0;
  cudaMemcpyToSymbol(gdn::g_tc_error, &zero, sizeof(int));
  return v;
}
