// Chunked gated delta rule prefill on the sm_100a tensor cores.
//
// Two kernels, both built on tcgen05.mma (M = 128, bf16 operands from
// 128-byte-swizzled shared tiles, fp32 accumulators in TMEM):
//
// 1. chunk_prep_kernel -- fully parallel over (64-token chunk, key head).
//    Everything of a chunk that does not depend on the recurrent state:
//      G    = [k; q] k^T                          (one MMA, shared by the
//                                                  value heads of the key head)
//      A    = strict_tril(beta_i D_ij (k k^T)_ij),  D_ij = e^{gc_i - gc_j}
//      T    = (I + A)^-1                          (for two value heads per key
//                                                  head: 16 x 16 diagonal blocks
//                                                  in registers, the rest as
//                                                  tf32 tcgen05 products; else
//                                                  blocked fp32 on CUDA cores)
//      T'   = T diag(beta)                        -> workspace (bf16)
//      -w   = -T diag(beta e^{gc}) k              (MMA)   -> workspace (bf16)
//      Aqk  = tril(q k^T * D)                     -> workspace (bf16)
//    per value head, where gc is the in-chunk cumsum of g.
//
// 2. chunk_chain_kernel -- one CTA per work item (a run of chunks of one
//    sequence and value head) walks the chunks in order.  Warp-specialised:
//    warp 0 prefetches the next chunk's tiles (k, q, v by TMA from the
//    inputs; w, T', Aqk by bulk copy from the workspace) into a second
//    stage; warp 1 issues every MMA from one thread; warps 2-17 hold the
//    fp32 state S^T[v][kk] in registers (32 values per thread) and run the
//    epilogues.  Per chunk:
//      D_u   = v^T T'^T + v^T diag(beta - bf16(beta))   (issued one chunk ahead)
//      [D_u | D_qh] += S^T [-w; q]^T  (one N = 128 product; v_new^T = D_u with
//                                      beta_i v_i kept fp32, D_qh = S^T q^T)
//      dS    = vt_hi^T k + vt_lo^T k,  vt = v_new e^{gc_last - gc} split bf16 hi+lo
//      D_o   = e^{gc} D_qh + v_new^T Aqk^T   (the product issued behind the
//                                             next chunk's [-w; q] product)
//      S    <- e^{gc_last} S + dS,  o = scale * D_o
//    The beta_i v_i diagonal term stays fp32 and the hi/lo split keeps the
//    fp32 state within ~1e-5 of the fp32 recurrence.
//
// The workspace (chunks x value heads x 32 KB, plus L2-normalised q/k when
// use_qk_l2norm_in_kernel) replaces the reference's A, Ai, w, u, h and v_new
// intermediates (npu_triton_chunk_gated_delta_rule.cpp:556-642); per-chunk
// states and v_new never leave the SM.
//
// Every wait is a bounded mbarrier poll: on timeout the CTA records an
// error in a device flag (xops_device_error_count) and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "gate_math.cuh"
#include "gdn_common.cuh"
#include "gdn_tc.cuh"
#include "tcgen05.cuh"

namespace xops {
namespace gdn {

__device__ int g_tc_error = 0;

namespace {

constexpr uint32_t WAIT_LIMIT = 1u << 26;
constexpr int WS_CHUNK = 33280;   // workspace bytes per (chunk, value head)
// -w image, T' image, Aqk image, then the chunk's gates as the preparation
// read or computed them: g[64], beta[64] fp32 (zero past the sequence end),
// so the chain reads one contiguous row and never evaluates a gate
constexpr int WS_W = 0, WS_TP = 16384, WS_AQK = 24576, WS_GB = 32768;

__device__ __forceinline__ void record_error() { atomicExch(&g_tc_error, 1); }

// Gates of the rule per (token, value head): precomputed g / beta [T, H]
// fp32, or computed where they are read from the layer's projections a, b
// [T, H] (the fused-gating entry) with the arithmetic of fused_gdn_gating
// (gate_math.cuh), so both entries see the same values bit for bit.
struct GateSrc {
  const float* g;     // precomputed gates; nullptr: computed from a / b
  const float* beta;
  const void* a;
  const void* b;
  const float* A_log;
  const float* dt_bias;
  float sp_beta, sp_thr;
  int a_dt, b_dt;     // XOPS_F32 / XOPS_BF16 / XOPS_F16
  int64_t ab_ld;      // elements between tokens of a and b
  int ba_r;           // 0: a, b [T, H]; r > 0: a = b = mixed_ba, per key head b (r) | a (r)
};
__device__ __forceinline__ float gate_elem(const void* p, int dt, int64_t i) {
  return dt == XOPS_BF16 ? __bfloat162float(static_cast<const bf16*>(p)[i])
         : dt == XOPS_F16 ? __half2float(static_cast<const __half*>(p)[i])
                          : static_cast<const float*>(p)[i];
}
__device__ __forceinline__ void gate_load(const GateSrc& s, int64_t t, int64_t H, int h, float& g,
                                          float& beta) {
  const int64_t i = t * H + h;
  if (s.g) {
    g = s.g[i];
    beta = s.beta[i];
    return;
  }
  int64_t ia = t * s.ab_ld + h, ib = ia;
  if (s.ba_r) {
    ib = t * s.ab_ld + (int64_t)(h / s.ba_r) * 2 * s.ba_r + h % s.ba_r;
    ia = ib + s.ba_r;
  }
  g = gate_g(-expf(s.A_log[h]), gate_elem(s.a, s.a_dt, ia), s.dt_bias[h], s.sp_beta, s.sp_thr);
  const float bv = gate_elem(s.b, s.b_dt, ib);
  beta = s.b_dt == XOPS_BF16  ? gate_beta<bf16>(bv)
         : s.b_dt == XOPS_F16 ? gate_beta<__half>(bv)
                              : gate_beta<float>(bv);
}

// ============================================================================
// q/k L2 normalisation pre-pass: x / sqrt(sum x^2 + 1e-6) per 128-wide head,
// rounded to bf16 (npu_l2norm_last_dim, npu_triton_chunk_gated_delta_rule.cpp:608-609).
// One warp per (token, head); reads strided token rows, writes contiguous.
// ============================================================================
__global__ void __launch_bounds__(256) l2norm_heads_kernel(const bf16* __restrict__ x,
                                                           bf16* __restrict__ y, int64_t rows,
                                                           int64_t heads, int64_t tstride) {
  const int lane = threadIdx.x & 31;
  const int64_t r = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  const int64_t t = r / heads, hh = r - t * heads;
  const uint2 raw = *reinterpret_cast<const uint2*>(x + t * tstride + hh * 128 + lane * 4);
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&raw);
  const float2 a = __bfloat1622float2(p[0]), b = __bfloat1622float2(p[1]);
  const float rn = rsqrtf(warp_sum(a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y) + 1e-6f);
  uint2 out;
  out.x = pack_bf16(a.x * rn, a.y * rn);
  out.y = pack_bf16(b.x * rn, b.y * rn);
  *reinterpret_cast<uint2*>(y + r * 128 + lane * 4) = out;
}


// ============================================================================
// Kernel 1: per-chunk preparation
// ============================================================================
constexpr int P_NT = 256;
constexpr int P_OFF_KQ = 0;        // [K h0 | Q h0 | K h1 | Q h1], 8 KB each
constexpr int P_KQ_HALF = 16384;
constexpr int P_OFF_Q = 8192;
// q is dead once the Gram product has read it: its two 8 KB halves then hold
// T'' (SW128, for the w product) and the inverse's scratch, which keeps the
// CTA at ~50 KB so four fit on an SM
constexpr int P_OFF_TPP = P_OFF_Q;            // T'' [64 x 64] SW128
constexpr int P_OFF_FM = P_OFF_Q + P_KQ_HALF; // inverse scratch (<= 32 x 33 fp32)
constexpr int P_OFF_FA = 32768;    // fp32 A, then T = (I+A)^-1 in place [64 x LDF]
constexpr int P_OFF_G = P_OFF_FA + 64 * LDF * 4;  // graw, gc, beta, e^gc
constexpr int P_SMEM = P_OFF_G + 4 * 64 * 4 + 1024;
constexpr uint32_t P_TM_G = 0, P_TM_W = 64, P_TM_COLS = 128;

__global__ void __launch_bounds__(P_NT, 4) chunk_prep_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const GateSrc gs,
    unsigned char* __restrict__ ws,
    const int32_t* __restrict__ cu, int64_t N, int64_t T, int64_t Hg, int64_t H,
    int64_t q_stride, int64_t k_stride) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_sh;
  __shared__ int64_t pos[4];
  __shared__ int ok_sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quarter = warp & 3, colhalf = warp >> 2;
  const int hk = blockIdx.y;
  if (tid == 0) {
    int64_t seq = 0, t0 = 0, eos = 0, cis = 0;
    const bool ok = locate_chunk(cu, N, T, blockIdx.x, seq, t0, eos, cis);
    pos[0] = ok ? chunk_offset(cu, seq, T) + cis : -1;
    pos[1] = t0;
    pos[2] = eos;
    ok_sh = ok ? 1 : 0;
  }
  __syncthreads();
  if (!ok_sh) return;
  const int64_t gci = pos[0], t0 = pos[1];
  const int L = (int)((pos[2] - t0) < BT ? (pos[2] - t0) : BT);
  float* graw = reinterpret_cast<float*>(sm + P_OFF_G);
  float* gcs = graw + 64;
  float* bet = gcs + 64;
  float* egc = bet + 64;
  const uint32_t sb = tc::smem_addr(sm);

  if (warp == 0) {
    tc::tmem_alloc(&tmem_sh, P_TM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::mbar_fence_init();
  }
  cp_tile128(sm + P_OFF_KQ, P_KQ_HALF, k + t0 * k_stride + (int64_t)hk * 128, k_stride, L, tid, P_NT);
  cp_tile128(sm + P_OFF_Q, P_KQ_HALF, q + t0 * q_stride + (int64_t)hk * 128, q_stride, L, tid, P_NT);
  cp_async_commit();
  // gates of the first value head load while k and q land; each head's
  // loop iteration fetches the next head's
  const int grp = (int)(H / Hg);
  float g_next = 0.f, b_next = 0.f;
  if (tid < L) {
    gate_load(gs, t0 + tid, H, hk * grp, g_next, b_next);
  }
  cp_async_wait_all();
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = tmem_sh;
  uint32_t phase = 0;
  bool alive = true;
  if (tid == 0) {
    const uint32_t id = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      tc::mma_bf16(tm + P_TM_G, kdesc(sb + P_OFF_KQ, P_KQ_HALF, j), kdesc(sb + P_OFF_KQ, P_KQ_HALF, j),
                   id, j > 0);
    tc::commit(&bar);
  }
  auto wait_mma = [&]() {
    const bool ok = tc::mbar_wait(&bar, phase, WAIT_LIMIT);
    phase ^= 1u;
    if (!ok) {
      record_error();
      atomicExch(&ok_sh, 0);
    }
    tc::fence_after();
    __syncthreads();
    alive = ok_sh != 0;
  };
  wait_mma();

  for (int hv = hk * grp; alive && hv < (hk + 1) * grp; ++hv) {
    unsigned char* wsb = ws + (gci * H + hv) * (int64_t)WS_CHUNK;
    if (tid < 64) {
      graw[tid] = g_next;
      bet[tid] = b_next;
      reinterpret_cast<float*>(wsb + WS_GB)[tid] = g_next;
      reinterpret_cast<float*>(wsb + WS_GB)[64 + tid] = b_next;
      g_next = b_next = 0.f;
      if (tid < L && hv + 1 < (hk + 1) * grp) {
        gate_load(gs, t0 + tid, H, hv + 1, g_next, b_next);
      }
    }
    __syncthreads();
    if (warp == 0) {
      chunk_cumsum_warp(graw, gcs, lane);
      __syncwarp();
      egc[lane] = __expf(gcs[lane]);
      egc[lane + 32] = __expf(gcs[lane + 32]);
    }
    __syncthreads();
    // Gram epilogue
    {
      const int row = quarter * 32 + lane;
      const int c0 = colhalf * 32;
      float vals[32];
      tc::tmem_ld32(tm_addr(tm, quarter, P_TM_G + c0), vals);
      tc::tmem_wait_ld();
      if (row < 64) {
        float* fa = reinterpret_cast<float*>(sm + P_OFF_FA);
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
          *reinterpret_cast<uint4*>(wsb + WS_AQK + chunk_off(i, (c0 + c) >> 3, 0)) = pk;
        }
      }
    }
    __syncthreads();
    {
      float* ft = reinterpret_cast<float*>(sm + P_OFF_FA);
      float* fm = reinterpret_cast<float*>(sm + P_OFF_FM);
      tri_inverse_64_inplace(ft, fm, tid);
      for (int e = tid; e < 64 * 8; e += P_NT) {
        const int i = e >> 3, cc = e & 7;
        float tp[8], tpp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = cc * 8 + u;
          const float tv = ft[i * LDF + j] * bet[j];
          tp[u] = tv;  // diagonal = bf16(beta_i); the chain adds beta_i - bf16(beta_i)
          tpp[u] = tv * egc[j];
        }
        uint4 a, b;
        a.x = pack_bf16(tp[0], tp[1]); a.y = pack_bf16(tp[2], tp[3]);
        a.z = pack_bf16(tp[4], tp[5]); a.w = pack_bf16(tp[6], tp[7]);
        b.x = pack_bf16(tpp[0], tpp[1]); b.y = pack_bf16(tpp[2], tpp[3]);
        b.z = pack_bf16(tpp[4], tpp[5]); b.w = pack_bf16(tpp[6], tpp[7]);
        *reinterpret_cast<uint4*>(wsb + WS_TP + chunk_off(i, cc, 0)) = a;
        *reinterpret_cast<uint4*>(sm + P_OFF_TPP + (uint32_t)(i * 128 + ((cc ^ (i & 7)) << 4))) = b;
      }
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (tid == 0) {
      const uint32_t id = tc::idesc_bf16(128, 64, true, false);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        tc::mma_bf16(tm + P_TM_W, mndesc(sb + P_OFF_KQ, P_KQ_HALF, j), kdesc64(sb + P_OFF_TPP, j), id,
                     j > 0);
      tc::commit(&bar);
    }
    wait_mma();
    if (!alive) break;
    {  // -w [t][kk] (bf16, row-major) from w^T in TMEM (lane = kk); stored
       // negated so the chain forms [-w; q] S in one N = 128 product
      const int kk = quarter * 32 + lane;
      const int c0 = colhalf * 32;
      float vals[32];
      tc::tmem_ld32(tm_addr(tm, quarter, P_TM_W + c0), vals);
      tc::tmem_wait_ld();
      // c0 is a multiple of 8, so the swizzle of token c0 + c depends on c & 7 only
      unsigned char* wrow = wsb + WS_W + (kk >> 6) * 8192 + (kk & 7) * 2 + c0 * 128;
      const int kc = (kk & 63) >> 3;
#pragma unroll
      for (int c = 0; c < 32; ++c)
        *reinterpret_cast<bf16*>(wrow + c * 128 + ((kc ^ (c & 7)) << 4)) =
            __float2bfloat16_rn(-vals[c]);
    }
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, P_TM_COLS);
}

// TMEM columns of the two heads' -w accumulators in the paired preparation
constexpr uint32_t P2_TM_W0 = 0, P2_TM_W1 = 64;

// ----------------------------------------------------------------------------
// Kernel 1c: the pair preparation with the triangular inverse on the tensor
// cores.  Let D = I + (the four 16 x 16 diagonal blocks of A) and L = the
// rest of A (strictly block-lower).  Then I + A = D (I + N) with
// N = D^-1 L, nilpotent of index 4, so
//     T = (I + A)^-1 = (I - N + N^2 - N^3) D^-1 = X_3,
//     X_0 = D^-1,  X_{r+1} = D^-1 + (-N) X_r.
// D^-1 is solved in registers by the two warps that hold those rows in the
// Gram epilogue (row-wise forward substitution, rows broadcast by shuffle).
// N and the three X products are tcgen05 kind::tf32 products with both
// heads stacked (M = 128 rows (head, row), N = 128 columns (head, column));
// each thread reads only its own head's quadrant.  Only 48 of the 64
// contraction indices carry anything: L's first block row and N's last
// block column are zero, so N = D^-1 L runs over rows 16..63 of L and the
// X products over columns 0..47 of N.  Operands are rounded to tf32
// (nearest) as they are written, so the inverse's error stays well below
// the bf16 rounding of T' and T'' that follows.  The 32 x 32 blocks above
// the diagonal are zero in A, L, D^-1, N and every X: the warps that own
// them only write zeros where a later reader needs them.
//
// Operand tiles (fp32, K-major, 128 rows): contraction indices 0-31 in an
// SW128 part (128-byte rows, 16-byte chunk c of row r at c ^ (r & 7)),
// 32-47 in an SW64 part (64-byte rows, chunk c at c ^ ((r >> 1) & 3)) that
// lives in a q tile left dead by the Gram product.  That keeps the CTA at
// ~69 KB, three per SM.  The A tile's rows are (head, row) and are written a
// row at a time; the B tile's rows are (head, column) with K = the row of
// the matrix, so a thread holding a matrix row writes one element into
// each of 32 B rows (one 128-byte warp store per column).  Aqk goes
// straight to the workspace; the T' and -w images are staged in shared
// memory and leave by bulk copy.
// ----------------------------------------------------------------------------
constexpr int P3_OFF_AM = 32768;     // A tile, K 0..31: D^-1 (shifted), then -N; later T''
constexpr int P3_OFF_BM = 49152;     // B tile, K 0..31: L (shifted), then X_r; later T'
constexpr int P3_OFF_AT = P_OFF_Q;              // A tile, K 32..47 (in the dead q half 0)
constexpr int P3_OFF_BT = P_OFF_Q + P_KQ_HALF;  // B tile, K 32..47 (in the dead q half 1)
constexpr int P3_OFF_G = 65536;      // per head: graw, gc, beta, e^gc (64 floats each)
constexpr int P3_OFF_D0 = 67584;     // per head: D^-1 of the first diagonal block [16][16]
constexpr int P3_SMEM = P3_OFF_D0 + 2048 + 1024;
constexpr uint32_t P3_TM_COLS = 128;

__device__ __forceinline__ float4 tf32x4(const float* v) {
  return make_float4(tc::to_tf32(v[0]), tc::to_tf32(v[1]), tc::to_tf32(v[2]), tc::to_tf32(v[3]));
}
// byte offset of the 16-byte chunk holding contraction indices 4 k4 .. 4 k4 + 3
// of operand row r (k4 < 12), from the tile's SW128 part (main) or SW64 part (tail)
__device__ __forceinline__ uint32_t op_chunk(uint32_t main, uint32_t tail, int r, int k4) {
  return k4 < 8 ? main + (uint32_t)(r * 128 + ((k4 ^ (r & 7)) << 4))
                : tail + (uint32_t)(r * 64 + (((k4 - 8) ^ ((r >> 1) & 3)) << 4));
}
__device__ __forceinline__ void st_shared_v4(uint32_t addr, float4 v) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};\n" ::"r"(addr), "f"(v.x), "f"(v.y),
               "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ float4 ld_shared_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];\n"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
// Column-wise stores into a B tile: element (row nbase + c, K = k), c < 32,
// nbase a multiple of 32, k < 48.  Rows 8 apart repeat the swizzle, so the
// address is base[c & 7] + c * stride (stride = the part's row bytes).
struct BColumn {
  uint32_t base[8];
  uint32_t stride;
  __device__ __forceinline__ BColumn(uint32_t main, uint32_t tail, int nbase, int k) {
    if (k < 32) {
      stride = 128;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        base[u] = main + (uint32_t)(nbase * 128 + ((((k >> 2) & 7) ^ u) << 4) + (k & 3) * 4);
    } else {
      stride = 64;
#pragma unroll
      for (int u = 0; u < 8; ++u)
        base[u] = tail + (uint32_t)(nbase * 64 + (((((k - 32) >> 2) & 3) ^ ((u >> 1) & 3)) << 4) +
                                    (k & 3) * 4);
    }
  }
  __device__ __forceinline__ void st(int c, float v) const {
    asm volatile("st.shared.f32 [%0], %1;\n" ::"r"(base[c & 7] + stride * (uint32_t)c), "f"(v)
                 : "memory");
  }
  // the same when the caller knows the part (S = 128: K < 32, S = 64: K >= 32)
  template <int S>
  __device__ __forceinline__ void st_s(int c, float v) const {
    asm volatile("st.shared.f32 [%0], %1;\n" ::"r"(base[c & 7] + (uint32_t)(S * c)), "f"(v)
                 : "memory");
  }
};
__device__ __forceinline__ uint64_t op_desc(uint32_t main, uint32_t tail, int kstep) {
  return kstep < 4 ? tc::smem_desc(main + (uint32_t)(kstep * 32), 16, 1024)
                   : tc::smem_desc_sw64(tail + (uint32_t)((kstep - 4) * 32));
}

__global__ void __launch_bounds__(P_NT, 3) chunk_prep_pair_tc_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const GateSrc gs, unsigned char* __restrict__ ws,
    const int32_t* __restrict__ cu, int64_t N, int64_t T, int64_t Hg, int64_t H) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ uint64_t bar, ldbar;
  __shared__ uint32_t tmem_sh;
  __shared__ int64_t pos[4];
  __shared__ int ok_sh;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int quarter = warp & 3, colhalf = warp >> 2;
  const int c0 = colhalf * 32;  // this thread's 32 columns of a head's 64
  const int hk = blockIdx.y;
  if (tid == 0) {
    int64_t seq = 0, t0 = 0, eos = 0, cis = 0;
    const bool ok = locate_chunk(cu, N, T, blockIdx.x, seq, t0, eos, cis);
    pos[0] = ok ? chunk_offset(cu, seq, T) + cis : -1;
    pos[1] = t0;
    pos[2] = eos;
    ok_sh = ok ? 1 : 0;
  }
  __syncthreads();
  if (!ok_sh) return;
  const int64_t gci = pos[0], t0 = pos[1];
  const int L = (int)((pos[2] - t0) < BT ? (pos[2] - t0) : BT);
  const int hv0 = 2 * hk;
  float* gsm = reinterpret_cast<float*>(sm + P3_OFF_G);
  auto graw = [&](int h) { return gsm + h * 256; };
  auto gcs = [&](int h) { return gsm + h * 256 + 64; };
  auto bet = [&](int h) { return gsm + h * 256 + 128; };
  auto egc = [&](int h) { return gsm + h * 256 + 192; };
  auto wsb = [&](int h) { return ws + (gci * H + hv0 + h) * (int64_t)WS_CHUNK; };
  const uint32_t sb = tc::smem_addr(sm);
  const uint32_t am = sb + P3_OFF_AM, at = sb + P3_OFF_AT, bm = sb + P3_OFF_BM, bt = sb + P3_OFF_BT;
  float* d0s = reinterpret_cast<float*>(sm + P3_OFF_D0);

  if (tid == 0) {
    tc::mbar_init(&bar, 1);
    tc::mbar_init(&ldbar, 1);
    tc::mbar_fence_init();
    // k and q of the chunk as four 64 x 64 boxes: [K0 | Q0 | K1 | Q1]
    tc::mbar_arrive_expect_tx(&ldbar, 32768);
    for (int hf = 0; hf < 2; ++hf) {
      tc::tma_load_2d(sm + P_OFF_KQ + hf * P_KQ_HALF, &tm_k, hk * 128 + hf * 64, (int)t0, &ldbar);
      tc::tma_load_2d(sm + P_OFF_Q + hf * P_KQ_HALF, &tm_q, hk * 128 + hf * 64, (int)t0, &ldbar);
    }
  }
  if (warp == 0) {  // after the loads are on their way
    tc::tmem_alloc(&tmem_sh, P3_TM_COLS);
    tc::tmem_relinquish();
  }
  if (tid < 128) {  // both heads' gates
    const int h = tid >> 6, t = tid & 63;
    float gv = 0.f, bv = 0.f;
    if (t < L) gate_load(gs, t0 + t, H, hv0 + h, gv, bv);
    graw(h)[t] = gv;
    bet(h)[t] = bv;
    reinterpret_cast<float*>(wsb(h) + WS_GB)[t] = gv;
    reinterpret_cast<float*>(wsb(h) + WS_GB)[64 + t] = bv;
  }
  __syncthreads();  // barrier inits visible before anyone waits
  if (tid == 0 && !tc::mbar_wait(&ldbar, 0, WAIT_LIMIT)) {
    record_error();
    ok_sh = 0;
  }
  __syncthreads();
  bool alive = ok_sh != 0;
  if (alive && L < BT) {
    // rows past the sequence end came from the next sequence (or the
    // tensor's zero fill): clear them so the Gram product sees only the chunk
    for (int e = tid; e < (BT - L) * 32; e += P_NT) {
      const int r = L + (e >> 5), part = e & 31;  // part: K0, Q0, K1, Q1 x 8 chunks
      *reinterpret_cast<uint4*>(sm + (part >> 3) * 8192 + r * 128 + (part & 7) * 16) =
          make_uint4(0, 0, 0, 0);
    }
  }
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = tmem_sh;
  uint32_t phase = 0;
  if (tid == 0 && alive) {
    const uint32_t id = tc::idesc_bf16(128, 64, false, false);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      tc::mma_bf16(tm, kdesc(sb + P_OFF_KQ, P_KQ_HALF, j), kdesc(sb + P_OFF_KQ, P_KQ_HALF, j), id,
                   j > 0);
    tc::commit(&bar);
  }
  if (warp == 0 || warp == 4) {  // cumsum of each head while the Gram product runs
    const int h = warp >> 2;
    chunk_cumsum_warp(graw(h), gcs(h), lane);
    __syncwarp();
    egc(h)[lane] = __expf(gcs(h)[lane]);
    egc(h)[lane + 32] = __expf(gcs(h)[lane + 32]);
  }
  // One thread polls the MMA barrier; the others wait at the block barrier,
  // which takes no issue slots.
  auto wait_mma = [&]() {
    if (tid == 0 && !tc::mbar_wait(&bar, phase, WAIT_LIMIT)) {
      record_error();
      ok_sh = 0;
    }
    phase ^= 1u;
    __syncthreads();
    tc::fence_after();
    alive = ok_sh != 0;
  };
  // The 32 x 32 block of (rows of this quarter, columns 32 half ..): entirely
  // above the diagonal (zero everywhere), straddling it, or entirely below.
  const bool blk_zero = colhalf > (quarter & 1), blk_diag = colhalf == (quarter & 1);
  if (alive) wait_mma();
  if (alive) {  // Gram epilogue: k rows give L and D^-1, q rows give Aqk; warp (quarter,
                // colhalf) takes head colhalf's 64 columns of its 32 rows
    const int row = quarter * 32 + lane;
    // v[c] * s * e^{min(gi - gc_j, 0)}, j = cb + c, c < 16 (TMEM columns cb ..)
    auto decayed16 = [&](int h, int cb, float gi, float s, float (&a)[16]) {
      float v[16];
      tc::tmem_ld16(tm_addr(tm, quarter, cb), v);
      tc::tmem_wait_ld();
      const float2 s2 = make_float2(s, s), gi2 = make_float2(gi, gi);
#pragma unroll
      for (int c = 0; c < 16; c += 4) {
        const float4 g4 = *reinterpret_cast<const float4*>(gcs(h) + cb + c);
        const float2 d0 = fsub2(gi2, make_float2(g4.x, g4.y)), d1 = fsub2(gi2, make_float2(g4.z, g4.w));
        const float2 e0 = make_float2(__expf(fminf(d0.x, 0.f)), __expf(fminf(d0.y, 0.f)));
        const float2 e1 = make_float2(__expf(fminf(d1.x, 0.f)), __expf(fminf(d1.y, 0.f)));
        const float2 p0 = fmul2(fmul2(make_float2(v[c], v[c + 1]), s2), e0);
        const float2 p1 = fmul2(fmul2(make_float2(v[c + 2], v[c + 3]), s2), e1);
        a[c] = p0.x; a[c + 1] = p0.y; a[c + 2] = p1.x; a[c + 3] = p1.y;
      }
    };
    if (row < 64) {
      // k row i; in a diagonal block i = c0 + lane, so column c is strictly
      // below the diagonal when c < lane.  L enters N = D^-1 L through its
      // rows 16..63: row i is contraction index i - 16 of both tiles.
      const int i = row, sub = lane >> 4, li = lane & 15;
      const bool has_k = i >= 16;
      const int h = colhalf;  // this warp's head; it covers all 64 columns
      const int r = 64 * h + i;
      const float bi = bet(h)[i], gi = gcs(h)[i];
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        const int c0 = 32 * half;
        const bool blk_zero = half > (quarter & 1), blk_diag = half == (quarter & 1);
        const BColumn lcol(bm, bt, 64 * h + c0, has_k ? i - 16 : 0);  // L[i][c0 + c]
        if (blk_zero) {  // L and D^-1 are zero here
          if (has_k) {
#pragma unroll
            for (int c = 0; c < 32; ++c) lcol.st(c, 0.f);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) st_shared_v4(op_chunk(am, at, r, 4 + u), make_float4(0.f, 0.f, 0.f, 0.f));
          continue;
        }
        if (!blk_diag) {  // rows 32-63 x columns 0-31: all of it is L, D^-1 is zero
#pragma unroll
          for (int cb = 0; cb < 32; cb += 16) {
            float a[16];
            decayed16(h, c0 + cb, gi, bi, a);
#pragma unroll
            for (int c = 0; c < 16; ++c) lcol.st(cb + c, tc::to_tf32(a[c]));
          }
#pragma unroll
          for (int u = 0; u < 4; ++u) st_shared_v4(op_chunk(am, at, r, u), make_float4(0.f, 0.f, 0.f, 0.f));
          continue;
        }
        // Diagonal block pair: columns 0-15 are lanes 0-15's diagonal block
        // and lanes 16-31's L; columns 16-31 are lanes 16-31's diagonal block.
        float dr[16];
        {
          float a[16];
          decayed16(h, c0, gi, bi, a);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            if (c >= lane) a[c] = 0.f;
            dr[c] = a[c];
            if (has_k) lcol.st(c, sub ? tc::to_tf32(a[c]) : 0.f);
          }
        }
        {
          float a[16];
          decayed16(h, c0 + 16, gi, bi, a);
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            if (16 + c >= lane) a[c] = 0.f;
            if (sub) dr[c] = a[c];
            if (has_k) lcol.st(16 + c, 0.f);
          }
        }
        // row li of (I + A_blk)^-1 of the row's 16 x 16 diagonal block
        float y[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) y[m] = (m == li) ? 1.f : 0.f;
        const int src0 = lane & 16;
#pragma unroll
        for (int m = 0; m < 15; ++m) {
#pragma unroll
          for (int c = 0; c <= m; ++c) {
            const float ym = __shfl_sync(0xffffffffu, y[c], src0 + m);
            y[c] = fmaf(-dr[m], ym, y[c]);
          }
        }
        // D^-1 row i, columns c0..c0+31, as contraction indices (column - 16)
        // of the A tile; the first block (columns 0-15) goes to its own scratch
        if (half == 0 && sub == 0) {
#pragma unroll
          for (int u = 0; u < 4; ++u)
            *reinterpret_cast<float4*>(d0s + (h * 16 + li) * 16 + 4 * u) = make_float4(y[4 * u], y[4 * u + 1], y[4 * u + 2], y[4 * u + 3]);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (half == 0 && u < 4) continue;  // columns 0-15: the first block, stored above
          float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
          if ((u >> 2) == sub) v = tf32x4(y + (u & 3) * 4);
          st_shared_v4(op_chunk(am, at, r, (c0 >> 2) - 4 + u), v);
        }
      }
    } else {  // Aqk rows, straight to the workspace image
      const int i = row - 64;
      const int h = colhalf;
      unsigned char* img = wsb(h) + WS_AQK;
      const float gi = gcs(h)[i];
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        const int c0 = 32 * half;
        const bool blk_zero = half > (quarter & 1), blk_diag = half == (quarter & 1);
        if (blk_zero) {
#pragma unroll
          for (int c = 0; c < 32; c += 8)
            *reinterpret_cast<uint4*>(img + chunk_off(i, (c0 + c) >> 3, 0)) = make_uint4(0, 0, 0, 0);
          continue;
        }
#pragma unroll
        for (int cb = 0; cb < 32; cb += 16) {
          float e[16];
          decayed16(h, c0 + cb, gi, 1.f, e);
          if (blk_diag) {
#pragma unroll
            for (int c = 0; c < 16; ++c)
              if (cb + c > lane) e[c] = 0.f;
          }
#pragma unroll
          for (int c = 0; c < 16; c += 8) {
            uint4 pk;
            pk.x = pack_bf16(e[c], e[c + 1]); pk.y = pack_bf16(e[c + 2], e[c + 3]);
            pk.z = pack_bf16(e[c + 4], e[c + 5]); pk.w = pack_bf16(e[c + 6], e[c + 7]);
            *reinterpret_cast<uint4*>(img + chunk_off(i, (c0 + cb + c) >> 3, 0)) = pk;
          }
        }
      }
    }
  }
  tc::fence_proxy_async();
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  // N = D^-1 L (A = D^-1, B = L, over L's rows 16..63), stored negated; then
  // X_{r+1} = D^-1 + (-N) X_r (A = -N, B = X_r, over N's columns 0..47)
  const uint32_t id_inv = tc::idesc_tf32(128, 128);
  auto issue_inv = [&]() {
#pragma unroll
    for (int j = 0; j < 6; ++j)
      tc::mma_tf32(tm, op_desc(am, at, j), op_desc(bm, bt, j), id_inv, j > 0);
    tc::commit(&bar);
  };
  if (tid == 0 && alive) issue_inv();
  // Round epilogues: TMEM lane 64 h + m holds row (h, m); this thread's
  // columns c0..c0+31 of its head are at TMEM column 64 h + c0.
  const int eh = quarter >> 1, em = (quarter & 1) * 32 + lane, er = 64 * eh + em;
  const int esub = (em >> 4) & 1;  // in a diagonal block: which 16 of the 32 columns are D^-1's
  const uint32_t tcol = 64u * eh + c0;
  const bool has_x = em < 48;      // X row em is contraction index em of the B tile
  float dinv[16];
#pragma unroll
  for (int m = 0; m < 16; ++m) dinv[m] = 0.f;
#pragma unroll 1
  for (int rd = 0; rd < 4; ++rd) {
    if (alive) wait_mma();
    if (rd == 0) {
      // this row's D^-1 block, read before -N overwrites the A tile
      if (alive && blk_diag) {
        const int blk = em >> 4;
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float4 t = blk == 0 ? *reinterpret_cast<const float4*>(d0s + (eh * 16 + em) * 16 + 4 * u)
                                    : ld_shared_v4(op_chunk(am, at, er, 4 * (blk - 1) + u));
          dinv[4 * u] = t.x; dinv[4 * u + 1] = t.y; dinv[4 * u + 2] = t.z; dinv[4 * u + 3] = t.w;
        }
      }
      __syncthreads();
    }
    if (alive && !blk_zero) {
      // 16 columns at a time: cb = 0 holds the diagonal block when esub == 0
#pragma unroll
      for (int cb = 0; cb < 32; cb += 16) {
        float acc[16];
        tc::tmem_ld16(tm_addr(tm, quarter, tcol + cb), acc);
        tc::tmem_wait_ld();
        const bool dblk = blk_diag && (cb >> 4) == esub;
        if (rd == 0) {  // acc = N: -N -> A tile (columns 0..47), X_0 = D^-1 -> B tile
#pragma unroll
          for (int c = 0; c < 16; ++c) acc[c] = -acc[c];
          if (c0 + cb < 48) {
#pragma unroll
            for (int u = 0; u < 4; ++u)
              st_shared_v4(op_chunk(am, at, er, ((c0 + cb) >> 2) + u), tf32x4(acc + 4 * u));
          }
          if (has_x) {
            const BColumn xcol(bm, bt, 64 * eh + c0, em);  // X[em][c0 + c]
            if (em < 32) {
#pragma unroll
              for (int c = 0; c < 16; ++c) xcol.st_s<128>(cb + c, dblk ? dinv[c] : 0.f);
            } else {
#pragma unroll
              for (int c = 0; c < 16; ++c) xcol.st_s<64>(cb + c, dblk ? dinv[c] : 0.f);
            }
          }
        } else {  // acc = -N X_{rd-1}: X_rd = D^-1 + acc
          if (dblk) {
#pragma unroll
            for (int c = 0; c < 16; ++c) acc[c] += dinv[c];
          }
          if (rd < 3) {
            if (has_x) {
              const BColumn xcol(bm, bt, 64 * eh + c0, em);
              if (em < 32) {
#pragma unroll
                for (int c = 0; c < 16; ++c) xcol.st_s<128>(cb + c, tc::to_tf32(acc[c]));
              } else {
#pragma unroll
                for (int c = 0; c < 16; ++c) xcol.st_s<64>(cb + c, tc::to_tf32(acc[c]));
              }
            }
          } else {  // acc = T: T' image (staged in the B tile) and T'' (in the A tile)
            unsigned char* tpi = sm + P3_OFF_BM + eh * 8192;
            unsigned char* tppi = sm + P3_OFF_AM + eh * 8192;
#pragma unroll
            for (int c = 0; c < 16; c += 8) {
              const int col = c0 + cb + c;
              uint32_t pa[4], pb[4];
#pragma unroll
              for (int u = 0; u < 8; u += 2) {
                // diagonal = bf16(beta); the chain adds beta - bf16(beta)
                const float2 bv = *reinterpret_cast<const float2*>(bet(eh) + col + u);
                const float2 ev = *reinterpret_cast<const float2*>(egc(eh) + col + u);
                const float2 p = fmul2(make_float2(acc[c + u], acc[c + u + 1]), bv);
                pa[u >> 1] = pack_bf16(p.x, p.y);
                const float2 qv = fmul2(p, ev);
                pb[u >> 1] = pack_bf16(qv.x, qv.y);
              }
              const uint4 a = make_uint4(pa[0], pa[1], pa[2], pa[3]);
              const uint4 b = make_uint4(pb[0], pb[1], pb[2], pb[3]);
              *reinterpret_cast<uint4*>(tpi + chunk_off(em, col >> 3, 0)) = a;
              *reinterpret_cast<uint4*>(tppi + chunk_off(em, col >> 3, 0)) = b;
            }
          }
        }
      }
    } else if (alive && rd == 3) {  // T is zero above the diagonal blocks
      unsigned char* tpi = sm + P3_OFF_BM + eh * 8192;
      unsigned char* tppi = sm + P3_OFF_AM + eh * 8192;
#pragma unroll
      for (int c = 0; c < 32; c += 8) {
        *reinterpret_cast<uint4*>(tpi + chunk_off(em, (c0 + c) >> 3, 0)) = make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(tppi + chunk_off(em, (c0 + c) >> 3, 0)) = make_uint4(0, 0, 0, 0);
      }
    }
    tc::fence_proxy_async();
    tc::fence_before();
    __syncthreads();
    tc::fence_after();
    if (tid == 0 && alive) {
      if (rd < 3) {
        issue_inv();
      } else {
        for (int h = 0; h < 2; ++h)
          tc::bulk_store(wsb(h) + WS_TP, sm + P3_OFF_BM + h * 8192, 8192);
        tc::bulk_commit_group();
        const uint32_t id = tc::idesc_bf16(128, 64, true, false);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            tc::mma_bf16(tm + (h ? P2_TM_W1 : P2_TM_W0), mndesc(sb + P_OFF_KQ, P_KQ_HALF, j),
                         kdesc64(am + h * 8192, j), id, j > 0);
        }
        tc::commit(&bar);
      }
    }
  }
  if (alive) wait_mma();
  if (alive) {
    // -w [t][kk] (bf16, SW128 image) from w^T in TMEM (lane = kk), staged in
    // the dead k / q tiles (head h at 16 KB x h): 16-lane TMEM loads give
    // 8 x 8 blocks in the mma fragment layout, transposing stmatrix stores put
    // each block's token rows at their swizzled places
    const int h = colhalf;
    unsigned char* stage = sm + h * 16384;
    const uint32_t wcol = h ? P2_TM_W1 : P2_TM_W0;
    const int mi = lane >> 3;
#pragma unroll 1
    for (int tb = 0; tb < 64; tb += 16) {
      uint32_t ra[8], rb[8];
      tc::tmem_ld16x256b_x2(tm_addr(tm, quarter, wcol + tb), ra);
      tc::tmem_ld16x256b_x2(tm_addr(tm, quarter, wcol + tb) + (16u << 16), rb);
      tc::tmem_wait_ld();
      auto pk = [](uint32_t x, uint32_t y) {
        return pack2<bf16>(make_float2(-__uint_as_float(x), -__uint_as_float(y)));
      };
      const int t = tb + ((mi >> 1) << 3) + (lane & 7);
#pragma unroll
      for (int lb = 0; lb < 32; lb += 16) {
        const int kk8 = quarter * 32 + lb + ((mi & 1) << 3);
        unsigned char* rowp =
            stage + (kk8 >> 6) * 8192 + t * 128 + ((((kk8 & 63) >> 3) ^ (t & 7)) << 4);
        const uint32_t(&r)[8] = lb ? rb : ra;
        stmatrix_x4_trans(rowp, pk(r[0], r[1]), pk(r[2], r[3]), pk(r[4], r[5]), pk(r[6], r[7]));
      }
    }
    tc::fence_proxy_async();
  }
  __syncthreads();
  if (tid == 0) {
    if (alive) {
      for (int h = 0; h < 2; ++h) tc::bulk_store(wsb(h) + WS_W, sm + h * 16384, 16384);
      tc::bulk_commit_group();
    }
    // shared memory may be released once the copies have read it; their
    // writes complete before the kernel does
    tc::bulk_wait_read<0>();
  }
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, P3_TM_COLS);
}

// ============================================================================
// Kernel 2: the chunk chain
// ============================================================================
constexpr int C_EPI_WARPS = 16;           // epilogue warps: 4 per TMEM lane quarter
constexpr int C_NT = 32 * (2 + C_EPI_WARPS);  // producer, MMA, epilogue
constexpr int C_SCOLS = 128 / (C_EPI_WARPS / 4);  // state columns per epilogue thread
constexpr int C_TCOLS = 64 / (C_EPI_WARPS / 4);   // token columns per epilogue thread
constexpr int STAGE = 81920;              // bytes per pipeline stage
// WQ: one [128 x 128] SW128 tile, halves 16 KB apart: rows 0-63 = -w, 64-127 = q.
constexpr int S_K = 0, S_WQ = 16384, S_V = 49152, S_TP = 65536, S_AQK = 73728;
constexpr int C_OFF_TPL = 2 * STAGE;          // diag(beta - bf16(beta)) [64 x 64]
constexpr int C_OFF_TAB = C_OFF_TPL + 8192;   // 4 slots (chunk & 3): e^{gl-gc}[64], e^{gc}[64], gl
constexpr int C_TAB = 1024;
// per epilogue warp: the output transpose [16 x 32] bf16, then the norm's
// gate rows z (and the normalised rows, in place) [16 x 32] bf16
constexpr int C_OFF_OST = C_OFF_TAB + 4 * C_TAB;
// fused output norm: weight [128] fp32, then the partial sums of squares of
// 8 values each [column quarter][2 alternating sets][token half][TMEM lane
// quarter][piece within the quarter][token % 8] fp32 (a lane's reads and
// writes fall in 32 distinct banks)
constexpr int C_OFF_NRM = C_OFF_OST + C_EPI_WARPS * 2048;
constexpr int C_SMEM = C_OFF_NRM + 512 + 8192 + 1024;
// TMEM columns.  fp32 accumulators: D_u, D_qh (adjacent: one N = 128 product
// fills both), D_o, dS.  bf16 A operands written by the epilogue (packed in
// pairs, so a [128 x K] operand takes K/2 columns): S^T, vt hi, vt lo, v_new.
constexpr uint32_t C_TM_U = 0, C_TM_QH = 64, C_TM_O = 128, C_TM_HT = 192, C_TM_DS = 256,
                   C_TM_VTH = 384, C_TM_VTL = 416, C_TM_VN = 448, C_TM_COLS = 512;
constexpr int KV = 128 * 128;

// Work of one chain CTA.  A CTA walks chunks [c0, c1) of one (sequence,
// value head) starting from a given state:
//   ITEM_OUT    the real recurrence, writing o (and the end state if asked)
//   ITEM_LOCAL  the recurrence from a zero state, no output: the segment's
//               additive part B
//   ITEM_TRANS  the recurrence from the identity with v = 0, no output: the
//               segment's transition X, so that S_end^T = S_start^T X + B^T
enum : int { ITEM_OUT = 0, ITEM_LOCAL = 1, ITEM_TRANS = 2 };

// Segment-parallel schedule for long sequences.  seg = 0: one ITEM_OUT per
// (sequence, head), longest sequences first.  seg > 0: every sequence is cut
// into segments of `seg` chunks; phase 1 runs segment 0 (ITEM_OUT) and the
// LOCAL / TRANS items of the middle segments; chunk_combine_kernel chains the
// segment start states; phase 3 runs segments 1.. with outputs.
struct ChainPlan {
  int seg;
  int phase;
  float* scratch;  // [slot][H][3][K*V]: start state, B, X (slot = segment index over all sequences)
};

// Gated RMSNorm of the output, fused into the chain's output epilogue: each
// (token, value head) row of V values becomes
//   y = ((o * rstd) * w) * silu(z),  rstd = 1 / sqrt(mean(o^2) + eps),
// o taken as the bf16 value the unfused operator would store.  This is the
// layer_norm_fwd (is_rms_norm, norm_before_gate, no bias, group = V) that
// the GDN layer applies to the rule's output next.  z == nullptr: no norm.
struct OutNorm {
  // gate rows: head h of token t at z + t * ldz + (h / zr) * zgs + (h % zr) * V
  // (zr = 1, zgs = V: [tokens, H * V] rows; a layer's projection interleaves
  // the z heads of each key head with its other blocks: zr = H / Hg)
  const bf16* z;
  const void* w;   // [V] weight, fp32 (w_f32) or bf16
  bf16* y;         // [tokens, H * V] normalised output
  int64_t ldz;
  int64_t zgs;
  int zr;
  float eps;
  int w_f32;
  int keep_o;      // also store o itself
};

__device__ __forceinline__ float* seg_state(const ChainPlan& p, int64_t slot, int64_t H, int h,
                                            int which) {
  return p.scratch + ((slot * H + h) * 3 + which) * (int64_t)KV;
}
__device__ __forceinline__ int seq_chunks(const int32_t* cu, int64_t n, int64_t T) {
  int64_t bos, eos;
  seq_span(cu, n, T, bos, eos);
  return (int)((eos - bos + BT - 1) / BT);
}

// q, k, v are read through 2-D tensor maps (rows = tokens, 64 x 64 boxes,
// 128-byte swizzle): the box lands exactly as one half of an SW128 tile.
// NORM: the fused output norm (a separate instantiation, so the plain rule
// keeps its own register allocation).
template <bool NORM>
__global__ void __launch_bounds__(C_NT, 1) chunk_chain_kernel(
    const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
    const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
    const __grid_constant__ CUtensorMap tm_y, const float* __restrict__ h0,
    const unsigned char* __restrict__ ws, bf16* __restrict__ o, float* __restrict__ ht,
    const int32_t* __restrict__ cu, int64_t N, int64_t T, int64_t Hg, int64_t H, float scale,
    ChainPlan plan, OutNorm nrm) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ uint64_t full[2], empty[2], early_free[2], tma[2], tma_a[2], aqk_free[2], bar_ht,
      bar_v, bar_q, bar_vt, bar_s, bar_o, bar_od, bar_fin;
  __shared__ uint64_t nbar[8];  // fused norm: [column quarter][set], the four lane-quarter warps
  __shared__ uint32_t tmem_sh;
  __shared__ int abort_sh;
  __shared__ int64_t it_n;
  __shared__ int it_valid, it_kind, it_c0, it_c1;
  __shared__ const float* it_init;
  __shared__ float* it_out;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t idx = blockIdx.x / H;
  const int h = (int)(blockIdx.x - idx * H);
  if (tid == 0) it_valid = 0;
  __syncthreads();
  if (plan.seg == 0) {
    // Longest sequences first: CTA rank r serves the r-th longest sequence
    // (ties by index), so the longest chains start in the first wave.
    if (!cu || N > 4096) {
      if (tid == 0 && idx < N) { it_n = idx; it_valid = 1; }
    } else {
      for (int64_t j = tid; j < N; j += blockDim.x) {
        const int64_t lj = (int64_t)cu[j + 1] - cu[j];
        int64_t r = 0;
        for (int64_t m = 0; m < N; ++m) {
          const int64_t lm = (int64_t)cu[m + 1] - cu[m];
          r += (lm > lj) || (lm == lj && m < j);
        }
        if (r == idx) { it_n = j; it_valid = 1; }
      }
    }
    __syncthreads();
    if (tid == 0 && it_valid) {
      const int64_t n = it_n;
      it_kind = ITEM_OUT;
      it_c0 = 0;
      it_c1 = seq_chunks(cu, n, T);
      it_init = h0 ? h0 + (n * H + h) * KV : nullptr;
      it_out = ht ? ht + (n * H + h) * KV : nullptr;
    }
  } else if (tid == 0) {
    int64_t acc = 0, slot = 0;
    for (int64_t n = 0; n < N; ++n) {
      const int nc = seq_chunks(cu, n, T);
      const int nseg = nc > plan.seg ? (nc + plan.seg - 1) / plan.seg : 1;
      const int64_t cnt = plan.phase == 1 ? 1 + 2 * (nseg > 2 ? nseg - 2 : 0) : nseg - 1;
      if (idx < acc + cnt) {
        const int j = (int)(idx - acc);
        int s;
        it_n = n;
        it_valid = 1;
        if (plan.phase == 1 && j == 0) {
          s = 0;
          it_kind = ITEM_OUT;
          it_init = h0 ? h0 + (n * H + h) * KV : nullptr;
          it_out = nseg == 1 ? (ht ? ht + (n * H + h) * KV : nullptr)
                             : seg_state(plan, slot + 1, H, h, 0);
        } else if (plan.phase == 1) {
          s = 1 + (j - 1) / 2;
          it_kind = ((j - 1) & 1) ? ITEM_TRANS : ITEM_LOCAL;
          it_init = nullptr;
          it_out = seg_state(plan, slot + s, H, h, it_kind == ITEM_LOCAL ? 1 : 2);
        } else {
          s = 1 + j;
          it_kind = ITEM_OUT;
          it_init = seg_state(plan, slot + s, H, h, 0);
          it_out = s == nseg - 1 ? (ht ? ht + (n * H + h) * KV : nullptr) : nullptr;
        }
        it_c0 = s * plan.seg;
        it_c1 = (s + 1) * plan.seg < nc ? (s + 1) * plan.seg : nc;
        break;
      }
      acc += cnt;
      slot += nseg;
    }
  }
  __syncthreads();
  if (!it_valid) return;  // uniform: spare CTAs of an upper-bound grid
  const int64_t n = it_n;
  const int kind = it_kind, c0 = it_c0, NI = it_c1 - it_c0;
  const bool has_v = kind != ITEM_TRANS, write_o = kind == ITEM_OUT;
  const int hk = (int)(h / (H / Hg));
  int64_t bos, eos;
  seq_span(cu, n, T, bos, eos);
  const int64_t boh = chunk_offset(cu, n, T);
  const uint32_t sb = tc::smem_addr(sm);
  constexpr int K = 128, V = 128;

  if (warp == 0) {
    tc::tmem_alloc(&tmem_sh, C_TM_COLS);
    tc::tmem_relinquish();
  }
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
      tc::mbar_init(&early_free[s], 1);
      tc::mbar_init(&tma[s], 1);
      tc::mbar_init(&tma_a[s], 1);
      tc::mbar_init(&aqk_free[s], 1);
    }
    tc::mbar_init(&bar_ht, C_EPI_WARPS);
    tc::mbar_init(&bar_v, 1);
    tc::mbar_init(&bar_vt, C_EPI_WARPS);
    tc::mbar_init(&bar_s, 1);
    tc::mbar_init(&bar_o, C_EPI_WARPS);
    tc::mbar_init(&bar_od, 1);
    tc::mbar_init(&bar_q, 1);
    tc::mbar_init(&bar_fin, 1);
    for (int e = 0; e < 8; ++e) tc::mbar_init(&nbar[e], 4);
    tc::mbar_fence_init();
    abort_sh = 0;
  }
  for (int e = tid; e < 8192 / 16; e += C_NT)  // diagonal-correction tile starts at zero
    reinterpret_cast<uint4*>(sm + C_OFF_TPL)[e] = make_uint4(0, 0, 0, 0);
  if (NORM && kind == ITEM_OUT && tid < 128)
    reinterpret_cast<float*>(sm + C_OFF_NRM)[tid] =
        nrm.w_f32 ? static_cast<const float*>(nrm.w)[tid]
                  : __bfloat162float(static_cast<const bf16*>(nrm.w)[tid]);
  tc::fence_before();
  __syncthreads();
  tc::fence_after();
  const uint32_t tm = tmem_sh;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Loads chunk i into stage i & 1, and computes its gate tables and the
    // diagonal correction tile, so the epilogue and MMA warps only consume.
    for (int i = 0; i < NI; ++i) {
      const int s = i & 1, c = c0 + i;
      // The stage is released in three parts: v, T', -w, q once chunk i-2's
      // [-w; q] product is done (early_free), k once its state product is
      // (empty), Aqk once its output product is (aqk_free).
      if (i >= 2 && !tc::mbar_wait(&early_free[s], ((i - 2) >> 1) & 1, WAIT_LIMIT)) {
        record_error();
        atomicExch(&abort_sh, 1);
      }
      if (*(volatile int*)&abort_sh) break;
      const int64_t t0 = bos + (int64_t)c * BT;
      const int L = (int)((eos - t0) < BT ? (eos - t0) : BT);
      unsigned char* st = sm + s * STAGE;
      const unsigned char* wsb = ws + ((boh + c) * H + h) * (int64_t)WS_CHUNK;
      const int y = (int)t0;
      if (lane == 0) {
        // the workspace pieces are stored as shared-memory images already
        const uint32_t bytes = 32768 + (write_o ? 16384 : 0) + (has_v ? 16384 + 8192 : 0);
        tc::mbar_arrive_expect_tx(&tma[s], bytes);
        for (int hf = 0; hf < 2; ++hf) {
          tc::bulk_load(st + S_WQ + hf * 16384, wsb + WS_W + hf * 8192, 8192, &tma[s]);
          if (write_o)
            tc::tma_load_2d(st + S_WQ + 8192 + hf * 16384, &tm_q, hk * K + hf * 64, y, &tma[s]);
          if (has_v) tc::tma_load_2d(st + S_V + hf * 8192, &tm_v, h * V + hf * 64, y, &tma[s]);
        }
        if (has_v) tc::bulk_load(st + S_TP, wsb + WS_TP, 8192, &tma[s]);
      }
      if (i >= 2 && !tc::mbar_wait(&empty[s], ((i - 2) >> 1) & 1, WAIT_LIMIT)) {
        record_error();
        atomicExch(&abort_sh, 1);
      }
      if (lane == 0 && !*(volatile int*)&abort_sh) {
        for (int hf = 0; hf < 2; ++hf)
          tc::tma_load_2d(st + S_K + hf * 8192, &tm_k, hk * K + hf * 64, y, &tma[s]);
      }
      // gates of tokens 2*lane, 2*lane+1: in-chunk cumsum (same association
      // as chunk_cumsum_warp, so it matches the preparation kernel bit for bit)
      float ga = 0.f, gb2 = 0.f, ba = 0.f, bb = 0.f;
      const int i0 = 2 * lane;
      {
        // the preparation kernel's copy of the chunk's gates (zero past L)
        const float2 gg = *reinterpret_cast<const float2*>(wsb + WS_GB + 8 * lane);
        const float2 bb2 = *reinterpret_cast<const float2*>(wsb + WS_GB + 256 + 8 * lane);
        ga = gg.x;
        gb2 = gg.y;
        ba = bb2.x;
        bb = bb2.y;
      }
      const float pair = ga + gb2;
      float incl = pair;
#pragma unroll
      for (int d = 1; d < 32; d <<= 1) {
        const float nb = __shfl_up_sync(0xffffffffu, incl, d);
        if (lane >= d) incl += nb;
      }
      const float excl = incl - pair;
      const float gc0 = excl + ga, gc1 = excl + ga + gb2;
      const float gl = __shfl_sync(0xffffffffu, gc1, 31);
      float* tab = reinterpret_cast<float*>(sm + C_OFF_TAB + (i & 3) * C_TAB);
      tab[i0] = __expf(fminf(gl - gc0, 0.f));
      tab[i0 + 1] = __expf(fminf(gl - gc1, 0.f));
      tab[64 + i0] = __expf(gc0);
      tab[64 + i0 + 1] = __expf(gc1);
      if (lane == 0) tab[128] = gl;
      if (has_v) {
        // the previous chunk's D_u product (the last reader of the tile) is
        // complete once bar_v of that chunk has fired
        if (i >= 1 && !tc::mbar_wait(&bar_v, (i - 1) & 1, WAIT_LIMIT)) {
          record_error();
          atomicExch(&abort_sh, 1);
        }
        *reinterpret_cast<bf16*>(sm + C_OFF_TPL + elem_off(i0, i0, 8192)) =
            __float2bfloat16_rn(ba - __bfloat162float(__float2bfloat16_rn(ba)));
        *reinterpret_cast<bf16*>(sm + C_OFF_TPL + elem_off(i0 + 1, i0 + 1, 8192)) =
            __float2bfloat16_rn(bb - __bfloat162float(__float2bfloat16_rn(bb)));
      }
      if (!tc::mbar_wait(&tma[s], (i >> 1) & 1, WAIT_LIMIT)) {
        record_error();
        atomicExch(&abort_sh, 1);
        break;
      }
      if (L < BT) {
        // rows past the sequence end came from the next sequence (or the
        // tensor's zero fill): clear them so the chunk sees only its tokens
        for (int e = lane; e < (BT - L) * 16; e += 32) {
          const int r = L + (e >> 4), part = e & 15, hf = part >> 3, c16 = part & 7;
          const uint32_t off = (uint32_t)(hf * 8192 + r * 128 + c16 * 16);
          *reinterpret_cast<uint4*>(st + S_K + off) = make_uint4(0, 0, 0, 0);
          if (has_v) *reinterpret_cast<uint4*>(st + S_V + off) = make_uint4(0, 0, 0, 0);
          if (write_o)
            *reinterpret_cast<uint4*>(st + S_WQ + 8192 + hf * 16384 + r * 128 + c16 * 16) =
                make_uint4(0, 0, 0, 0);
        }
      }
      tc::fence_proxy_async();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&full[s]);
      if (write_o) {
        // Aqk is read last (by the output product, a chunk later): it has its
        // own buffer release and transaction barrier
        if (i >= 2 && !tc::mbar_wait(&aqk_free[s], ((i - 2) >> 1) & 1, WAIT_LIMIT)) {
          record_error();
          atomicExch(&abort_sh, 1);
          break;
        }
        if (lane == 0) {
          tc::mbar_arrive_expect_tx(&tma_a[s], 8192);
          tc::bulk_load(st + S_AQK, wsb + WS_AQK, 8192, &tma_a[s]);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    // These products are short (N <= 128, K <= 128), so the issue rate of
    // tcgen05.mma bounds them, not the tensor pipe: every descriptor is a
    // per-stage base plus a compile-time offset (one 64-bit add per MMA).
    if (lane == 0 && NI > 0) {
      const uint32_t id_u = tc::idesc_bf16(128, 64, true, false);
      const uint32_t id_w = tc::idesc_bf16(128, 64, false, false);
      const uint32_t id_wq = tc::idesc_bf16(128, 128, false, false);
      const uint32_t id_s = tc::idesc_bf16(128, 128, false, true);
      const uint32_t id_o = tc::idesc_bf16(128, 64, false, false);
      const uint64_t d_tpl = kdesc64(sb + C_OFF_TPL, 0);
      // descriptor address steps (16-byte units): K-step j of a K-major
      // [rows x 64] tile is 32 bytes on; of the [128 x 128] [-w; q] tile,
      // (j / 4) halves of 16 KB plus (j % 4) * 32 bytes; of an MN-major tile,
      // 16 rows (2 KB) on
      constexpr uint64_t KSTEP64 = 32 >> 4, MNSTEP = 2048 >> 4;
      auto wq_step = [](int j) -> uint64_t { return (uint64_t)(((j >> 2) * 16384 + (j & 3) * 32) >> 4); };
      // D_u = v^T T'^T with T' = T diag(beta) in bf16, plus v^T diag(beta -
      // bf16(beta)): the unit diagonal's beta_i v_i term is exact to ~2^-17.
      auto issue_u = [&](int i) {
        const uint32_t st = sb + (i & 1) * STAGE;
        const uint64_t dv = mndesc(st + S_V, 8192, 0), dtp = kdesc64(st + S_TP, 0);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::mma_bf16(tm + C_TM_U, dv + j * MNSTEP, dtp + j * KSTEP64, id_u, j > 0);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::mma_bf16(tm + C_TM_U, dv + j * MNSTEP, d_tpl + j * KSTEP64, id_u, true);
      };
      // D_o(c) += v_new^T Aqk^T, once the epilogue has put e^{gc} D_qh there.
      // Issued behind the next chunk's [-w; q] product, off the state path.
      auto issue_o = [&](int c) -> bool {
        const int sc = c & 1;
        if (!tc::mbar_wait(&bar_o, c & 1, WAIT_LIMIT) ||
            !tc::mbar_wait(&tma_a[sc], (c >> 1) & 1, WAIT_LIMIT))
          return false;
        tc::fence_after();
        const uint64_t da = kdesc64(sb + sc * STAGE + S_AQK, 0);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::mma_bf16_ts(tm + C_TM_O, tm + C_TM_VN + 8 * j, da + j * KSTEP64, id_o, true);
        tc::commit(&bar_od);
        tc::commit(&aqk_free[sc]);
        return true;
      };
      bool live = true;
      if (has_v) {
        live = tc::mbar_wait(&full[0], 0, WAIT_LIMIT);
        tc::fence_after();
        if (live) issue_u(0);
      }
      for (int i = 0; i < NI && live; ++i) {
        const int s = i & 1;
        const uint32_t st = sb + s * STAGE;
        if (!has_v && !(live = tc::mbar_wait(&full[s], (i >> 1) & 1, WAIT_LIMIT))) break;
        const uint64_t dwq = kdesc(st + S_WQ, 16384, 0);
        if (!(live = tc::mbar_wait(&bar_ht, i & 1, WAIT_LIMIT))) break;
        tc::fence_after();
        if (write_o) {
          // one N = 128 product over the [-w; q] tile: D_u += S^T (-w)^T next
          // to D_qh = S^T q^T (the epilogue zeroed D_qh after reading it)
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::mma_bf16_ts(tm + C_TM_U, tm + C_TM_HT + 8 * j, dwq + wq_step(j), id_wq, true);
          tc::commit(&bar_v);
          tc::commit(&bar_q);
        } else {
          // D_u (+)= S^T (-w)^T
#pragma unroll
          for (int j = 0; j < 8; ++j)
            tc::mma_bf16_ts(tm + C_TM_U, tm + C_TM_HT + 8 * j, dwq + wq_step(j), id_w,
                            has_v || j > 0);
          tc::commit(&bar_v);
        }
        tc::commit(&early_free[s]);
        if (write_o && i > 0 && !(live = issue_o(i - 1))) break;
        // dS = vt_hi^T k + vt_lo^T k
        const uint64_t dk = mndesc(st + S_K, 8192, 0);
        if (!(live = tc::mbar_wait(&bar_vt, i & 1, WAIT_LIMIT))) break;
        tc::fence_after();
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::mma_bf16_ts(tm + C_TM_DS, tm + C_TM_VTH + 8 * j, dk + j * MNSTEP, id_s, j > 0);
#pragma unroll
        for (int j = 0; j < 4; ++j)
          tc::mma_bf16_ts(tm + C_TM_DS, tm + C_TM_VTL + 8 * j, dk + j * MNSTEP, id_s, true);
        tc::commit(&bar_s);
        tc::commit(&empty[s]);
        // the next chunk's D_u runs while the epilogue applies dS
        if (has_v && i + 1 < NI) {
          if (!(live = tc::mbar_wait(&full[s ^ 1], ((i + 1) >> 1) & 1, WAIT_LIMIT))) break;
          tc::fence_after();
          issue_u(i + 1);
        }
      }
      if (live && write_o) live = issue_o(NI - 1);
      if (!live) {
        record_error();
        atomicExch(&abort_sh, 1);
      }
      // every MMA has landed before TMEM is released
      tc::commit(&bar_fin);
      if (!tc::mbar_wait(&bar_fin, 0, WAIT_LIMIT)) record_error();
    }
  } else {
    // ------------------------------------------------------------ epilogue warps
    const int cw = warp - 2;             // 0..15: four warps per TMEM lane quarter
    const int quarter = warp & 3;        // TMEM lane quarter
    const int colq = cw >> 2;            // which quarter of the columns this warp owns
    const int vrow = quarter * 32 + lane;
    const int kc0 = colq * C_SCOLS;      // state columns owned
    const int tc0 = colq * C_TCOLS;      // token columns owned in 64-wide regions
    // the state as fp32 pairs (columns 2m, 2m+1), updated with packed f32x2
    // instructions: the epilogue is issue-bound, 16 warps on 4 schedulers
    float2 S[C_SCOLS / 2];
    {
      const float* src = it_init;
#pragma unroll
      for (int m = 0; m < C_SCOLS / 2; ++m) {
        const int c = kc0 + 2 * m;
        S[m] = kind == ITEM_TRANS
                   ? make_float2(c == vrow ? 1.f : 0.f, c + 1 == vrow ? 1.f : 0.f)
                   : (src ? make_float2(src[c * V + vrow], src[(c + 1) * V + vrow])
                          : make_float2(0.f, 0.f));
      }
    }
    float gl_prev = 0.f;
    int L_prev = 0;
    int64_t t0_prev = 0;
    bool live = true;
    // Each thread waits on its own; a timeout flags the CTA and every role
    // leaves its loop (no named barrier inside the loop can strand a warp).
    auto wait_ok = [&](uint64_t* b, uint32_t par) -> bool {
      if (!tc::mbar_wait(b, par, WAIT_LIMIT)) {
        record_error();
        atomicExch(&abort_sh, 1);
        return false;
      }
      tc::fence_after();
      return true;
    };
    // all 32 lanes' TMEM writes have landed: one arrive per warp (the epilogue
    // writes no shared memory, so no proxy fence is needed)
    auto warp_arrive = [&](uint64_t* b) {
      tc::tmem_wait_st();
      tc::fence_before();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(b);
    };
    static_assert(C_TCOLS == 16 && C_SCOLS == 32, "epilogue tiling assumes 16 warps");
    // o = scale * D_o of a finished chunk.  A warp owns 16 tokens x 32 values
    // (TMEM lane = value): two 16-lane TMEM loads deliver them in the mma
    // fragment layout, and two transposing stmatrix stores write them as bf16
    // rows [token][value] into the warp's own 1 KB shared buffer; lane 0 then
    // stores the box with one TMA store.  A warp whose rows cross the
    // sequence end (the rows after it belong to the next sequence) stores its
    // valid rows with plain 16-byte stores instead.
    unsigned char* ost = sm + C_OFF_OST + cw * 2048;
    // Fused output norm.  A row's 128 values are spread over the four warps
    // of one column quarter (one per TMEM lane quarter), 8 values per lane.
    // Each lane's sum of squares of its 8 values goes to shared memory; after
    // an mbarrier on which the four warps meet (bounded wait, two sets
    // alternating by call) every lane reads the row's 16 partial sums and
    // adds them in the butterfly order of the stand-alone gated-norm kernel
    // (pieces 8 apart, then 4, 2, 1), so y equals that kernel's result on
    // the stored o bit for bit.  Lane (r, m) loads, normalises and stores
    // back exactly the 16 bytes it reads (token rows r and r + 8, values
    // 8m .. 8m + 7 of the warp's 32), in place over o.
    // The norm of chunk c runs one chunk late, while the tensor core forms
    // chunk c + 2's [-w; q] product (the epilogue's idle wait), not in the
    // dS window that bounds the chain; chunk c's z rows arrive by cp.async
    // into the second half of the warp's buffer one chunk ahead of that.
    const bool norm = NORM && write_o;
    const bool store_o = !NORM || nrm.keep_o;
    unsigned char* zst = ost + 1024;
    const int64_t zh = NORM ? (int64_t)(h / nrm.zr) * nrm.zgs + (int64_t)(h % nrm.zr) * V : 0;
    uint32_t ncall = 0;
    auto load_z = [&](int64_t tb, int Lc) {
      __syncwarp();  // every lane has read the previous chunk's z
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int r = (lane >> 2) + 8 * j, m = lane & 3;
        const bool in = tc0 + r < Lc;
        cp_async16(zst + r * 64 + m * 16,
                   nrm.z + (in ? tb + tc0 + r : tb) * nrm.ldz + zh + quarter * 32 + m * 8,
                   in ? 16 : 0);
      }
      cp_async_commit();
    };
    // (the o pieces are read from shared memory twice, before and after the
    // exchange, rather than held in registers across it)
    auto norm_rows = [&]() -> bool {
      const int m = lane & 3;
      const int set = colq * 2 + (int)(ncall & 1);
      float* red = reinterpret_cast<float*>(sm + C_OFF_NRM + 512) + set * 256;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int r = (lane >> 2) + 8 * j;
        const uint4 p = *reinterpret_cast<const uint4*>(ost + r * 64 + m * 16);
        const uint32_t pw[4] = {p.x, p.y, p.z, p.w};
        float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 x = unpack2<bf16>(pw[u]);
          s2 = ffma2(x, x, s2);
        }
        red[j * 128 + quarter * 32 + m * 8 + (lane >> 2)] = s2.x + s2.y;
      }
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&nbar[set]);
      cp_async_wait_all();  // this lane's z pieces, while the other warps arrive
      if (!wait_ok(&nbar[set], (ncall >> 1) & 1)) return false;
      ++ncall;
      const float* wt = reinterpret_cast<const float*>(sm + C_OFF_NRM) + quarter * 32 + m * 8;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int r = (lane >> 2) + 8 * j;
        // the row's pieces P = 4 q + m: this lane reads the four with its m
        // and the butterfly's last two levels (m ^ 2, m ^ 1) are shuffles
        const float* rp = red + j * 128 + m * 8 + (lane >> 2);
        float b = (rp[0] + rp[64]) + (rp[32] + rp[96]);  // (P_m + P_m+8) + (P_m+4 + P_m+12)
        b += __shfl_xor_sync(0xffffffffu, b, 2);
        const float tot = b + __shfl_xor_sync(0xffffffffu, b, 1);
        const float rs = rsqrtf(tot * (1.0f / 128) + nrm.eps);
        const float2 r2 = make_float2(rs, rs);
        uint4* op = reinterpret_cast<uint4*>(ost + r * 64 + m * 16);
        const uint4 p = *op;
        const uint4 zr = *reinterpret_cast<const uint4*>(zst + r * 64 + m * 16);
        const uint32_t pw[4] = {p.x, p.y, p.z, p.w}, zw[4] = {zr.x, zr.y, zr.z, zr.w};
        uint32_t yw[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float2 w2 = *reinterpret_cast<const float2*>(wt + 2 * u);
          const float2 g = silu2_lowp(unpack2<bf16>(zw[u]));
          yw[u] = pack2<bf16>(fmul2(fmul2(fmul2(unpack2<bf16>(pw[u]), r2), w2), g));
        }
        if (j == 0 && nrm.keep_o) {  // o's own store has read the buffer
          if (lane == 0) tc::bulk_wait_read<0>();
          __syncwarp();
        }
        *op = make_uint4(yw[0], yw[1], yw[2], yw[3]);
      }
      return true;
    };
    // rows [tc0, tc0 + 16) of the staged buffer buf to dst: one TMA store
    // when all 16 are in the sequence, else the valid rows by 16-byte stores
    auto store_rows = [&](const CUtensorMap* map, bf16* dst, const unsigned char* buf,
                          int64_t tb, int Lc) {
      if (tc0 + C_TCOLS <= Lc) {
        tc::fence_proxy_async();
        __syncwarp();
        if (lane == 0) {
          tc::tma_store_2d(map, (int)(h * V + quarter * 32), (int)(tb + tc0), buf);
          tc::bulk_commit_group();
        }
        return;
      }
      __syncwarp();
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int r = (lane >> 2) + 8 * j, m = lane & 3;  // token row, 8-value piece
        if (tc0 + r < Lc) {
          const uint4 piece = *reinterpret_cast<const uint4*>(buf + r * 64 + m * 16);
          *reinterpret_cast<uint4*>(dst + (tb + tc0 + r) * (H * V) + (int64_t)h * V +
                                    quarter * 32 + m * 8) = piece;
        }
      }
    };
    auto write_out = [&](int64_t tb, int Lc) {
      uint32_t ra[8], rb[8];  // values 0-15 and 16-31 of the warp's lanes
      tc::tmem_ld16x256b_x2(tm_addr(tm, quarter, C_TM_O + tc0), ra);
      tc::tmem_ld16x256b_x2(tm_addr(tm, quarter, C_TM_O + tc0) + (16u << 16), rb);
      if (lane == 0) tc::bulk_wait_read<0>();  // the previous store has read the buffer
      tc::tmem_wait_ld();
      __syncwarp();
      {
        const float2 sc2 = make_float2(scale, scale);
        auto pk = [&](uint32_t x, uint32_t y) {
          return pack2<bf16>(fmul2(make_float2(__uint_as_float(x), __uint_as_float(y)), sc2));
        };
        // 8 x 8 blocks (values vb.., tokens 8 (mi >> 1)..): thread t gives
        // the shared row of token row t % 8 of block t / 8
        const int mi = lane >> 3, tok = ((mi >> 1) << 3) + (lane & 7), vb = (mi & 1) << 3;
        stmatrix_x4_trans(ost + tok * 64 + vb * 2, pk(ra[0], ra[1]), pk(ra[2], ra[3]),
                          pk(ra[4], ra[5]), pk(ra[6], ra[7]));
        stmatrix_x4_trans(ost + tok * 64 + (16 + vb) * 2, pk(rb[0], rb[1]), pk(rb[2], rb[3]),
                          pk(rb[4], rb[5]), pk(rb[6], rb[7]));
      }
      if (store_o) store_rows(&tm_o, o, ost, tb, Lc);
    };
    // chunk c's y from the o rows write_out left in ost (and its z rows)
    auto norm_out = [&](int64_t tb, int Lc) -> bool {
      __syncwarp();  // every lane's transposed rows are in ost
      if (!norm_rows()) return false;
      store_rows(&tm_y, nrm.y, ost, tb, Lc);
      return true;
    };
    auto apply_ds = [&](float dl) {  // S = e^{gl} S + dS
      const float2 dl2 = make_float2(dl, dl);
      float d[32];  // both 16-column loads in flight before one wait
      tc::tmem_ld16(tm_addr(tm, quarter, C_TM_DS + kc0), *reinterpret_cast<float(*)[16]>(d));
      tc::tmem_ld16(tm_addr(tm, quarter, C_TM_DS + kc0 + 16), *reinterpret_cast<float(*)[16]>(d + 16));
      tc::tmem_wait_ld();
#pragma unroll
      for (int m = 0; m < 16; ++m) S[m] = ffma2(S[m], dl2, make_float2(d[2 * m], d[2 * m + 1]));
    };
    // D_qh starts at zero: the [-w; q] product accumulates into it
    if (write_o) tc::tmem_st16_zero(tm_addr(tm, quarter, C_TM_QH + tc0));
    for (int i = 0; i < NI; ++i) {
      const int s = i & 1;
      // the abort flag and e^{gl} are read ahead of the wait, off the critical path
      const bool aborted = *(volatile int*)&abort_sh != 0;
      if (i > 0) {
        const float dl = __expf(gl_prev);
        if (!(live = wait_ok(&bar_s, (i - 1) & 1))) break;
        apply_ds(dl);
      }
      if (aborted) { live = false; break; }
      // E0: bf16 S^T -> TMEM (columns kc0/2 .. kc0/2 + 15), then let the MMA warp go
      {
        uint32_t pk[16];
#pragma unroll
        for (int m = 0; m < 16; ++m) pk[m] = pack2<bf16>(S[m]);
        tc::tmem_st16u(tm_addr(tm, quarter, C_TM_HT + kc0 / 2), pk);
      }
      warp_arrive(&bar_ht);
      if (norm && i > 0) {  // while the tensor core forms [-w; q] of this chunk
        // chunk i - 2: a whole chunk (only a sequence's last chunk is partial)
        if (i > 1 && !(live = norm_out(t0_prev - BT, BT))) break;
        load_z(t0_prev, L_prev);
      }
      if (!(live = wait_ok(&full[s], (i >> 1) & 1))) break;
      const float* tab = reinterpret_cast<const float*>(sm + C_OFF_TAB + (i & 3) * C_TAB);
      float4 ev[4];  // the chunk's e^{gl-gc} (ready with the stage), before the product lands
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) ev[q4] = *reinterpret_cast<const float4*>(tab + tc0 + 4 * q4);
      const int64_t t0 = bos + (int64_t)(c0 + i) * BT;
      const int L = (int)((eos - t0) < BT ? (eos - t0) : BT);
      if (!(live = wait_ok(&bar_v, i & 1))) break;
      // E1a: v_new = D_u (exact diagonal included); vt = v_new e^{gl-gc} as
      // bf16 hi + lo for the state product (critical path: hand it over first)
      float du[16];
      tc::tmem_ld16(tm_addr(tm, quarter, C_TM_U + tc0), du);
      tc::tmem_wait_ld();
      {
        uint32_t hi[8], lo[8];
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float4 e4 = ev[q4];
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            const int u = 2 * q4 + p;
            const float2 sc = fmul2(make_float2(du[2 * u], du[2 * u + 1]),
                                    p == 0 ? make_float2(e4.x, e4.y) : make_float2(e4.z, e4.w));
            hi[u] = pack2<bf16>(sc);
            lo[u] = pack2<bf16>(fsub2(sc, unpack2<bf16>(hi[u])));
          }
        }
        tc::tmem_st8u(tm_addr(tm, quarter, C_TM_VTH + tc0 / 2), hi);
        tc::tmem_st8u(tm_addr(tm, quarter, C_TM_VTL + tc0 / 2), lo);
      }
      warp_arrive(&bar_vt);
      gl_prev = tab[128];
      if (write_o) {
        // the previous chunk's output (its product ran behind this chunk's
        // [-w; q] product) while the tensor core forms dS
        if (i > 0) {
          if (!(live = wait_ok(&bar_od, (i - 1) & 1))) break;
          write_out(t0_prev, L_prev);
        }
        // E1b, while the tensor core forms dS: D_o = e^{gc} D_qh (the previous
        // chunk's output has just been read out of it), bf16 v_new -> TMEM
        if (!(live = wait_ok(&bar_q, i & 1))) break;
        float qh[16];
        tc::tmem_ld16(tm_addr(tm, quarter, C_TM_QH + tc0), qh);
        tc::tmem_wait_ld();
        tc::tmem_st16_zero(tm_addr(tm, quarter, C_TM_QH + tc0));
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const float4 e4 = *reinterpret_cast<const float4*>(tab + 64 + tc0 + 4 * q4);
          const float2 a = fmul2(make_float2(qh[4 * q4], qh[4 * q4 + 1]), make_float2(e4.x, e4.y));
          const float2 b = fmul2(make_float2(qh[4 * q4 + 2], qh[4 * q4 + 3]), make_float2(e4.z, e4.w));
          qh[4 * q4] = a.x; qh[4 * q4 + 1] = a.y; qh[4 * q4 + 2] = b.x; qh[4 * q4 + 3] = b.y;
        }
        tc::tmem_st16(tm_addr(tm, quarter, C_TM_O + tc0), qh);
        uint32_t vn[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) vn[u] = pack2<bf16>(make_float2(du[2 * u], du[2 * u + 1]));
        tc::tmem_st8u(tm_addr(tm, quarter, C_TM_VN + tc0 / 2), vn);
        warp_arrive(&bar_o);
      }
      L_prev = L;
      t0_prev = t0;
    }
    if (live && NI > 0) {
      if ((live = wait_ok(&bar_s, (NI - 1) & 1))) apply_ds(__expf(gl_prev));
      if (live && norm) {
        if (NI > 1) live = norm_out(t0_prev - BT, BT);
        load_z(t0_prev, L_prev);
      }
      if (live && write_o && (live = wait_ok(&bar_od, (NI - 1) & 1))) {
        write_out(t0_prev, L_prev);
        if (norm) live = norm_out(t0_prev, L_prev);
      }
    }
    cp_async_wait_all();  // no z copy outlives the loop
    if (live && it_out) {
      float* dst = it_out;
#pragma unroll
      for (int m = 0; m < C_SCOLS / 2; ++m) {
        dst[(kc0 + 2 * m) * V + vrow] = S[m].x;
        dst[(kc0 + 2 * m + 1) * V + vrow] = S[m].y;
      }
    }
  }
  // the output stores have completed before the CTA exits
  if (warp >= 2 && lane == 0) tc::bulk_wait_all();
  tc::fence_before();
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tm, C_TM_COLS);
}

// ============================================================================
// Kernel 3: segment start states, h_{s+1} = X_s^T h_s + B_s (fp32)
// ============================================================================
// Serial over the middle segments of one (sequence, head):
//   h_{s+1}[kk][c] = sum_r X_s^T[kk][r] h_s[r][c] + B_s[kk][c].
// The value columns c are independent, so each (sequence, head) is cut into
// column slices of COLS; and the sum over r is cut over a cluster of CB_CR
// CTAs: CTA j of a slice holds rows r in [32 j, 32 j + 32) of h_s and only
// those 32 columns of every X^T row (16 KB a step, not the whole 64 KB
// matrix; the transitions stream through L2 once per slice, not once per
// CTA).  CTA j computes the partial sums of all 128 output rows and sends
// those of rows [32 q, 32 q + 32) to CTA q's receive slot j with
// asynchronous distributed-shared-memory stores that complete on CTA q's
// transaction barrier `full`; CTA q adds its four slots (in rank order) and
// B, which gives exactly the rows of h_{s+1} it holds for the next step, and
// hands the slot set back to the writers through their `empty` barriers.
// Slot sets alternate between steps.  X_{s+1} and B_{s+1} are requested
// (cp.async) at the start of step s.  Every wait is bounded: on a timeout the
// CTA records the error and leaves its loop; the cluster then meets at the
// exit barrier, so no CTA leaves while another may still write into it.
// CB_NT worker threads compute; one more warp (the producer) issues the copies
constexpr int CB_NT = 256, CB_THREADS = CB_NT + 32, CB_CR = 4, CB_XLD = 36;  // X^T part rows: 32 floats + 4 padding
// shared bytes of a COLS-column CTA: two X^T parts, h_s rows, two B row sets,
// two sets of CB_CR receive slots [32][COLS]
constexpr int cb_smem(int cols) {
  return (2 * 128 * CB_XLD + 32 * cols + 2 * 32 * cols + 2 * CB_CR * 32 * cols) * 4 + 16;
}

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::
                   : "memory");
}
__device__ __forceinline__ uint32_t mapa(uint32_t local, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(local), "r"(rank));
  return remote;
}
// 16 bytes into another CTA's shared memory, completing on its barrier
__device__ __forceinline__ void st_async_f4(uint32_t raddr, uint32_t rbar, float4 v) {
  asm volatile(
      "st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];\n" ::"r"(
          raddr),
      "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(rbar)
      : "memory");
}
// announce `bytes` of incoming transfers on a local barrier (this arrival
// publishes no data of its own, so it needs no release ordering)
__device__ __forceinline__ void mbar_expect_relaxed(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.relaxed.cta.shared::cta.b64 _, [%0], %1;\n" ::"r"(
                   tc::smem_addr(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t rbar) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(rbar)
               : "memory");
}
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, uint32_t limit) {
  const uint32_t addr = tc::smem_addr(bar);
  for (uint32_t i = 0; i < limit; ++i) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}\n"
        : "=r"(ok)
        : "r"(addr), "r"(parity)
        : "memory");
    if (ok) return true;
  }
  return false;
}

template <int COLS>
__global__ void __launch_bounds__(CB_THREADS) chunk_combine_kernel(const int32_t* __restrict__ cu,
                                                              int64_t N, int64_t T, int64_t H,
                                                              ChainPlan plan) {
  constexpr int NCC = COLS / 4;            // 4-column chunks
  constexpr int NKG = CB_NT / NCC;         // output row groups
  constexpr int KB = 128 / NKG;            // rows per group: kg, kg + NKG, ...
  constexpr int FPT = (32 * NCC) / CB_NT > 0 ? (32 * NCC) / CB_NT : 1;  // finals per thread
  constexpr int FT = 32 * NCC < CB_NT ? 32 * NCC : CB_NT;  // threads that finalise
  constexpr int SLOT = 32 * COLS;          // floats per receive slot
  constexpr uint32_t RX_BYTES = (CB_CR - 1) * SLOT * 4;  // remote bytes per step
  static_assert(COLS % 16 == 0 && COLS <= 128 && KB * NKG == 128, "combine tiling");
  extern __shared__ __align__(16) float cbs[];
  float* xbuf = cbs;                             // two X^T parts [128][CB_XLD]
  float* hcur = xbuf + 2 * 128 * CB_XLD;         // h_s rows [32][COLS]
  float* bbuf = hcur + SLOT;                     // two B row sets [32][COLS]
  float* rbuf = bbuf + 2 * SLOT;                 // [2][CB_CR][32][COLS] receive slots
  __shared__ uint64_t full[2], empty[2];
  __shared__ int64_t slot_sh;
  __shared__ int nseg_sh, abort_sh;
  const int tid = threadIdx.x;
  const bool producer = tid >= CB_NT;
  const int lane = tid & 31;
  const int j = (int)cluster_rank();
  const int64_t n = blockIdx.y / H;
  const int h = (int)(blockIdx.y - n * H);
  const int v0 = (blockIdx.x / CB_CR) * COLS;
  if (tid == 0) {
    int64_t slot = 0;
    int nseg = 1;
    for (int64_t m = 0; m <= n; ++m) {
      const int nc = seq_chunks(cu, m, T);
      nseg = nc > plan.seg ? (nc + plan.seg - 1) / plan.seg : 1;
      if (m < n) slot += nseg;
    }
    slot_sh = slot;
    nseg_sh = nseg;
    abort_sh = 0;
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&full[b], 1);
      tc::mbar_init(&empty[b], CB_CR - 1);
    }
    tc::mbar_fence_init();
  }
  // barriers initialised cluster-wide before any CTA stores into another
  cluster_sync();
  const int nseg = nseg_sh;
  const int64_t slot = slot_sh;
  const int cc = tid % NCC, kg = tid / NCC;
  // X^T rows [kk][32 j .. 32 j + 31] and B rows [32 j .. 32 j + 31][v0 ..
  // v0 + COLS) of transition s, as one cp.async group of the producer warp
  auto load_step = [&](int s, int buf) {
    const float* xs = seg_state(plan, slot + s, H, h, 2);
    float* xd = xbuf + buf * 128 * CB_XLD;
    for (int e = lane; e < 128 * 8; e += 32) {
      const int row = e >> 3, q4 = e & 7;
      cp_async16(xd + row * CB_XLD + q4 * 4, xs + row * 128 + 32 * j + q4 * 4, 16);
    }
    const float* bs = seg_state(plan, slot + s, H, h, 1) + v0;
    float* bd = bbuf + buf * SLOT;
    for (int e = lane; e < 32 * NCC; e += 32) {
      const int r = e / NCC, c4 = e % NCC;
      cp_async16(bd + r * COLS + 4 * c4, bs + (32 * j + r) * 128 + 4 * c4, 16);
    }
    cp_async_commit();
  };
  if (nseg >= 3) {
    if (producer) load_step(1, 0);
    const float* h1 = seg_state(plan, slot + 1, H, h, 0) + v0;
    for (int e = tid; e < 32 * NCC; e += CB_THREADS) {
      const int r = e / NCC, c4 = e % NCC;
      *reinterpret_cast<float4*>(hcur + r * COLS + 4 * c4) =
          *reinterpret_cast<const float4*>(h1 + (32 * j + r) * 128 + 4 * c4);
    }
    cp_async_wait_all();
    __syncthreads();
  }
  const uint32_t rbuf_a = tc::smem_addr(rbuf);
  for (int s = 1; s <= nseg - 2; ++s) {
    const int b = (s - 1) & 1;
    const uint32_t use = (uint32_t)((s - 1) >> 1);  // how often slot set b was used before
    if (producer) {
      if (s + 1 <= nseg - 2) load_step(s + 1, b ^ 1);
      if (lane == 0) mbar_expect_relaxed(&full[b], RX_BYTES);
      __syncthreads();
      if (*(volatile int*)&abort_sh) break;
      if (s + 1 <= nseg - 2) cp_async_wait_all();  // X_{s+1}, B_{s+1} have landed
      __syncthreads();
      continue;
    }
    const float* xs = xbuf + b * 128 * CB_XLD;
    float acc[KB][4];
#pragma unroll
    for (int i = 0; i < KB; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.f;
#pragma unroll
    for (int r = 0; r < 32; r += 4) {
      float4 hv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        hv[u] = *reinterpret_cast<const float4*>(hcur + (r + u) * COLS + 4 * cc);
#pragma unroll
      for (int i = 0; i < KB; ++i) {
        const float4 x4 = *reinterpret_cast<const float4*>(xs + (kg + i * NKG) * CB_XLD + r);
        const float xv[4] = {x4.x, x4.y, x4.z, x4.w};
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          acc[i][0] = fmaf(xv[u], hv[u].x, acc[i][0]);
          acc[i][1] = fmaf(xv[u], hv[u].y, acc[i][1]);
          acc[i][2] = fmaf(xv[u], hv[u].z, acc[i][2]);
          acc[i][3] = fmaf(xv[u], hv[u].w, acc[i][3]);
        }
      }
    }
    // the owners have read this slot set's previous use
    bool ok = use == 0 || mbar_wait_cluster(&empty[b], (use - 1) & 1, WAIT_LIMIT);
    // row kk's partial goes to slot j of its owner CTA kk / 32
    const uint32_t slot_off = (uint32_t)((b * CB_CR + j) * SLOT) * 4u;
#pragma unroll
    for (int i = 0; i < KB && ok; ++i) {
      const int kk = kg + i * NKG;
      const int q = kk >> 5;
      const float4 v = make_float4(acc[i][0], acc[i][1], acc[i][2], acc[i][3]);
      const uint32_t off = slot_off + (uint32_t)(((kk & 31) * COLS + 4 * cc) * 4);
      if (q == j)
        *reinterpret_cast<float4*>(reinterpret_cast<unsigned char*>(rbuf) + off) = v;
      else
        st_async_f4(mapa(rbuf_a + off, (uint32_t)q), mapa(tc::smem_addr(&full[b]), (uint32_t)q), v);
    }
    ok = ok && mbar_wait_cluster(&full[b], use & 1, WAIT_LIMIT);
    if (!ok) {
      record_error();
      atomicExch(&abort_sh, 1);
    }
    __syncthreads();  // own slot written, every read of h_s done, abort flag seen
    if (*(volatile int*)&abort_sh) break;
    float* gout = seg_state(plan, slot + s + 1, H, h, 0) + v0;
    const float* bsrc = bbuf + b * SLOT;
    const float* rb = rbuf + b * CB_CR * SLOT;
#pragma unroll
    for (int f = 0; f < FPT; ++f) {
      if (tid >= FT) break;
      const int e = tid + f * CB_NT, fr = e / NCC, fc = e % NCC;
      const float* src = rb + fr * COLS + 4 * fc;
      float4 t = *reinterpret_cast<const float4*>(src);
#pragma unroll
      for (int q = 1; q < CB_CR; ++q) {  // partials in cluster-rank order
        const float4 p = *reinterpret_cast<const float4*>(src + q * SLOT);
        t.x += p.x; t.y += p.y; t.z += p.z; t.w += p.w;
      }
      const float4 bb = *reinterpret_cast<const float4*>(bsrc + fr * COLS + 4 * fc);
      t.x += bb.x; t.y += bb.y; t.z += bb.z; t.w += bb.w;
      *reinterpret_cast<float4*>(hcur + fr * COLS + 4 * fc) = t;
      *reinterpret_cast<float4*>(gout + (32 * j + fr) * 128 + 4 * fc) = t;
    }
    __syncthreads();  // slot set b read; h_{s+1} rows, X_{s+1}, B_{s+1} visible
    if (tid < CB_CR && tid != j)  // hand slot set b back to the other writers
      mbar_arrive_remote(mapa(tc::smem_addr(&empty[b]), (uint32_t)tid));
  }
  cp_async_wait_all();
  // no CTA leaves while another may still store into its receive slots
  cluster_sync();
}

}  // namespace
}  // namespace gdn
}  // namespace xops

using namespace xops;

static int64_t chunk_bound(const int32_t* cu, int64_t B, int64_t T, int64_t N) {
  return cu ? T / gdn::BT + N : B * ((T + gdn::BT - 1) / gdn::BT);
}

// Segment length (in chunks) for the chain, 0 = unsegmented.  The host does
// not know the sequence lengths (cu_seqlens stays on the device), so the plan
// assumes the worst case of one sequence holding every chunk and picks the
// segment count P minimising (phase-1 waves + phase-3 waves) x segment length
// + combine steps, counted in chunk steps on a 148-SM B200.  Segmenting runs
// each chunk of a middle segment three times (local, transition, output) on
// otherwise idle SMs, so it only pays when (sequence, head) pairs are scarce.
static int chain_segment_chunks(int64_t B, int64_t T, int64_t N, int64_t H, bool varlen) {
  constexpr int64_t kSMs = 148;
  const int64_t C = (T + gdn::BT - 1) / gdn::BT;  // longest possible chain
  (void)B;
  if (N * H >= kSMs || C < 32) return 0;
  const int64_t others = varlen ? (N - 1) * H : 0;  // the other sequences' first items
  const int64_t pairs = varlen ? H : N * H;
  const double plain = (double)((N * H + kSMs - 1) / kSMs) * (double)C;
  double best = plain;
  int best_seg = 0;
  for (int64_t P = 3; P <= 64; ++P) {
    const int64_t seg = (C + P - 1) / P;
    if (seg < 8) break;
    const int64_t nseg = (C + seg - 1) / seg;
    const int64_t items1 = pairs * (1 + 2 * (nseg - 2)) + others;
    const int64_t items3 = pairs * (nseg - 1);
    const double cost = (double)((items1 + kSMs - 1) / kSMs + (items3 + kSMs - 1) / kSMs) * seg +
                        (double)(nseg - 2);
    if (cost < best) {
      best = cost;
      best_seg = (int)seg;
    }
  }
  return best < 0.9 * plain ? best_seg : 0;
}

// Upper bound of the segment slots (sum over sequences of their segment count).
static int64_t chain_segment_slots(int64_t T, int64_t N, bool varlen, int seg) {
  if (seg == 0) return 0;
  const int64_t C = (T + gdn::BT - 1) / gdn::BT;
  if (!varlen) return N * ((C + seg - 1) / seg);
  return (C + N + seg - 1) / seg + N;
}

static int64_t round_up256(int64_t x) { return (x + 255) / 256 * 256; }

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// dependency on libcuda).
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
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

// bf16 rows of `cols` elements, `rows` rows `stride` elements apart, moved
// as box_cols x box_rows boxes (64 x 64 with the 128-byte swizzle by
// default).  Loads read rows past `rows` as zero; stores drop them.
static int token_rows_map(CUtensorMap* m, const void* base, int64_t cols, int64_t rows,
                          int64_t stride, const char* what, uint32_t box_cols = 64,
                          uint32_t box_rows = 64, bool swizzle = true) {
  auto enc = tensor_map_encoder();
  if (!enc) return set_error(XOPS_ERR_CUDA, "%s: cuTensorMapEncodeTiled is unavailable", what);
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(stride * 2)};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                         strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(XOPS_ERR_CUDA, "%s: tensor map encoding failed (%d)", what, (int)r);
  return XOPS_OK;
}

extern "C" int64_t xops_chunk_gated_delta_rule_workspace_size(int64_t B, int64_t T, int64_t N,
                                                              int64_t Hg, int64_t H, int64_t K,
                                                              int use_qk_l2norm_in_kernel,
                                                              int varlen) {
  if (B < 1 || T < 0 || N < 0 || Hg < 1 || H < 1 || K <= 0) return -1;
  const int64_t chunks = varlen ? T / gdn::BT + N : B * ((T + gdn::BT - 1) / gdn::BT);
  int64_t bytes = chunks * H * (int64_t)gdn::WS_CHUNK;
  if (use_qk_l2norm_in_kernel) bytes += round_up256(2 * B * T * Hg * K * 2);
  const int seg = chain_segment_chunks(B, T, N, H, varlen != 0);
  bytes += chain_segment_slots(T, N, varlen != 0, seg) * H * 3 * (int64_t)gdn::KV * 4;
  return bytes;
}

// The chunked rule behind both C-ABI entries; `gs` says where the gates
// come from.
static int chunk_gdn_run(const void* q, const void* k, const void* v, const gdn::GateSrc& gs,
                         const float* h0, void* o, float* ht, const int32_t* cu_seqlens,
                         int64_t B, int64_t T, int64_t N, int64_t Hg, int64_t H, int64_t K,
                         int64_t V, int64_t q_token_stride, int64_t k_token_stride,
                         int64_t v_token_stride, float scale, int use_qk_l2norm_in_kernel,
                         void* workspace, int64_t workspace_bytes, void* stream,
                         const gdn::OutNorm* nrm = nullptr) {
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
  XOPS_REQUIRE(q && k && v && (o || nrm) && (gs.g ? gs.beta != nullptr
                                                  : gs.a && gs.b && gs.A_log && gs.dt_bias),
               "chunk_gated_delta_rule: null pointer");
  XOPS_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && (!o || aligned16(o)),
               "chunk_gated_delta_rule: tensors must be 16-byte aligned");
  const int64_t need = xops_chunk_gated_delta_rule_workspace_size(
      B, T, N, Hg, H, K, use_qk_l2norm_in_kernel, cu_seqlens != nullptr);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return set_error(XOPS_ERR_WORKSPACE,
                     "chunk_gated_delta_rule: workspace of %lld bytes (16-byte aligned) required, "
                     "got %lld", (long long)need, (long long)workspace_bytes);
  cudaStream_t st = (cudaStream_t)stream;
  unsigned char* ws = static_cast<unsigned char*>(workspace);
  const gdn::bf16* qq = (const gdn::bf16*)q;
  const gdn::bf16* kk = (const gdn::bf16*)k;
  int64_t qs = q_token_stride, ks = k_token_stride;
  const int64_t nchunks = chunk_bound(cu_seqlens, B, T, N);
  if (use_qk_l2norm_in_kernel) {
    gdn::bf16* qn = reinterpret_cast<gdn::bf16*>(ws + nchunks * H * (int64_t)gdn::WS_CHUNK);
    gdn::bf16* kn = qn + B * T * Hg * K;
    const int64_t rows = B * T * Hg;
    // bulk-copy streaming path when the shape suits it, else a warp per row
    for (int which = 0; which < 2; ++which) {
      const gdn::bf16* src = which ? kk : qq;
      gdn::bf16* dst = which ? kn : qn;
      const int64_t stride = which ? ks : qs;
      int rc = xops::l2norm_rows_stream(src, dst, B * T, Hg, stride, 1e-6f, st);
      if (rc < 0) {
        gdn::l2norm_heads_kernel<<<(unsigned)cdiv64(rows, 8), 256, 0, st>>>(src, dst, rows, Hg,
                                                                            stride);
        rc = check_launch(which ? "chunk_gated_delta_rule(l2norm k)"
                                : "chunk_gated_delta_rule(l2norm q)");
      }
      if (rc) return rc;
    }
    qq = qn;
    kk = kn;
    qs = ks = Hg * K;
  }
  CUtensorMap mq, mk, mv;
  if (int rc = token_rows_map(&mq, qq, Hg * K, B * T, qs, "chunk_gated_delta_rule(q map)"))
    return rc;
  if (int rc = token_rows_map(&mk, kk, Hg * K, B * T, ks, "chunk_gated_delta_rule(k map)"))
    return rc;
  if (H == 2 * Hg) {  // two value heads per key head: both in one CTA
    if (int rc = gdn::ensure_smem_attr((const void*)gdn::chunk_prep_pair_tc_kernel, gdn::P3_SMEM,
                                       "chunk_gated_delta_rule(prep)"))
      return rc;
    gdn::chunk_prep_pair_tc_kernel<<<dim3((unsigned)nchunks, (unsigned)Hg), gdn::P_NT,
                                     gdn::P3_SMEM, st>>>(mq, mk, gs, ws, cu_seqlens, N, T, Hg, H);
  } else {
    if (int rc = gdn::ensure_smem_attr((const void*)gdn::chunk_prep_kernel, gdn::P_SMEM,
                                       "chunk_gated_delta_rule(prep)"))
      return rc;
    gdn::chunk_prep_kernel<<<dim3((unsigned)nchunks, (unsigned)Hg), gdn::P_NT, gdn::P_SMEM, st>>>(
        qq, kk, gs, ws, cu_seqlens, N, T, Hg, H, qs, ks);
  }
  if (int rc = check_launch("chunk_gated_delta_rule(prep)")) return rc;
  auto chain = nrm ? gdn::chunk_chain_kernel<true> : gdn::chunk_chain_kernel<false>;
  if (int rc = gdn::ensure_smem_attr((const void*)chain, gdn::C_SMEM,
                                     "chunk_gated_delta_rule(chain)"))
    return rc;
  if (int rc = token_rows_map(&mv, v, H * V, B * T, v_token_stride,
                              "chunk_gated_delta_rule(v map)"))
    return rc;
  // o (and y) as [tokens, H * V]: each epilogue warp stores 16 tokens x 32 values
  CUtensorMap mo, my;
  gdn::OutNorm on{};
  if (nrm) {
    on = *nrm;
    on.keep_o = o != nullptr;
    if (int rc = token_rows_map(&my, on.y, H * V, B * T, H * V, "chunk_gated_delta_rule(y map)",
                                32, 16, false))
      return rc;
  }
  if (int rc = token_rows_map(&mo, o ? o : on.y, H * V, B * T, H * V,
                              "chunk_gated_delta_rule(o map)", 32, 16, false))
    return rc;
  if (!nrm) my = mo;
  const bool varlen = cu_seqlens != nullptr;
  const int seg = chain_segment_chunks(B, T, N, H, varlen);
  gdn::ChainPlan plan{seg, 1, nullptr};
  if (seg == 0) {
    chain<<<(unsigned)(N * H), gdn::C_NT, gdn::C_SMEM, st>>>(
        mq, mk, mv, mo, my, h0, ws, (gdn::bf16*)o, ht, cu_seqlens, N, T, Hg, H, scale,
      plan, on);
    return check_launch("chunk_gated_delta_rule(chain)");
  }
  // Segment-parallel chain: grids are upper bounds, spare CTAs exit at once.
  int64_t off = nchunks * H * (int64_t)gdn::WS_CHUNK;
  if (use_qk_l2norm_in_kernel) off += round_up256(2 * B * T * Hg * K * 2);
  plan.scratch = reinterpret_cast<float*>(ws + off);
  const int64_t slots = chain_segment_slots(T, N, varlen, seg);
  chain<<<(unsigned)((N + 2 * slots) * H), gdn::C_NT, gdn::C_SMEM, st>>>(
      mq, mk, mv, mo, my, h0, ws, (gdn::bf16*)o, ht, cu_seqlens, N, T, Hg, H, scale,
      plan, on);
  if (int rc = check_launch("chunk_gated_delta_rule(chain, first segments)")) return rc;
  {
    // the narrowest column slice whose clusters (4 CTAs each) still fit one
    // wave of one CTA per SM
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess)
      cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int cols = 16;
    while (cols < 128 && (int64_t)N * H * (128 / cols) * gdn::CB_CR > sms) cols *= 2;
    auto launch = [&](auto kern, int c) -> int {
      if (int rc = gdn::ensure_smem_attr((const void*)kern, gdn::cb_smem(c),
                                         "chunk_gated_delta_rule(combine)"))
        return rc;
      cudaLaunchConfig_t lc = {};
      lc.gridDim = dim3((unsigned)((128 / c) * gdn::CB_CR), (unsigned)(N * H));
      lc.blockDim = dim3(gdn::CB_THREADS);
      lc.dynamicSmemBytes = (size_t)gdn::cb_smem(c);
      lc.stream = st;
      cudaLaunchAttribute at[1];
      at[0].id = cudaLaunchAttributeClusterDimension;
      at[0].val.clusterDim.x = gdn::CB_CR;
      at[0].val.clusterDim.y = 1;
      at[0].val.clusterDim.z = 1;
      lc.attrs = at;
      lc.numAttrs = 1;
      if (cudaLaunchKernelEx(&lc, kern, (const int32_t*)cu_seqlens, N, T, H, plan) != cudaSuccess)
        return set_error(XOPS_ERR_CUDA, "chunk_gated_delta_rule(combine): cluster launch failed");
      return 0;
    };
    int rc = cols == 16   ? launch(gdn::chunk_combine_kernel<16>, 16)
             : cols == 32 ? launch(gdn::chunk_combine_kernel<32>, 32)
             : cols == 64 ? launch(gdn::chunk_combine_kernel<64>, 64)
                          : launch(gdn::chunk_combine_kernel<128>, 128);
    if (rc) return rc;
  }
  if (int rc = check_launch("chunk_gated_delta_rule(combine)")) return rc;
  plan.phase = 3;
  chain<<<(unsigned)(slots * H), gdn::C_NT, gdn::C_SMEM, st>>>(
      mq, mk, mv, mo, my, h0, ws, (gdn::bf16*)o, ht, cu_seqlens, N, T, Hg, H, scale,
      plan, on);
  return check_launch("chunk_gated_delta_rule(chain, remaining segments)");
}

extern "C" int xops_chunk_gated_delta_rule(const void* q, const void* k, const void* v,
                                           const float* g, const float* beta, const float* h0,
                                           void* o, float* ht, const int32_t* cu_seqlens,
                                           int64_t B, int64_t T, int64_t N, int64_t Hg,
                                           int64_t H, int64_t K, int64_t V,
                                           int64_t q_token_stride, int64_t k_token_stride,
                                           int64_t v_token_stride, float scale,
                                           int use_qk_l2norm_in_kernel, void* workspace,
                                           int64_t workspace_bytes, void* stream) {
  gdn::GateSrc gs{};
  gs.g = g;
  gs.beta = beta;
  return chunk_gdn_run(q, k, v, gs, h0, o, ht, cu_seqlens, B, T, N, Hg, H, K, V, q_token_stride,
                       k_token_stride, v_token_stride, scale, use_qk_l2norm_in_kernel, workspace,
                       workspace_bytes, stream);
}

// The gates of the fused-gating entries, from the layer's projections.
static int gated_source(const float* A_log, const void* a, const void* b, const float* dt_bias,
                        int a_dtype, int b_dtype, int64_t ab_token_stride, int ba_interleaved,
                        float softplus_beta, float softplus_threshold, int64_t Hg, int64_t H,
                        gdn::GateSrc* out) {
  auto ok_dtype = [](int d) { return d == XOPS_F32 || d == XOPS_BF16 || d == XOPS_F16; };
  XOPS_REQUIRE(ok_dtype(a_dtype) && ok_dtype(b_dtype),
               "chunk_gated_delta_rule_gated: a and b must be fp32, bf16 or fp16");
  XOPS_REQUIRE(softplus_beta > 0.f, "chunk_gated_delta_rule_gated: softplus beta must be positive");
  XOPS_REQUIRE(!ba_interleaved || (a == b && a_dtype == b_dtype && Hg >= 1 && H % Hg == 0),
               "chunk_gated_delta_rule_gated: an interleaved mixed_ba passes the same tensor as "
               "a and b");
  if (ab_token_stride == 0) ab_token_stride = ba_interleaved ? 2 * H : H;
  XOPS_REQUIRE(ab_token_stride >= (ba_interleaved ? 2 * H : H),
               "chunk_gated_delta_rule_gated: a/b token stride smaller than the row");
  gdn::GateSrc gs{};
  gs.a = a;
  gs.b = b;
  gs.A_log = A_log;
  gs.dt_bias = dt_bias;
  gs.sp_beta = softplus_beta;
  gs.sp_thr = softplus_threshold;
  gs.a_dt = a_dtype;
  gs.b_dt = b_dtype;
  gs.ab_ld = ab_token_stride;
  gs.ba_r = ba_interleaved ? (int)(H / Hg) : 0;
  *out = gs;
  return XOPS_OK;
}

extern "C" int xops_chunk_gated_delta_rule_gated(
    const void* q, const void* k, const void* v, const float* A_log, const void* a, const void* b,
    const float* dt_bias, int a_dtype, int b_dtype, int64_t ab_token_stride, int ba_interleaved,
    float softplus_beta, float softplus_threshold,
    const float* h0, void* o, float* ht, const int32_t* cu_seqlens, int64_t B, int64_t T,
    int64_t N, int64_t Hg, int64_t H, int64_t K, int64_t V, int64_t q_token_stride,
    int64_t k_token_stride, int64_t v_token_stride, float scale, int use_qk_l2norm_in_kernel,
    void* workspace, int64_t workspace_bytes, void* stream) {
  gdn::GateSrc gs{};
  if (int rc = gated_source(A_log, a, b, dt_bias, a_dtype, b_dtype, ab_token_stride,
                            ba_interleaved, softplus_beta, softplus_threshold, Hg, H, &gs))
    return rc;
  return chunk_gdn_run(q, k, v, gs, h0, o, ht, cu_seqlens, B, T, N, Hg, H, K, V, q_token_stride,
                       k_token_stride, v_token_stride, scale, use_qk_l2norm_in_kernel, workspace,
                       workspace_bytes, stream);
}

// Checks and fills the fused output norm of the _out_norm entries.
static int out_norm_args(const void* z, int64_t z_token_stride, int64_t z_heads_per_group,
                         int64_t z_group_stride, const void* norm_weight, int weight_dtype,
                         float eps, void* y, int64_t N, int64_t T, int64_t H, int64_t V,
                         gdn::OutNorm* out) {
  XOPS_REQUIRE(weight_dtype == XOPS_F32 || weight_dtype == XOPS_BF16,
               "chunk_gated_delta_rule_out_norm: the norm weight must be fp32 or bf16");
  if (z_heads_per_group <= 0) z_heads_per_group = 1;
  if (z_group_stride == 0) z_group_stride = z_heads_per_group * V;
  if (z_token_stride == 0) z_token_stride = (H / z_heads_per_group) * z_group_stride;
  XOPS_REQUIRE(H % z_heads_per_group == 0 && z_group_stride >= z_heads_per_group * V &&
                   z_group_stride % 8 == 0 && z_token_stride % 8 == 0 &&
                   z_token_stride >= ((H / z_heads_per_group - 1) * z_group_stride +
                                      z_heads_per_group * V),
               "chunk_gated_delta_rule_out_norm: z strides must cover the heads and be "
               "multiples of 8");
  if (N > 0 && T > 0)
    XOPS_REQUIRE(z && norm_weight && y && aligned16(z) && aligned16(y),
                 "chunk_gated_delta_rule_out_norm: z, weight and y must be given, z and y "
                 "16-byte aligned");
  gdn::OutNorm nrm{};
  nrm.z = static_cast<const gdn::bf16*>(z);
  nrm.w = norm_weight;
  nrm.y = static_cast<gdn::bf16*>(y);
  nrm.ldz = z_token_stride;
  nrm.zgs = z_group_stride;
  nrm.zr = (int)z_heads_per_group;
  nrm.eps = eps;
  nrm.w_f32 = weight_dtype == XOPS_F32;
  *out = nrm;
  return XOPS_OK;
}

extern "C" int xops_chunk_gated_delta_rule_gated_out_norm(
    const void* q, const void* k, const void* v, const float* A_log, const void* a, const void* b,
    const float* dt_bias, int a_dtype, int b_dtype, int64_t ab_token_stride, int ba_interleaved,
    float softplus_beta, float softplus_threshold,
    const float* h0, void* o, float* ht, const int32_t* cu_seqlens, int64_t B, int64_t T,
    int64_t N, int64_t Hg, int64_t H, int64_t K, int64_t V, int64_t q_token_stride,
    int64_t k_token_stride, int64_t v_token_stride, float scale, int use_qk_l2norm_in_kernel,
    const void* z, int64_t z_token_stride, int64_t z_heads_per_group, int64_t z_group_stride,
    const void* norm_weight, int weight_dtype, float eps, void* y, void* workspace,
    int64_t workspace_bytes, void* stream) {
  gdn::GateSrc gs{};
  if (int rc = gated_source(A_log, a, b, dt_bias, a_dtype, b_dtype, ab_token_stride,
                            ba_interleaved, softplus_beta, softplus_threshold, Hg, H, &gs))
    return rc;
  gdn::OutNorm nrm{};
  if (int rc = out_norm_args(z, z_token_stride, z_heads_per_group, z_group_stride, norm_weight,
                             weight_dtype, eps, y, N, T, H, V, &nrm))
    return rc;
  return chunk_gdn_run(q, k, v, gs, h0, o, ht, cu_seqlens, B, T, N, Hg, H, K, V, q_token_stride,
                       k_token_stride, v_token_stride, scale, use_qk_l2norm_in_kernel, workspace,
                       workspace_bytes, stream, &nrm);
}

extern "C" int xops_chunk_gated_delta_rule_out_norm(
    const void* q, const void* k, const void* v, const float* g, const float* beta,
    const float* h0, void* o, float* ht, const int32_t* cu_seqlens, int64_t B, int64_t T,
    int64_t N, int64_t Hg, int64_t H, int64_t K, int64_t V, int64_t q_token_stride,
    int64_t k_token_stride, int64_t v_token_stride, float scale, int use_qk_l2norm_in_kernel,
    const void* z, int64_t z_token_stride, const void* norm_weight, int weight_dtype, float eps,
    void* y, void* workspace, int64_t workspace_bytes, void* stream) {
  gdn::OutNorm nrm{};
  if (int rc = out_norm_args(z, z_token_stride, 1, V, norm_weight, weight_dtype, eps, y, N, T,
                             H, V, &nrm))
    return rc;
  gdn::GateSrc gs{};
  gs.g = g;
  gs.beta = beta;
  return chunk_gdn_run(q, k, v, gs, h0, o, ht, cu_seqlens, B, T, N, Hg, H, K, V, q_token_stride,
                       k_token_stride, v_token_stride, scale, use_qk_l2norm_in_kernel, workspace,
                       workspace_bytes, stream, &nrm);
}

extern "C" int xops_device_error_count(void) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, gdn::g_tc_error, sizeof(int)) != cudaSuccess) return -1;
  const int zero = 0;
  cudaMemcpyToSymbol(gdn::g_tc_error, &zero, sizeof(int));
  const int vn = xops::take_norm_error(), vc = xops::take_conv_error();
  const int vr = xops::take_rope_error(), vs = xops::take_subop_error();
  if (vn < 0 || vc < 0 || vr < 0 || vs < 0) return -1;
  return v + vn + vc + vr + vs;
}

// ---------------------------------------------------------------------------
// Chunked gated delta rule for callers that cannot allocate device memory
// when they run: some serving setups reserve every device byte up front, or
// run where the caching allocator is not available.  The computation is the
// one of xops_chunk_gated_delta_rule; only its scratch differs: instead of a
// caller workspace it uses one fixed array of this library's own device
// memory, kStaticScratchBytes long.  Problems whose workspace would exceed
// that size are rejected (XOPS_ERR_WORKSPACE) rather than partially served.
//
// The array's device address comes from cudaGetSymbolAddress, called with
// the caller's device current.  It is looked up again on every call made
// outside stream capture, so a new context on that device (after
// cudaDeviceReset, or a non-primary driver context, both of which load the
// module anew at another address) gets its own array.  A call made while its
// stream is capturing reuses the address found by the last uncaptured call on
// that device: make the first call on each device before any capture begins
// (a captured call with no earlier uncaptured one is rejected).  The array is
// shared by every call on a device, so two calls whose kernels may overlap on
// the GPU (for example on two streams without ordering between them) race on
// it; keep such calls ordered.  No scratch byte needs to start at zero: every
// byte the kernels read is written earlier in the same call.
//
// The array belongs to this file's device module: whenever that module is
// loaded on a device (on the first launch of any chunked-GDN kernel under
// lazy module loading, at context creation under eager loading) the device
// gives up kStaticScratchBytes for it until the process exits, whether or not
// this entry point is ever called.
// ---------------------------------------------------------------------------
namespace {
constexpr int64_t kStaticScratchBytes = 64ll << 20;  // 64 MiB
constexpr int kMaxDevices = 64;
static __device__ __align__(256) unsigned char g_static_scratch[kStaticScratchBytes];
std::mutex g_static_scratch_mu;
void* g_static_scratch_ptr[kMaxDevices] = {};

int static_scratch(cudaStream_t stream, void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess)
    return set_error(XOPS_ERR_CUDA, "chunk_gated_delta_rule_noalloc: cudaGetDevice: %s",
                     cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices)
    return set_error(XOPS_ERR_UNSUPPORTED, "chunk_gated_delta_rule_noalloc: device %d >= %d", dev,
                     kMaxDevices);
  cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
  e = cudaStreamIsCapturing(stream, &cs);
  if (e != cudaSuccess)
    return set_error(XOPS_ERR_CUDA, "chunk_gated_delta_rule_noalloc: cudaStreamIsCapturing: %s",
                     cudaGetErrorString(e));
  std::lock_guard<std::mutex> lock(g_static_scratch_mu);
  if (cs == cudaStreamCaptureStatusNone) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_static_scratch);
    if (e != cudaSuccess || !p)
      return set_error(XOPS_ERR_CUDA,
                       "chunk_gated_delta_rule_noalloc: cudaGetSymbolAddress of the scratch: %s",
                       cudaGetErrorString(e));
    g_static_scratch_ptr[dev] = p;
  } else if (!g_static_scratch_ptr[dev]) {
    return set_error(XOPS_ERR_INVALID_ARGUMENT,
                     "chunk_gated_delta_rule_noalloc: the first call on device %d was made during "
                     "stream capture; make one call outside capture first",
                     dev);
  }
  *out = g_static_scratch_ptr[dev];
  return XOPS_OK;
}
}  // namespace

extern "C" int xops_chunk_gated_delta_rule_noalloc(
    const void* q, const void* k, const void* v, const float* g, const float* beta,
    const float* h0, void* o, float* ht, const int32_t* cu_seqlens, int64_t B, int64_t T,
    int64_t N, int64_t Hg, int64_t H, int64_t K, int64_t V, int64_t q_token_stride,
    int64_t k_token_stride, int64_t v_token_stride, float scale, int use_qk_l2norm_in_kernel,
    void* stream) {
  const int64_t need = xops_chunk_gated_delta_rule_workspace_size(
      B, T, N, Hg, H, K, use_qk_l2norm_in_kernel, cu_seqlens != nullptr);
  if (need < 0)
    return set_error(XOPS_ERR_INVALID_ARGUMENT, "chunk_gated_delta_rule_noalloc: bad shape");
  if (need > kStaticScratchBytes)
    return set_error(XOPS_ERR_WORKSPACE,
                     "chunk_gated_delta_rule_noalloc: this problem needs %lld bytes of scratch but "
                     "the fixed scratch holds %lld; call xops_chunk_gated_delta_rule with a "
                     "workspace instead",
                     (long long)need, (long long)kStaticScratchBytes);
  void* ws = nullptr;
  if (int rc = static_scratch((cudaStream_t)stream, &ws)) return rc;
  return xops_chunk_gated_delta_rule(q, k, v, g, beta, h0, o, ht, cu_seqlens, B, T, N, Hg, H, K,
                                     V, q_token_stride, k_token_stride, v_token_stride, scale,
                                     use_qk_l2norm_in_kernel, ws, kStaticScratchBytes, stream);
}
