// Chunked gated delta rule prefill, fully fused: one CTA per (sequence,
// value head) walks the sequence's 64-token chunks in order and keeps the
// 128 x 128 fp32 state on chip for the whole sequence.  Nothing of the
// reference's decomposition -- g cumsum, A, (I+A)^-1, w, u, per-chunk h,
// v_new (npu_triton_chunk_gated_delta_rule.cpp:556-642 materialises all of
// them in HBM) -- ever leaves shared memory or registers; HBM sees q, k, v,
// g, beta and h0 once and o, ht once.
//
// Per chunk (gc = in-chunk cumsum of g, D_ij = e^{gc_i - gc_j} for i >= j):
//   A   = strict_tril(beta_i D_ij k_i.k_j)          Gram on tensor cores
//   T   = (I + A)^-1                                 blocked inverse, fp32
//   T'  = (T - I) diag(beta), T'' = T diag(beta e^{gc}) folded into bf16 operands
//   v'  = beta v + T' v - T'' k S                    (= u - w S)
//   o   = scale ((q e^{gc}) S + tril(q k^T D) v')
//   S  <- e^{gc_last} S + k^T (v' e^{gc_last - gc}) split into bf16 hi + lo
// Precision: beta is folded into the off-diagonal of T instead of into v, so v
// enters the tensor core exactly and the dominant beta_i v_i term of u stays
// fp32; the state update uses a two-term bf16 split of the scaled v' so the
// accumulated fp32 state tracks the fp32 recurrence to ~1e-5 relative (a
// bf16 beta on the diagonal, or a bf16 u, costs ~2e-3).
//
// Tensor-core work uses warp-level mma.sync m16n8k16 (bf16 in, fp32
// accumulate) with ldmatrix fragment loads from padded shared tiles.
#include "gdn_common.cuh"

namespace xops {
namespace gdn {
namespace {

constexpr int NTHREADS = 256;

struct __align__(16) FusedSmem {
  bf16 k[BT * LD128];
  bf16 q[BT * LD128];
  bf16 v[BT * LD128];
  bf16 h[128 * LD128];     // state (bf16) for this chunk's products, [K][V]
  union {
    float A[BT * LDF];     // strictly lower A (fp32)
    bf16 w[BT * LD128];    // -w = -(T'' k), [t][K]
  } u1;
  union {
    float M[32 * 33];      // inverse scratch
    bf16 vn[BT * LD128];   // v' (bf16) for the output product
  } u2;
  union {
    float T[BT * LDF];     // (I+A)^-1 (fp32)
    struct {
      bf16 hi[BT * LD128]; // v' e^{gl-gc}, high bf16 part
      bf16 lo[BT * LD128]; // and the residual
    } vt;
  } u3;
  bf16 tp[BT * LD64];      // T diag(beta)
  bf16 tpp[BT * LD64];     // T diag(beta e^gc)
  bf16 aqk[BT * LD64];     // tril(q k^T D)
  float graw[BT];
  float gc[BT];
  float beta[BT];
};

__global__ void __launch_bounds__(NTHREADS, 1) chunk_gdn_fused_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v,
    const float* __restrict__ g, const float* __restrict__ beta, const float* __restrict__ h0,
    bf16* __restrict__ o, float* __restrict__ ht, const int32_t* __restrict__ cu, int64_t T,
    int64_t Hg, int64_t H, int64_t q_stride, int64_t k_stride, int64_t v_stride, float scale,
    bool l2norm) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  FusedSmem& sm = *reinterpret_cast<FusedSmem*>(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int64_t n = blockIdx.x / H;
  const int h = (int)(blockIdx.x - n * H);
  const int hk = (int)(h / (H / Hg));
  int64_t bos, eos;
  seq_span(cu, n, T, bos, eos);
  constexpr int K = 128, V = 128;

  // state rows [16*warp, 16*warp+16) x all 128 columns, mma accumulator layout
  float S[16][4];
  {
    const float* src = h0 ? h0 + ((int64_t)n * H + h) * K * V : nullptr;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int r = 16 * warp + g8, c = 8 * j + 2 * t4;
      if (src) {
        const float2 a = *reinterpret_cast<const float2*>(src + r * V + c);
        const float2 b = *reinterpret_cast<const float2*>(src + (r + 8) * V + c);
        S[j][0] = a.x; S[j][1] = a.y; S[j][2] = b.x; S[j][3] = b.y;
      } else {
        S[j][0] = S[j][1] = S[j][2] = S[j][3] = 0.f;
      }
    }
  }

  const int64_t o_stride = H * V;
  for (int64_t t0 = bos; t0 < eos; t0 += BT) {
    const int L = (int)((eos - t0) < BT ? (eos - t0) : BT);
    // ---- stage inputs -------------------------------------------------------
    load_tile_64x128(sm.k, k + t0 * k_stride + (int64_t)hk * K, k_stride, L, tid, NTHREADS);
    load_tile_64x128(sm.q, q + t0 * q_stride + (int64_t)hk * K, q_stride, L, tid, NTHREADS);
    load_tile_64x128(sm.v, v + t0 * v_stride + (int64_t)h * V, v_stride, L, tid, NTHREADS);
    cp_async_commit();
    if (tid < BT) {
      sm.graw[tid] = tid < L ? g[(t0 + tid) * H + h] : 0.f;
      sm.beta[tid] = tid < L ? beta[(t0 + tid) * H + h] : 0.f;
    }
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int r = 16 * warp + g8, c = 8 * j + 2 * t4;
      *reinterpret_cast<uint32_t*>(&sm.h[r * LD128 + c]) = pack_bf16(S[j][0], S[j][1]);
      *reinterpret_cast<uint32_t*>(&sm.h[(r + 8) * LD128 + c]) = pack_bf16(S[j][2], S[j][3]);
    }
    cp_async_wait_all();
    __syncthreads();
    if (warp == 0) chunk_cumsum_warp(sm.graw, sm.gc, lane);
    if (l2norm) {
      // rows 0..63 of k (warps 0-3) and q (warps 4-7); 16 rows per warp
      bf16* base = warp < 4 ? sm.k : sm.q;
      for (int r = 16 * (warp & 3); r < 16 * (warp & 3) + 16; ++r) {
        __nv_bfloat162* row = reinterpret_cast<__nv_bfloat162*>(base + r * LD128);
        float2 a = __bfloat1622float2(row[lane]), b = __bfloat1622float2(row[lane + 32]);
        const float ss = warp_sum(a.x * a.x + a.y * a.y + b.x * b.x + b.y * b.y);
        const float rn = rsqrtf(ss + 1e-6f);
        row[lane] = __floats2bfloat162_rn(a.x * rn, a.y * rn);
        row[lane + 32] = __floats2bfloat162_rn(b.x * rn, b.y * rn);
      }
    }
    __syncthreads();
    const float gl = sm.gc[L - 1];

    // ---- Gram: [k; q] k^T ---------------------------------------------------
    {
      float G[8][4];
      zero_acc(G);
      const int m0 = 16 * (warp & 3);
      warp_gemm_a_bnk<8, 128>(G, warp < 4 ? sm.k : sm.q, LD128, m0, sm.k, LD128, 0, lane);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int i = m0 + g8 + ((e >> 1) << 3);
          const int c = 8 * j + 2 * t4 + (e & 1);
          const float d = __expf(fminf(sm.gc[i] - sm.gc[c], 0.f));
          if (warp < 4) {
            sm.u1.A[i * LDF + c] = (c < i) ? G[j][e] * sm.beta[i] * d : 0.f;
          } else {
            sm.aqk[i * LD64 + c] = __float2bfloat16_rn((c <= i) ? G[j][e] * d : 0.f);
          }
        }
      }
    }
    __syncthreads();

    // ---- (I + A)^-1 and the folded operands --------------------------------
    tri_inverse_64(sm.u1.A, sm.u3.T, sm.u2.M, tid);
    // T' holds only the strictly lower part of T diag(beta): the unit
    // diagonal's beta_i v_i term is added in fp32 below, so the dominant
    // term of u never goes through a bf16 rounding of beta.
    for (int e = tid; e < BT * BT; e += NTHREADS) {
      const int i = e >> 6, j = e & 63;
      const float tv = sm.u3.T[i * LDF + j] * sm.beta[j];
      sm.tp[i * LD64 + j] = __float2bfloat16_rn(i == j ? 0.f : tv);
      sm.tpp[i * LD64 + j] = __float2bfloat16_rn(tv * __expf(sm.gc[j]));
    }
    __syncthreads();

    // ---- u = T' v, w = T'' k, o_inter = q S --------------------------------
    const int mi = warp & 3, ni = warp >> 2;
    const int m0 = 16 * mi, n0 = 64 * ni;
    float U[8][4], O[8][4];
    {
      const float b0 = sm.beta[m0 + g8], b1 = sm.beta[m0 + g8 + 8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = m0 + g8, c = n0 + 8 * j + 2 * t4;
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.v[r * LD128 + c]));
        const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sm.v[(r + 8) * LD128 + c]));
        U[j][0] = b0 * a.x; U[j][1] = b0 * a.y; U[j][2] = b1 * b.x; U[j][3] = b1 * b.y;
      }
    }
    zero_acc(O);
    warp_gemm_a_bkn<8, 64>(U, sm.tp, LD64, m0, sm.v, LD128, n0, lane);
    {
      float W[8][4];
      zero_acc(W);
      warp_gemm_a_bkn<8, 64>(W, sm.tpp, LD64, m0, sm.k, LD128, n0, lane);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = m0 + g8, c = n0 + 8 * j + 2 * t4;
        *reinterpret_cast<uint32_t*>(&sm.u1.w[r * LD128 + c]) = pack_bf16(-W[j][0], -W[j][1]);
        *reinterpret_cast<uint32_t*>(&sm.u1.w[(r + 8) * LD128 + c]) = pack_bf16(-W[j][2], -W[j][3]);
      }
    }
    warp_gemm_a_bkn<8, 128>(O, sm.q, LD128, m0, sm.h, LD128, n0, lane);
    __syncthreads();

    // ---- v' = u - w S ; split the scaled v' for the state update -------------
    warp_gemm_a_bkn<8, 128>(U, sm.u1.w, LD128, m0, sm.h, LD128, n0, lane);
    {
      const float eg0 = __expf(sm.gc[m0 + g8]), eg1 = __expf(sm.gc[m0 + g8 + 8]);
      const float fd0 = __expf(fminf(gl - sm.gc[m0 + g8], 0.f));
      const float fd1 = __expf(fminf(gl - sm.gc[m0 + g8 + 8], 0.f));
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = m0 + g8, c = n0 + 8 * j + 2 * t4;
        O[j][0] *= eg0; O[j][1] *= eg0; O[j][2] *= eg1; O[j][3] *= eg1;
        *reinterpret_cast<uint32_t*>(&sm.u2.vn[r * LD128 + c]) = pack_bf16(U[j][0], U[j][1]);
        *reinterpret_cast<uint32_t*>(&sm.u2.vn[(r + 8) * LD128 + c]) = pack_bf16(U[j][2], U[j][3]);
        float s0 = U[j][0] * fd0, s1 = U[j][1] * fd0, s2 = U[j][2] * fd1, s3 = U[j][3] * fd1;
        const __nv_bfloat162 h01 = __floats2bfloat162_rn(s0, s1);
        const __nv_bfloat162 h23 = __floats2bfloat162_rn(s2, s3);
        const float2 f01 = __bfloat1622float2(h01), f23 = __bfloat1622float2(h23);
        *reinterpret_cast<__nv_bfloat162*>(&sm.u3.vt.hi[r * LD128 + c]) = h01;
        *reinterpret_cast<__nv_bfloat162*>(&sm.u3.vt.hi[(r + 8) * LD128 + c]) = h23;
        *reinterpret_cast<uint32_t*>(&sm.u3.vt.lo[r * LD128 + c]) = pack_bf16(s0 - f01.x, s1 - f01.y);
        *reinterpret_cast<uint32_t*>(&sm.u3.vt.lo[(r + 8) * LD128 + c]) = pack_bf16(s2 - f23.x, s3 - f23.y);
      }
    }
    __syncthreads();

    // ---- o = scale (o_inter + Aqk v') ---------------------------------------
    warp_gemm_a_bkn<8, 64>(O, sm.aqk, LD64, m0, sm.u2.vn, LD128, n0, lane);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = m0 + g8, c = n0 + 8 * j + 2 * t4;
      if (r < L)
        *reinterpret_cast<uint32_t*>(o + (t0 + r) * o_stride + (int64_t)h * V + c) =
            pack_bf16(O[j][0] * scale, O[j][1] * scale);
      if (r + 8 < L)
        *reinterpret_cast<uint32_t*>(o + (t0 + r + 8) * o_stride + (int64_t)h * V + c) =
            pack_bf16(O[j][2] * scale, O[j][3] * scale);
    }

    // ---- S <- e^{gl} S + k^T (vt_hi + vt_lo) ---------------------------------
    {
      const float dl = __expf(gl);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        S[j][0] *= dl; S[j][1] *= dl; S[j][2] *= dl; S[j][3] *= dl;
      }
      warp_gemm_at_bkn<16, 64>(S, sm.k, LD128, 16 * warp, sm.u3.vt.hi, LD128, 0, lane);
      warp_gemm_at_bkn<16, 64>(S, sm.k, LD128, 16 * warp, sm.u3.vt.lo, LD128, 0, lane);
    }
    __syncthreads();
  }

  if (ht) {
    float* dst = ht + ((int64_t)n * H + h) * K * V;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int r = 16 * warp + g8, c = 8 * j + 2 * t4;
      *reinterpret_cast<float2*>(dst + r * V + c) = make_float2(S[j][0], S[j][1]);
      *reinterpret_cast<float2*>(dst + (r + 8) * V + c) = make_float2(S[j][2], S[j][3]);
    }
  }
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
  XOPS_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(o) &&
                   (!h0 || aligned16(h0)) && (!ht || aligned16(ht)),
               "chunk_gated_delta_rule: tensors must be 16-byte aligned");
  const size_t smem = sizeof(gdn::FusedSmem);
  if (int rc = gdn::ensure_smem_attr((const void*)gdn::chunk_gdn_fused_kernel, smem,
                                     "chunk_gated_delta_rule"))
    return rc;
  cudaStream_t st = (cudaStream_t)stream;
  gdn::chunk_gdn_fused_kernel<<<(unsigned)(N * H), gdn::NTHREADS, smem, st>>>(
      (const gdn::bf16*)q, (const gdn::bf16*)k, (const gdn::bf16*)v, g, beta, h0, (gdn::bf16*)o,
      ht, cu_seqlens, T, Hg, H, q_token_stride, k_token_stride, v_token_stride, scale,
      use_qk_l2norm_in_kernel != 0);
  return check_launch("chunk_gated_delta_rule");
}
