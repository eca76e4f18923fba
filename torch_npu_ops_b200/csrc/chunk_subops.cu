// The reference's chunk pipeline as separate operators (drop-in for callers
// that run the stages themselves): chunk_local_cumsum, chunk_scaled_dot_kkt,
// solve_tril, recompute_w_u, chunk_gated_delta_rule_fwd_h and chunk_fwd_o
// (triton_npu/torch_api/npu_triton_chunk_gated_delta_rule.cpp:151-802).
// Each follows the layouts of the reference's Triton kernels
// (triton_npu/triton_src/chunk_gated_delta_rule/*.py) and computes in fp32
// with bf16 tensor-core operands.  The fused xops_chunk_gated_delta_rule is
// the production path; these exist so every stage can also be called alone.
//
// Varlen chunk addressing is derived on the device from cu_seqlens (no host
// copy of the offsets, unlike prepare_chunk_indices_like_python at :38-75):
// chunk-parallel kernels launch an upper bound of T/64 + N chunk slots and
// the CTAs past the last chunk exit.
#include "gdn_common.cuh"

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
__global__ void __launch_bounds__(128) kkt_kernel(const bf16* __restrict__ k,
                                                  const float* __restrict__ beta,
                                                  const float* __restrict__ gc,
                                                  float* __restrict__ A,
                                                  const int32_t* __restrict__ cu, int64_t N,
                                                  int64_t T, int64_t Hg, int64_t H) {
  __shared__ __align__(16) bf16 sk[BT * LD128];
  __shared__ float sg[BT], sb[BT];
  const ChunkPos p = resolve_chunk(cu, N, T);
  if (!p.valid) return;
  const int h = blockIdx.y, hk = (int)(h / (H / Hg));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  load_tile_64x128(sk, k + p.t0 * Hg * 128 + (int64_t)hk * 128, Hg * 128, p.L, tid, 128);
  cp_async_commit();
  if (tid < BT) {
    sg[tid] = (gc && tid < p.L) ? gc[(p.t0 + tid) * H + h] : 0.f;
    sb[tid] = tid < p.L ? beta[(p.t0 + tid) * H + h] : 0.f;
  }
  cp_async_wait_all();
  __syncthreads();
  float G[8][4];
  zero_acc(G);
  const int m0 = 16 * warp;
  warp_gemm_a_bnk<8, 128>(G, sk, LD128, m0, sk, LD128, 0, lane);
  const int g8 = lane >> 2, t4 = lane & 3;
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = m0 + g8 + ((e >> 1) << 3), c = 8 * j + 2 * t4 + (e & 1);
      if (i < p.L) {
        const float d = __expf(fminf(sg[i] - sg[c], 0.f));
        A[((p.t0 + i) * H + h) * BT + c] = (c < i) ? G[j][e] * sb[i] * d : 0.f;
      }
    }
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
template <typename TA>
__global__ void __launch_bounds__(256) recompute_wu_kernel(
    const bf16* __restrict__ k, const bf16* __restrict__ v, const float* __restrict__ beta,
    const float* __restrict__ gc, const TA* __restrict__ Ai, bf16* __restrict__ w,
    bf16* __restrict__ u, const int32_t* __restrict__ cu, int64_t N, int64_t T, int64_t Hg,
    int64_t H) {
  extern __shared__ __align__(16) unsigned char raw[];
  bf16* sk = reinterpret_cast<bf16*>(raw);
  bf16* sv = sk + BT * LD128;
  bf16* tp = sv + BT * LD128;
  bf16* tpp = tp + BT * LD64;
  const ChunkPos p = resolve_chunk(cu, N, T);
  if (!p.valid) return;
  const int h = blockIdx.y, hk = (int)(h / (H / Hg));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  load_tile_64x128(sk, k + p.t0 * Hg * 128 + (int64_t)hk * 128, Hg * 128, p.L, tid, 256);
  load_tile_64x128(sv, v + p.t0 * H * 128 + (int64_t)h * 128, H * 128, p.L, tid, 256);
  cp_async_commit();
  for (int e = tid; e < BT * BT; e += 256) {
    const int i = e >> 6, j = e & 63;
    float tv = 0.f, eg = 0.f;
    if (i < p.L && j < p.L) {
      tv = to_f32<TA>(Ai[((p.t0 + i) * H + h) * BT + j]) * beta[(p.t0 + j) * H + h];
      eg = __expf(gc[(p.t0 + j) * H + h]);
    }
    tp[i * LD64 + j] = __float2bfloat16_rn(i == j ? 0.f : tv);  // diagonal added in fp32
    tpp[i * LD64 + j] = __float2bfloat16_rn(tv * eg);
  }
  cp_async_wait_all();
  __syncthreads();
  const int m0 = 16 * (warp & 3), n0 = 64 * (warp >> 2);
  const int g8 = lane >> 2, t4 = lane & 3;
  float U[8][4], W[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) {  // u starts from Ai_ii * beta_i * v_i in fp32
    const int r = m0 + g8, c = n0 + 8 * j + 2 * t4;
    const float d0 = r < p.L ? to_f32<TA>(Ai[((p.t0 + r) * H + h) * BT + r]) * beta[(p.t0 + r) * H + h] : 0.f;
    const float d1 = r + 8 < p.L ? to_f32<TA>(Ai[((p.t0 + r + 8) * H + h) * BT + r + 8]) * beta[(p.t0 + r + 8) * H + h] : 0.f;
    const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sv[r * LD128 + c]));
    const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&sv[(r + 8) * LD128 + c]));
    U[j][0] = d0 * a.x; U[j][1] = d0 * a.y; U[j][2] = d1 * b.x; U[j][3] = d1 * b.y;
  }
  zero_acc(W);
  warp_gemm_a_bkn<8, 64>(U, tp, LD64, m0, sv, LD128, n0, lane);
  warp_gemm_a_bkn<8, 64>(W, tpp, LD64, m0, sk, LD128, n0, lane);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int r = m0 + g8, c = n0 + 8 * j + 2 * t4;
    if (r < p.L) {
      *reinterpret_cast<uint32_t*>(u + ((p.t0 + r) * H + h) * 128 + c) = pack_bf16(U[j][0], U[j][1]);
      *reinterpret_cast<uint32_t*>(w + ((p.t0 + r) * H + h) * 128 + c) = pack_bf16(W[j][0], W[j][1]);
    }
    if (r + 8 < p.L) {
      *reinterpret_cast<uint32_t*>(u + ((p.t0 + r + 8) * H + h) * 128 + c) = pack_bf16(U[j][2], U[j][3]);
      *reinterpret_cast<uint32_t*>(w + ((p.t0 + r + 8) * H + h) * 128 + c) = pack_bf16(W[j][2], W[j][3]);
    }
  }
}

// ---- chunk_gated_delta_rule_fwd_h (chunk_delta_h.py:30-199) ------------------
__global__ void __launch_bounds__(256, 1) fwd_h_kernel(
    const bf16* __restrict__ k, const bf16* __restrict__ w, const bf16* __restrict__ u,
    const float* __restrict__ gc, const float* __restrict__ h0, bf16* __restrict__ hout,
    bf16* __restrict__ vnew, float* __restrict__ ht, const int32_t* __restrict__ cu, int64_t N,
    int64_t T, int64_t Hg, int64_t H) {
  extern __shared__ __align__(16) unsigned char raw[];
  bf16* sk = reinterpret_cast<bf16*>(raw);
  bf16* sw = sk + BT * LD128;
  bf16* su = sw + BT * LD128;
  bf16* sh = su + BT * LD128;           // 128 rows
  bf16* vhi = sh + 128 * LD128;
  bf16* vlo = vhi + BT * LD128;
  float* sg = reinterpret_cast<float*>(vlo + BT * LD128);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int64_t n = blockIdx.x / H;
  const int h = (int)(blockIdx.x - n * H), hk = (int)(h / (H / Hg));
  int64_t bos, eos;
  seq_span(cu, n, T, bos, eos);
  const int64_t boh = chunk_offset(cu, n, T);
  float S[16][4];
  const float* src = h0 ? h0 + ((int64_t)n * H + h) * 128 * 128 : nullptr;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int r = 16 * warp + g8, c = 8 * j + 2 * t4;
    S[j][0] = src ? src[r * 128 + c] : 0.f;
    S[j][1] = src ? src[r * 128 + c + 1] : 0.f;
    S[j][2] = src ? src[(r + 8) * 128 + c] : 0.f;
    S[j][3] = src ? src[(r + 8) * 128 + c + 1] : 0.f;
  }
  int64_t ci = 0;
  for (int64_t t0 = bos; t0 < eos; t0 += BT, ++ci) {
    const int L = (int)((eos - t0) < BT ? (eos - t0) : BT);
    load_tile_64x128(sk, k + t0 * Hg * 128 + (int64_t)hk * 128, Hg * 128, L, tid, 256);
    load_tile_64x128(sw, w + t0 * H * 128 + (int64_t)h * 128, H * 128, L, tid, 256);
    load_tile_64x128(su, u + t0 * H * 128 + (int64_t)h * 128, H * 128, L, tid, 256);
    cp_async_commit();
    if (tid < BT) sg[tid] = (gc && tid < L) ? gc[(t0 + tid) * H + h] : 0.f;
    bf16* hdst = hout + ((boh + ci) * H + h) * 128 * 128;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int r = 16 * warp + g8, c = 8 * j + 2 * t4;
      const uint32_t a = pack_bf16(S[j][0], S[j][1]), b = pack_bf16(S[j][2], S[j][3]);
      *reinterpret_cast<uint32_t*>(&sh[r * LD128 + c]) = a;
      *reinterpret_cast<uint32_t*>(&sh[(r + 8) * LD128 + c]) = b;
      *reinterpret_cast<uint32_t*>(hdst + r * 128 + c) = a;
      *reinterpret_cast<uint32_t*>(hdst + (r + 8) * 128 + c) = b;
    }
    cp_async_wait_all();
    __syncthreads();
    // pad rows of g with the chunk's last value (cumsum of zeros)
    const float gl = sg[L - 1];
    const int m0 = 16 * (warp & 3), n0 = 64 * (warp >> 2);
    // v' = u - w h   (start from u, accumulate -w h with negated w)
    float U[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = m0 + g8, c = n0 + 8 * j + 2 * t4;
      const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&su[r * LD128 + c]));
      const float2 b = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&su[(r + 8) * LD128 + c]));
      U[j][0] = a.x; U[j][1] = a.y; U[j][2] = b.x; U[j][3] = b.y;
    }
    // negate w in place (each element owned by exactly one thread)
    for (int e = tid; e < BT * 64; e += 256) {
      const int r = e >> 6, c2 = (e & 63) << 1;
      __nv_bfloat162* pw = reinterpret_cast<__nv_bfloat162*>(&sw[r * LD128 + c2]);
      *pw = __hneg2(*pw);
    }
    __syncthreads();
    warp_gemm_a_bkn<8, 128>(U, sw, LD128, m0, sh, LD128, n0, lane);
    const bool gated = gc != nullptr;
    const float f0 = gated ? __expf(fminf(gl - sg[m0 + g8], 0.f)) : 1.f;
    const float f1 = gated ? __expf(fminf(gl - sg[m0 + g8 + 8], 0.f)) : 1.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = m0 + g8, c = n0 + 8 * j + 2 * t4;
      if (vnew) {
        if (r < L) *reinterpret_cast<uint32_t*>(vnew + ((t0 + r) * H + h) * 128 + c) = pack_bf16(U[j][0], U[j][1]);
        if (r + 8 < L) *reinterpret_cast<uint32_t*>(vnew + ((t0 + r + 8) * H + h) * 128 + c) = pack_bf16(U[j][2], U[j][3]);
      }
      const float s0 = U[j][0] * f0, s1 = U[j][1] * f0, s2 = U[j][2] * f1, s3 = U[j][3] * f1;
      const __nv_bfloat162 h01 = __floats2bfloat162_rn(s0, s1), h23 = __floats2bfloat162_rn(s2, s3);
      const float2 a = __bfloat1622float2(h01), b = __bfloat1622float2(h23);
      *reinterpret_cast<__nv_bfloat162*>(&vhi[r * LD128 + c]) = h01;
      *reinterpret_cast<__nv_bfloat162*>(&vhi[(r + 8) * LD128 + c]) = h23;
      *reinterpret_cast<uint32_t*>(&vlo[r * LD128 + c]) = pack_bf16(s0 - a.x, s1 - a.y);
      *reinterpret_cast<uint32_t*>(&vlo[(r + 8) * LD128 + c]) = pack_bf16(s2 - b.x, s3 - b.y);
    }
    __syncthreads();
    const float dl = gated ? __expf(gl) : 1.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      S[j][0] *= dl; S[j][1] *= dl; S[j][2] *= dl; S[j][3] *= dl;
    }
    warp_gemm_at_bkn<16, 64>(S, sk, LD128, 16 * warp, vhi, LD128, 0, lane);
    warp_gemm_at_bkn<16, 64>(S, sk, LD128, 16 * warp, vlo, LD128, 0, lane);
    __syncthreads();
  }
  if (ht) {
    float* dst = ht + ((int64_t)n * H + h) * 128 * 128;
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int r = 16 * warp + g8, c = 8 * j + 2 * t4;
      *reinterpret_cast<float2*>(dst + r * 128 + c) = make_float2(S[j][0], S[j][1]);
      *reinterpret_cast<float2*>(dst + (r + 8) * 128 + c) = make_float2(S[j][2], S[j][3]);
    }
  }
}

// ---- chunk_fwd_o (chunk_o.py:26-116) -----------------------------------------
__global__ void __launch_bounds__(256) fwd_o_kernel(
    const bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ vnew,
    const bf16* __restrict__ hs, const float* __restrict__ gc, bf16* __restrict__ o,
    const int32_t* __restrict__ cu, int64_t N, int64_t T, int64_t Hg, int64_t H, float scale) {
  extern __shared__ __align__(16) unsigned char raw[];
  bf16* sq = reinterpret_cast<bf16*>(raw);
  bf16* sk = sq + BT * LD128;
  bf16* sv = sk + BT * LD128;
  bf16* sh = sv + BT * LD128;  // 128 rows
  bf16* aqk = sh + 128 * LD128;
  float* sg = reinterpret_cast<float*>(aqk + BT * LD64);
  const ChunkPos p = resolve_chunk(cu, N, T);
  if (!p.valid) return;
  const int h = blockIdx.y, hk = (int)(h / (H / Hg));
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g8 = lane >> 2, t4 = lane & 3;
  const int64_t gidx = chunk_offset(cu, p.seq, T) + p.cis;
  load_tile_64x128(sq, q + p.t0 * Hg * 128 + (int64_t)hk * 128, Hg * 128, p.L, tid, 256);
  load_tile_64x128(sk, k + p.t0 * Hg * 128 + (int64_t)hk * 128, Hg * 128, p.L, tid, 256);
  load_tile_64x128(sv, vnew + p.t0 * H * 128 + (int64_t)h * 128, H * 128, p.L, tid, 256);
  const bf16* hsrc = hs + (gidx * H + h) * 128 * 128;
  for (int e = tid; e < 128 * 16; e += 256) {
    const int r = e >> 4, c = (e & 15) << 3;
    cp_async16(sh + r * LD128 + c, hsrc + r * 128 + c, 16);
  }
  cp_async_commit();
  if (tid < BT) sg[tid] = (gc && tid < p.L) ? gc[(p.t0 + tid) * H + h] : 0.f;
  cp_async_wait_all();
  __syncthreads();
  if (warp < 4) {
    float G[8][4];
    zero_acc(G);
    const int m0 = 16 * warp;
    warp_gemm_a_bnk<8, 128>(G, sq, LD128, m0, sk, LD128, 0, lane);
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = m0 + g8 + ((e >> 1) << 3), c = 8 * j + 2 * t4 + (e & 1);
        const float d = gc ? __expf(fminf(sg[i] - sg[c], 0.f)) : 1.f;
        aqk[i * LD64 + c] = __float2bfloat16_rn(c <= i ? G[j][e] * d : 0.f);
      }
  }
  const int m0 = 16 * (warp & 3), n0 = 64 * (warp >> 2);
  float O[8][4];
  zero_acc(O);
  warp_gemm_a_bkn<8, 128>(O, sq, LD128, m0, sh, LD128, n0, lane);
  const float e0 = gc ? __expf(sg[m0 + g8]) : 1.f, e1 = gc ? __expf(sg[m0 + g8 + 8]) : 1.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    O[j][0] *= e0; O[j][1] *= e0; O[j][2] *= e1; O[j][3] *= e1;
  }
  __syncthreads();
  warp_gemm_a_bkn<8, 64>(O, aqk, LD64, m0, sv, LD128, n0, lane);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int r = m0 + g8, c = n0 + 8 * j + 2 * t4;
    if (r < p.L)
      *reinterpret_cast<uint32_t*>(o + ((p.t0 + r) * H + h) * 128 + c) = pack_bf16(O[j][0] * scale, O[j][1] * scale);
    if (r + 8 < p.L)
      *reinterpret_cast<uint32_t*>(o + ((p.t0 + r + 8) * H + h) * 128 + c) = pack_bf16(O[j][2] * scale, O[j][3] * scale);
  }
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
  if (N == 0 || T == 0) return XOPS_OK;
  XOPS_REQUIRE(k && beta && A && aligned16(k), "chunk_scaled_dot_kkt_fwd: bad pointer");
  dim3 grid(chunk_slots(cu_seqlens, B, T, N), (unsigned)H);
  kkt_kernel<<<grid, 128, 0, (cudaStream_t)stream>>>((const bf16*)k, beta, g_cumsum, A,
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
  const size_t smem = 2 * BT * LD128 * sizeof(bf16) + 2 * BT * LD64 * sizeof(bf16);
  dim3 grid(chunk_slots(cu_seqlens, B, T, N), (unsigned)H);
  cudaStream_t st = (cudaStream_t)stream;
#define XOPS_WU(TA)                                                                                \
  {                                                                                                \
    if (int rc = ensure_smem_attr((const void*)recompute_wu_kernel<TA>, smem, "recompute_w_u_fwd")) \
      return rc;                                                                                   \
    recompute_wu_kernel<TA><<<grid, 256, smem, st>>>((const bf16*)k, (const bf16*)v, beta,         \
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
  const size_t smem = (5 * BT + 128) * LD128 * sizeof(bf16) + BT * sizeof(float);
  if (int rc = ensure_smem_attr((const void*)fwd_h_kernel, smem, "chunk_gated_delta_rule_fwd_h"))
    return rc;
  fwd_h_kernel<<<(unsigned)(N * H), 256, smem, (cudaStream_t)stream>>>(
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
  const size_t smem = (3 * BT + 128) * LD128 * sizeof(bf16) + BT * LD64 * sizeof(bf16) + BT * sizeof(float);
  if (int rc = ensure_smem_attr((const void*)fwd_o_kernel, smem, "chunk_fwd_o")) return rc;
  dim3 grid(chunk_slots(cu_seqlens, B, T, N), (unsigned)H);
  fwd_o_kernel<<<grid, 256, smem, (cudaStream_t)stream>>>(
      (const bf16*)q, (const bf16*)k, (const bf16*)v_new, (const bf16*)h, g_cumsum, (bf16*)o,
      cu_seqlens, N, T, Hg, H, scale);
  return check_launch("chunk_fwd_o");
}
