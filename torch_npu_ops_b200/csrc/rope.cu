// Fused q/k RMSNorm + NeoX RoPE (full or partial rotary) + v copy.
//
// Semantics follow split_rmsnorm_rope_kernel
// (triton_npu/triton_src/test_split_rmsnorm_rope.py:63-221): split the packed
// row into q | k | v, RMS-normalise every q and k head with the shared
// weight (and bias), rotate with x*cos + rotate_half(x)*sin, copy v.  The
// rotation here covers the first rotary_dim dims of each head (the reference
// kernel only handles rotary_dim == head_dim); the rest pass through.
//
// HBM-bound: every input element is read once and written once.  One warp
// per (token, head); a lane owns head_dim/32 contiguous elements (16-byte
// vectors for head_dim 256 in fp32/bf16), the RMS statistic is a warp
// shuffle reduction and the rotate-half partner comes from a per-warp
// shared-memory row, so any even rotary_dim works.
#include "common.cuh"
#include "tcgen05.cuh"

namespace xops {
namespace {

template <typename T, typename TW, typename TS, int EPL>
__global__ void __launch_bounds__(256) split_rmsnorm_rope_kernel(
    const T* __restrict__ in, const TS* __restrict__ sin_t, const TS* __restrict__ cos_t,
    T* __restrict__ qo, T* __restrict__ ko, T* __restrict__ vo, const TW* __restrict__ qw,
    const TW* __restrict__ qb, const TW* __restrict__ kw, const TW* __restrict__ kb,
    int64_t T_, int qh, int kvh, int rd, float eps) {
  constexpr int HD = EPL * 32;
  __shared__ float rowbuf[8][HD];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int heads = qh + 2 * kvh;
  const int64_t item = (int64_t)blockIdx.x * 8 + warp;
  if (item >= T_ * heads) return;
  const int64_t t = item / heads;
  const int hh = (int)(item - t * heads);
  const int64_t total = (int64_t)heads * HD;
  const T* src = in + t * total + (int64_t)hh * HD + lane * EPL;
  float v[EPL];
  load_vec<T, EPL>(src, v);
  if (hh >= qh + kvh) {  // v head: plain copy
    store_vec<T, EPL>(vo + t * (int64_t)kvh * HD + (int64_t)(hh - qh - kvh) * HD + lane * EPL, v);
    return;
  }
  const bool is_q = hh < qh;
  const TW* w = is_q ? qw : kw;
  const TW* b = is_q ? qb : kb;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < EPL; ++i) ss += v[i] * v[i];
  const float r = 1.0f / sqrtf(warp_sum(ss) * (1.0f / HD) + eps);
  float wv[EPL];
  load_vec<TW, EPL>(w + lane * EPL, wv);
  if (b != nullptr) {
    float bv[EPL];
    load_vec<TW, EPL>(b + lane * EPL, bv);
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = v[i] * r * wv[i] + bv[i];
  } else {
#pragma unroll
    for (int i = 0; i < EPL; ++i) v[i] = v[i] * r * wv[i];
  }
#pragma unroll
  for (int i = 0; i < EPL; ++i) rowbuf[warp][lane * EPL + i] = v[i];
  __syncwarp();
  const int half = rd >> 1;
#pragma unroll
  for (int i = 0; i < EPL; ++i) {
    const int d = lane * EPL + i;
    if (d < rd) {
      const float c = to_f32<TS>(cos_t[t * rd + d]);
      const float s = to_f32<TS>(sin_t[t * rd + d]);
      const float partner = d < half ? -rowbuf[warp][d + half] : rowbuf[warp][d - half];
      v[i] = v[i] * c + partner * s;
    }
  }
  T* dst = is_q ? qo + t * (int64_t)qh * HD + (int64_t)hh * HD
                : ko + t * (int64_t)kvh * HD + (int64_t)(hh - qh) * HD;
  store_vec<T, EPL>(dst + lane * EPL, v);
}

// ----------------------------------------------------------------------------
// Streaming path for large token counts.  The packed input [T, heads * HD] is
// a flat list of T * heads head segments of HD elements; a persistent CTA
// streams tiles of whole segments (32 KB) into a ring of RP_NS shared stages
// with 1-D bulk copies (warp 0), together with the cos / sin rows of the
// tokens the tile touches (when those rows are 16-byte multiples), and 8
// consumer warps take two segments at a time: v heads are copied out, q / k
// heads are normalised and rotated.  A lane owns interleaved 16-byte chunks
// of a segment (chunk c of lane l holds elements (32 c + l) V .. + V - 1, V
// elements per 16 bytes), so every shared-memory read of the segment, of the
// weight rows and every global store of a warp is one contiguous, bank- and
// sector-aligned 512-byte access.  The rotate-half partner of element d is
// element d +- rotary_dim / 2: (mode 1) in chunk 0 of lane +- half / V, a
// shuffle, when every rotated element is in chunk 0 and half is a whole
// number of chunks; (mode 2) in the same lane's chunk c +- half / (32 V)
// when half is a whole number of chunk rows; (mode 0) otherwise recomputed
// from the raw input of the partner in the stage (same r, weight and bias).
// Weight and bias rows live in shared memory for the whole kernel.
// ----------------------------------------------------------------------------
constexpr int RP_NS = 3, RP_TILE = 32768, RP_NT = 32 + 256;
constexpr uint32_t RP_WAIT = 1u << 26;
__device__ int g_rope_error = 0;

struct RopeStage {
  int stage;    // bytes per ring stage: x tile, then cos rows, then sin rows
  int cs;       // bytes reserved for each table's rows in a stage (0: read global)
  int maxtok;   // tokens one tile can touch
};

template <typename T, typename TW, typename TS, int HD, int MODE>
__global__ void __launch_bounds__(RP_NT, 2) split_rmsnorm_rope_stream_kernel(
    const T* __restrict__ in, const TS* __restrict__ sin_t, const TS* __restrict__ cos_t,
    T* __restrict__ qo, T* __restrict__ ko, T* __restrict__ vo, const TW* __restrict__ qw,
    const TW* __restrict__ qb, const TW* __restrict__ kw, const TW* __restrict__ kb,
    int64_t T_, int qh, int kvh, int rd, RopeStage L, float eps) {
  constexpr int EPL = HD / 32;                // elements per lane
  constexpr int SEG = HD * (int)sizeof(T);    // bytes per head segment
  constexpr int SPT = RP_TILE / SEG;          // segments per tile
  static_assert(SPT % 8 == 0, "a tile must give every consumer warp the same count");
  static_assert(EPL % 4 == 0 && EPL * sizeof(T) % 16 == 0, "lane slice must be whole vectors");
  extern __shared__ unsigned char rp_raw[];
  unsigned char* sm = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(rp_raw) + 127) & ~static_cast<uintptr_t>(127));
  float* swt = reinterpret_cast<float*>(sm + RP_NS * L.stage);  // qw | qb | kw | kb as fp32
  __shared__ uint64_t full[RP_NS], empty[RP_NS];
  __shared__ int abort_sh;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int heads = qh + 2 * kvh;
  const int64_t total = T_ * heads;
  const int64_t tiles = (total + SPT - 1) / SPT;
  const bool has_b = qb != nullptr;
  const bool staged = L.cs > 0;
  if (tid == 0) {
    for (int s = 0; s < RP_NS; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 8);
    }
    tc::mbar_fence_init();
    abort_sh = 0;
  }
  constexpr int V = 16 / (int)sizeof(T);  // elements per 16-byte chunk
  constexpr int HV = V / 2;                // element pairs per chunk
  // weight rows in float4 units ordered [chunk][quarter of chunk][lane], so
  // that the float4 of pairs (j, j + 1) of every lane is one conflict-free read
  auto widx = [](int d) {
    const int m = d / V, e = d % V;
    return (((m >> 5) * (V / 4) + e / 4) * 32 + (m & 31)) * 4 + (e & 3);
  };
  for (int i = tid; i < HD; i += blockDim.x) {
    const int w = widx(i);
    swt[w] = to_f32<TW>(qw[i]);
    swt[2 * HD + w] = to_f32<TW>(kw[i]);
    swt[HD + w] = has_b ? to_f32<TW>(qb[i]) : 0.f;
    swt[3 * HD + w] = has_b ? to_f32<TW>(kb[i]) : 0.f;
  }
  __syncthreads();
  if (warp == 0) {
    if (lane == 0) {
      for (int64_t k = 0;; ++k) {
        const int64_t t = blockIdx.x + k * gridDim.x;
        if (t >= tiles) break;
        const int s = (int)(k % RP_NS);
        if (k >= RP_NS && !tc::mbar_wait(&empty[s], (uint32_t)((k / RP_NS - 1) & 1), RP_WAIT)) {
          atomicExch(&g_rope_error, 1);
          atomicExch(&abort_sh, 1);
          break;
        }
        if (*(volatile int*)&abort_sh) break;
        const int64_t s0 = t * SPT;
        const int64_t n = total - s0 < SPT ? total - s0 : SPT;
        unsigned char* st = sm + s * L.stage;
        uint32_t cb = 0;
        int64_t tf = 0;
        if (staged) {
          tf = s0 / heads;
          cb = (uint32_t)(((s0 + n - 1) / heads - tf + 1) * rd * (int64_t)sizeof(TS));
        }
        tc::mbar_arrive_expect_tx(&full[s], (uint32_t)(n * SEG) + 2 * cb);
        tc::bulk_load(st, in + s0 * HD, (uint32_t)(n * SEG), &full[s]);
        if (staged) {
          tc::bulk_load(st + RP_TILE, cos_t + tf * rd, cb, &full[s]);
          tc::bulk_load(st + RP_TILE + L.cs, sin_t + tf * rd, cb, &full[s]);
        }
      }
    }
    return;
  }
  const int cw = warp - 1;
  const int half = rd >> 1;
  constexpr int NC = EPL / V;  // chunks per lane
  // MODE (the partner rule, chosen at launch by rope_partner_mode):
  // 1: partner lane of chunk 0; 2: partner chunk distance; 0: recompute
  const int db0 = lane * V;
  const int src = MODE != 1 ? lane : db0 < half ? lane + half / V : db0 < rd ? lane - half / V : lane;
  const int coff = MODE == 2 ? half / (32 * V) : 0;
  constexpr int NSEG = EPL <= 8 ? 2 : 1;  // segments in flight per warp
  constexpr int P = EPL / 2;              // element pairs per lane
  for (int64_t k = 0;; ++k) {
    const int64_t t = blockIdx.x + k * gridDim.x;
    if (t >= tiles) break;
    const int s = (int)(k % RP_NS);
    if (!tc::mbar_wait(&full[s], (uint32_t)((k / RP_NS) & 1), RP_WAIT)) {
      atomicExch(&g_rope_error, 1);
      break;
    }
    const unsigned char* stb = sm + s * L.stage;
    const T* st = reinterpret_cast<const T*>(stb);
    const TS* scos = reinterpret_cast<const TS*>(stb + RP_TILE);
    const TS* ssin = reinterpret_cast<const TS*>(stb + RP_TILE + L.cs);
    const int64_t s0 = t * SPT;
    const int64_t tf = s0 / heads;          // first token of the tile
    const int h0 = (int)(s0 - tf * heads);  // its head
#pragma unroll 1
    for (int i0 = cw; i0 < SPT; i0 += 8 * NSEG) {
      // element pairs of the lane's chunks as packed fp32 pairs: pair j is
      // elements (32 (j / HV) + lane) V + 2 (j % HV) and the next one
      float2 x[NSEG][P];
      float ss[NSEG];
      int dt[NSEG], hh[NSEG];  // token offset from tf, head
      bool live[NSEG];
#pragma unroll
      for (int u = 0; u < NSEG; ++u) {
        const int i = i0 + 8 * u;
        live[u] = i < SPT && s0 + i < total;
        const int a = h0 + (live[u] ? i : 0);
        dt[u] = a / heads;
        hh[u] = live[u] ? a - dt[u] * heads : heads - 1;
        const uint4* xs = reinterpret_cast<const uint4*>(st + (live[u] ? i : 0) * HD);
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          const uint4 r = xs[c * 32 + lane];
          if constexpr (sizeof(T) == 4) {
            x[u][2 * c] = make_float2(__uint_as_float(r.x), __uint_as_float(r.y));
            x[u][2 * c + 1] = make_float2(__uint_as_float(r.z), __uint_as_float(r.w));
          } else {
            x[u][4 * c] = unpack2<T>(r.x);
            x[u][4 * c + 1] = unpack2<T>(r.y);
            x[u][4 * c + 2] = unpack2<T>(r.z);
            x[u][4 * c + 3] = unpack2<T>(r.w);
          }
        }
      }
#pragma unroll
      for (int u = 0; u < NSEG; ++u) {
        float2 q2 = fmul2(x[u][0], x[u][0]);
#pragma unroll
        for (int j = 1; j < P; ++j) q2 = ffma2(x[u][j], x[u][j], q2);
        ss[u] = q2.x + q2.y;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
#pragma unroll
        for (int u = 0; u < NSEG; ++u) ss[u] += __shfl_xor_sync(0xffffffffu, ss[u], o);
      }
#pragma unroll
      for (int u = 0; u < NSEG; ++u) {
        const bool is_v = hh[u] >= qh + kvh;
        const bool is_q = hh[u] < qh;
        float2 v[P];
        const float r = rsqrtf(ss[u] * (1.0f / HD) + eps);
        const float2 r2 = make_float2(r, r);
        const float* wrow = swt + (is_q ? 0 : 2 * HD);
        const float* brow = wrow + HD;
        const float4* w4p = reinterpret_cast<const float4*>(wrow) + lane;
        const float4* b4p = reinterpret_cast<const float4*>(brow) + lane;
#pragma unroll
        for (int j = 0; j < P; j += 2) {
          // without a bias the shared-memory read of the zero row is skipped
          const float4 w4 = w4p[(j / 2) * 32];
          const float4 b4 = has_b ? b4p[(j / 2) * 32] : make_float4(0.f, 0.f, 0.f, 0.f);
          v[j] = ffma2(fmul2(x[u][j], r2), make_float2(w4.x, w4.y), make_float2(b4.x, b4.y));
          v[j + 1] = ffma2(fmul2(x[u][j + 1], r2), make_float2(w4.z, w4.w), make_float2(b4.z, b4.w));
        }
        // cos / sin pair of elements (d, d + 1) of this segment's token
        const int64_t tok_u = tf + dt[u];
        const bool cs_vec = staged && sizeof(TS) == 4;
        auto cos_at = [&](int d) {
          return staged ? to_f32<TS>(scos[dt[u] * rd + d]) : to_f32<TS>(cos_t[tok_u * rd + d]);
        };
        auto sin_at = [&](int d) {
          return staged ? to_f32<TS>(ssin[dt[u] * rd + d]) : to_f32<TS>(sin_t[tok_u * rd + d]);
        };
        auto cs2 = [&](int d, float2& c2, float2& s2) {
          if (cs_vec) {
            c2 = *reinterpret_cast<const float2*>(scos + dt[u] * rd + d);
            s2 = *reinterpret_cast<const float2*>(ssin + dt[u] * rd + d);
          } else {
            c2 = make_float2(cos_at(d), cos_at(d + 1));
            s2 = make_float2(sin_at(d), sin_at(d + 1));
          }
        };
        if constexpr (MODE == 1) {
          // every lane shuffles (uniform); only rotated, live q / k chunks
          // use it.  Pair j of every lane is read by the shuffles before any
          // lane updates its own pair j.
          const bool apply = db0 < rd && !is_v;
          const float sg = db0 < half ? -1.f : 1.f;  // the rotate-half sign
#pragma unroll
          for (int j = 0; j < HV; ++j) {
            const float2 pv = make_float2(__shfl_sync(0xffffffffu, v[j].x, src),
                                          __shfl_sync(0xffffffffu, v[j].y, src));
            if (apply) {
              float2 c2, s2;
              cs2(db0 + 2 * j, c2, s2);
              v[j] = ffma2(v[j], c2, fmul2(pv, fmul2(s2, make_float2(sg, sg))));
            }
          }
        } else if constexpr (MODE == 2) {
          if (!is_v) {
            // chunk rows c < coff hold the first rotary half and pair with
            // c + coff, rows [coff, 2 coff) the second half: the distance is
            // one of a few compile-time values, so every register index is
            // static
#pragma unroll
            for (int o = 1; o <= NC / 2; ++o) {
              if (coff != o) continue;
              float2 w[P];
#pragma unroll
              for (int j = 0; j < P; ++j) w[j] = v[j];
#pragma unroll
              for (int c = 0; c < 2 * o; ++c) {
                const int db = (c * 32 + lane) * V;
                const bool lo = c < o;
                const int pc = lo ? c + o : c - o;
                const float sg = lo ? -1.f : 1.f;
#pragma unroll
                for (int jj = 0; jj < HV; ++jj) {
                  float2 c2, s2;
                  cs2(db + 2 * jj, c2, s2);
                  v[c * HV + jj] =
                      ffma2(w[c * HV + jj], c2, fmul2(w[pc * HV + jj], fmul2(s2, make_float2(sg, sg))));
                }
              }
            }
          }
        } else {
          if (!is_v) {
            // partner from the raw input in the stage, normalised the same way
            const T* xs = st + (i0 + 8 * u) * HD;
#pragma unroll
            for (int j = 0; j < 2 * P; ++j) {
              const int d = ((j / V) * 32 + lane) * V + (j % V);
              if (d < rd) {
                const int p = d < half ? d + half : d - half;
                const int wp = widx(p);
                const float pvv = to_f32<T>(xs[p]) * r * wrow[wp] + brow[wp];
                float& e = (j & 1) ? v[j >> 1].y : v[j >> 1].x;
                e = e * cos_at(d) + (d < half ? -pvv : pvv) * sin_at(d);
              }
            }
          }
        }
        if (!live[u]) continue;
        const int64_t tok = tok_u;
        T* dst = is_v ? vo + tok * (int64_t)kvh * HD + (int64_t)(hh[u] - qh - kvh) * HD
                 : is_q ? qo + tok * (int64_t)qh * HD + (int64_t)hh[u] * HD
                        : ko + tok * (int64_t)kvh * HD + (int64_t)(hh[u] - qh) * HD;
        float2 o[P];  // v heads are copied through unchanged
#pragma unroll
        for (int j = 0; j < P; ++j) o[j] = is_v ? x[u][j] : v[j];
#pragma unroll
        for (int c = 0; c < NC; ++c) {
          uint4 w;
          if constexpr (sizeof(T) == 4) {
            w = make_uint4(__float_as_uint(o[2 * c].x), __float_as_uint(o[2 * c].y),
                           __float_as_uint(o[2 * c + 1].x), __float_as_uint(o[2 * c + 1].y));
          } else {
            w = make_uint4(pack2<T>(o[4 * c]), pack2<T>(o[4 * c + 1]), pack2<T>(o[4 * c + 2]),
                           pack2<T>(o[4 * c + 3]));
          }
          reinterpret_cast<uint4*>(dst)[c * 32 + lane] = w;
        }
      }
    }
    __syncwarp();
    if (lane == 0) tc::mbar_arrive(&empty[s]);
  }
}

// partner rule of the streaming kernel for a rotary width (see the kernel)
template <typename T>
int rope_partner_mode(int rd) {
  constexpr int V = 16 / (int)sizeof(T);
  const int half = rd >> 1;
  return (half % V == 0 && rd <= 32 * V) ? 1 : (half % (32 * V) == 0 ? 2 : 0);
}

template <typename T, typename TW, typename TS, int HD>
int launch_rope_stream(const void* in, const void* s, const void* c, void* q, void* k, void* v,
                       const void* qw, const void* qb, const void* kw, const void* kb,
                       int64_t T_, int qh, int kvh, int rd, float eps, cudaStream_t st) {
  constexpr int SPT = RP_TILE / (HD * (int)sizeof(T));
  constexpr int WB = 4 * HD * 4;
  const int heads = qh + 2 * kvh;
  RopeStage L;
  L.maxtok = (SPT - 1) / heads + 2;
  // cos / sin rows ride in the stage when every tile's first row starts on a
  // 16-byte boundary and three stages still fit in shared memory
  const int64_t row = (int64_t)rd * sizeof(TS);
  L.cs = (row % 16 == 0 && aligned16(s) && aligned16(c)) ? (int)((L.maxtok * row + 127) / 128 * 128) : 0;
  L.stage = RP_TILE + 2 * L.cs;
  if (RP_NS * L.stage + WB + 128 > 227 * 1024) {
    L.cs = 0;
    L.stage = RP_TILE;
  }
  const int smem = RP_NS * L.stage + WB + 128;
  const int mode = rope_partner_mode<T>(rd);
  auto kern = mode == 1   ? split_rmsnorm_rope_stream_kernel<T, TW, TS, HD, 1>
              : mode == 2 ? split_rmsnorm_rope_stream_kernel<T, TW, TS, HD, 2>
                          : split_rmsnorm_rope_stream_kernel<T, TW, TS, HD, 0>;
  if (!set_stream_smem(kern, smem))
    return set_error(XOPS_ERR_CUDA, "split_rmsnorm_rope: shared-memory attribute failed");
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t tiles = cdiv64(T_ * heads, SPT);
  const unsigned grid = (unsigned)(tiles < 2 * (int64_t)sms ? tiles : 2 * (int64_t)sms);
  kern<<<grid, RP_NT, smem, st>>>((const T*)in, (const TS*)s, (const TS*)c, (T*)q, (T*)k, (T*)v,
                                  (const TW*)qw, (const TW*)qb, (const TW*)kw, (const TW*)kb, T_,
                                  qh, kvh, rd, L, eps);
  return check_launch("split_rmsnorm_rope");
}

template <typename T, typename TW, typename TS>
int dispatch_rope(const void* in, const void* s, const void* c, void* q, void* k, void* v,
                  const void* qw, const void* qb, const void* kw, const void* kb, int64_t T_,
                  int qh, int kvh, int hd, int rd, float eps, cudaStream_t st) {
  const int64_t items = T_ * (qh + 2 * kvh);
  const unsigned blocks = (unsigned)cdiv64(items, 8);
  // streaming path once the input is a few MB: enough tiles for a persistent grid
  if (items * hd * (int64_t)sizeof(T) >= (int64_t(4) << 20)) {
    if constexpr (sizeof(T) == 4) {  // a 128-wide bf16 head is 8 bytes per lane
      if (hd == 128)
        return launch_rope_stream<T, TW, TS, 128>(in, s, c, q, k, v, qw, qb, kw, kb, T_, qh, kvh, rd, eps, st);
    }
    if (hd == 256)
      return launch_rope_stream<T, TW, TS, 256>(in, s, c, q, k, v, qw, qb, kw, kb, T_, qh, kvh, rd, eps, st);
    if (hd == 512)
      return launch_rope_stream<T, TW, TS, 512>(in, s, c, q, k, v, qw, qb, kw, kb, T_, qh, kvh, rd, eps, st);
  }
  switch (hd) {
#define XOPS_R_CASE(EPL)                                                                      \
  case 32 * EPL:                                                                              \
    split_rmsnorm_rope_kernel<T, TW, TS, EPL><<<blocks, 256, 0, st>>>(                        \
        (const T*)in, (const TS*)s, (const TS*)c, (T*)q, (T*)k, (T*)v, (const TW*)qw,         \
        (const TW*)qb, (const TW*)kw, (const TW*)kb, T_, qh, kvh, rd, eps);                   \
    return check_launch("split_rmsnorm_rope");
    XOPS_R_CASE(2)
    XOPS_R_CASE(4)
    XOPS_R_CASE(8)
    XOPS_R_CASE(16)
#undef XOPS_R_CASE
    default:
      return set_error(XOPS_ERR_UNSUPPORTED,
                       "split_rmsnorm_rope: head_dim %d not in {64,128,256,512}", hd);
  }
}

// ----------------------------------------------------------------------------
// rope_inplace: interleaved (GPT-J style) RoPE on the last rope_dim dims of
// every (row, head) vector, in place (rope_inplace_kernel,
// triton_npu/triton_src/test_rope_inplace.py:17-46): pairs (2i, 2i+1) become
//   (x0 c0 - x1 s0,  x1 c1 + x0 s1)
// with sin / cos rows per batch entry shared by its heads.  One thread per
// pair, both elements loaded and stored as one 2-element vector.
// ----------------------------------------------------------------------------
template <typename T, typename TS>
__global__ void __launch_bounds__(256) rope_inplace_kernel(
    T* x, const TS* __restrict__ sin_t, const TS* __restrict__ cos_t, int64_t rows,
    int heads, int64_t sb, int64_t sh, int tail0, int pairs, int64_t scs) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= rows * heads * pairs) return;
  const int64_t v = i / pairs;
  const int p = (int)(i - v * pairs);
  const int64_t b = v / heads;
  const int h = (int)(v - b * heads);
  T* e = x + b * sb + h * sh + tail0 + 2 * p;
  const TS* sr = sin_t + b * scs + 2 * p;
  const TS* cr = cos_t + b * scs + 2 * p;
  const float x0 = to_f32<T>(e[0]), x1 = to_f32<T>(e[1]);
  const float o0 = x0 * to_f32<TS>(cr[0]) - x1 * to_f32<TS>(sr[0]);
  const float o1 = x1 * to_f32<TS>(cr[1]) + x0 * to_f32<TS>(sr[1]);
  e[0] = from_f32<T>(o0);
  e[1] = from_f32<T>(o1);
}

}  // namespace

int take_rope_error() {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_rope_error, sizeof(int)) != cudaSuccess) return -1;
  const int zero = 0;
  cudaMemcpyToSymbol(g_rope_error, &zero, sizeof(int));
  return v;
}
}  // namespace xops

using namespace xops;

extern "C" int xops_split_rmsnorm_rope(const void* input, const void* sin, const void* cos,
                                       void* q_out, void* k_out, void* v_out,
                                       const void* q_weight, const void* q_bias,
                                       const void* k_weight, const void* k_bias,
                                       int64_t num_tokens, int64_t q_hidden, int64_t kv_hidden,
                                       int64_t head_dim, int64_t rotary_dim, float eps,
                                       int dtype, int w_dtype, int sincos_dtype, void* stream) {
  XOPS_REQUIRE(num_tokens >= 0, "split_rmsnorm_rope: bad num_tokens");
  XOPS_REQUIRE(head_dim > 0 && (head_dim & (head_dim - 1)) == 0,
               "split_rmsnorm_rope head_dim must be a power of two");
  XOPS_REQUIRE(kv_hidden > 0 && kv_hidden % head_dim == 0,
               "split_rmsnorm_rope kv_hidden_size must be divisible by head_dim");
  XOPS_REQUIRE(q_hidden % kv_hidden == 0,
               "split_rmsnorm_rope q_hidden_size must be divisible by kv_hidden_size");
  XOPS_REQUIRE(rotary_dim > 0 && rotary_dim <= head_dim && rotary_dim % 2 == 0,
               "split_rmsnorm_rope: rotary_dim must be even and in (0, head_dim]");
  XOPS_REQUIRE(dtype == XOPS_F32 || dtype == XOPS_BF16, "split_rmsnorm_rope: bad dtype");
  XOPS_REQUIRE(w_dtype == XOPS_F32 || w_dtype == XOPS_BF16, "split_rmsnorm_rope: bad weight dtype");
  XOPS_REQUIRE(sincos_dtype == XOPS_F32 || sincos_dtype == XOPS_BF16,
               "split_rmsnorm_rope: bad sin/cos dtype");
  if (num_tokens == 0) return XOPS_OK;
  XOPS_REQUIRE(input && sin && cos && q_out && k_out && v_out && q_weight && k_weight,
               "split_rmsnorm_rope: null pointer");
  XOPS_REQUIRE((q_bias == nullptr) == (k_bias == nullptr),
               "split_rmsnorm_rope: q_bias and k_bias must both be given or both be null");
  XOPS_REQUIRE(aligned16(input) && aligned16(q_out) && aligned16(k_out) && aligned16(v_out) &&
                   aligned16(q_weight) && aligned16(k_weight),
               "split_rmsnorm_rope: tensors must be 16-byte aligned");
  const int qh = (int)(q_hidden / head_dim), kvh = (int)(kv_hidden / head_dim);
  cudaStream_t st = (cudaStream_t)stream;
  auto run = [&](auto t, auto tw, auto ts) {
    return dispatch_rope<decltype(t), decltype(tw), decltype(ts)>(
        input, sin, cos, q_out, k_out, v_out, q_weight, q_bias, k_weight, k_bias, num_tokens, qh,
        kvh, (int)head_dim, (int)rotary_dim, eps, st);
  };
  auto with_s = [&](auto t, auto tw) {
    return sincos_dtype == XOPS_F32 ? run(t, tw, float{}) : run(t, tw, __nv_bfloat16{});
  };
  auto with_w = [&](auto t) {
    return w_dtype == XOPS_F32 ? with_s(t, float{}) : with_s(t, __nv_bfloat16{});
  };
  return dtype == XOPS_F32 ? with_w(float{}) : with_w(__nv_bfloat16{});
}

extern "C" int xops_rope_inplace(void* x, const void* sin, const void* cos, int64_t rows,
                                 int64_t heads, int64_t hidden, int64_t rope_dim,
                                 int64_t x_stride_row, int64_t x_stride_head,
                                 int64_t sincos_stride, int x_dtype, int sincos_dtype,
                                 void* stream) {
  const char* what = "rope_inplace";
  XOPS_REQUIRE(rows >= 0 && heads >= 1 && hidden >= 1, "%s: bad shape", what);
  XOPS_REQUIRE(rope_dim >= 2 && rope_dim % 2 == 0 && rope_dim <= hidden,
               "%s: rope_dim must be even and in [2, hidden] (got %lld, hidden %lld)", what,
               (long long)rope_dim, (long long)hidden);
  XOPS_REQUIRE(sincos_stride >= rope_dim, "%s: sin/cos rows shorter than rope_dim", what);
  auto ok = [](int d) { return d == XOPS_F32 || d == XOPS_BF16 || d == XOPS_F16; };
  XOPS_REQUIRE(ok(x_dtype) && ok(sincos_dtype), "%s: unsupported dtype", what);
  const int64_t n = rows * heads * (rope_dim / 2);
  if (n == 0) return XOPS_OK;
  XOPS_REQUIRE(x && sin && cos, "%s: null pointer", what);
  cudaStream_t st = (cudaStream_t)stream;
  auto run = [&](auto tx, auto ts) {
    using TX = decltype(tx);
    using TS = decltype(ts);
    rope_inplace_kernel<TX, TS><<<(unsigned)cdiv64(n, 256), 256, 0, st>>>(
        (TX*)x, (const TS*)sin, (const TS*)cos, rows, (int)heads, x_stride_row, x_stride_head,
        (int)(hidden - rope_dim), (int)(rope_dim / 2), sincos_stride);
    return check_launch(what);
  };
  auto with_s = [&](auto tx) {
    switch (sincos_dtype) {
      case XOPS_F32: return run(tx, float{});
      case XOPS_BF16: return run(tx, __nv_bfloat16{});
      default: return run(tx, __half{});
    }
  };
  switch (x_dtype) {
    case XOPS_F32: return with_s(float{});
    case XOPS_BF16: return with_s(__nv_bfloat16{});
    default: return with_s(__half{});
  }
}
