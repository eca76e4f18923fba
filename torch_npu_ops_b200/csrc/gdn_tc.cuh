// Shared-memory tile addressing, operand descriptors and TMEM addressing
// for the tcgen05 kernels of the chunked gated delta rule (the fused
// operator in chunk_gdn.cu and the stand-alone stages in chunk_subops.cu).
// Tiles are 128-byte-swizzled (SW128) bf16: a [rows x 128] tile is two
// [rows x 64] halves `half_stride` bytes apart; a row of a half is 128 bytes
// of eight 16-byte chunks, chunk c of row r stored at c ^ (r & 7).
#pragma once
#include "gdn_common.cuh"
#include "tcgen05.cuh"

namespace xops {
namespace gdn {

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
// 16-byte chunk c of row r of an SW128 tile (c < 8: first half)
__device__ __forceinline__ uint32_t chunk_off(int r, int c, uint32_t half_stride) {
  return (uint32_t)((c >> 3) * half_stride + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}
__device__ __forceinline__ uint32_t elem_off(int r, int col, uint32_t half_stride) {
  return (uint32_t)((col >> 6) * half_stride + r * 128 + ((((col & 63) >> 3) ^ (r & 7)) << 4) +
                    (col & 7) * 2);
}
__device__ __forceinline__ uint32_t tm_addr(uint32_t base, int quarter, uint32_t col) {
  return base + ((uint32_t)(quarter * 32) << 16) + col;
}
// [64 x 128] bf16 rows (global row stride in elements) -> SW128 tile
__device__ __forceinline__ void cp_tile128(unsigned char* dst, uint32_t half_stride,
                                           const bf16* src, int64_t stride, int L, int t,
                                           int nthr) {
  for (int e = t; e < 64 * 16; e += nthr) {
    const int r = e >> 4, c = e & 15;
    const bool ok = r < L;
    cp_async16(dst + chunk_off(r, c, half_stride), src + (int64_t)(ok ? r : 0) * stride + c * 8,
               ok ? 16 : 0);
  }
}


// Four 8 x 8 bf16 blocks from the mma fragment layout (thread t holds row
// t / 4, elements 2 (t % 4) + {0, 1} of each) to shared memory transposed:
// block b's row i (its column i) goes to the address lane 8 b + i gives.
__device__ __forceinline__ void stmatrix_x4_trans(void* row, uint32_t b0, uint32_t b1, uint32_t b2,
                                                  uint32_t b3) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.trans.shared.b16 [%0], {%1, %2, %3, %4};\n" ::"r"(
                   tc::smem_addr(row)),
               "r"(b0), "r"(b1), "r"(b2), "r"(b3)
               : "memory");
}

}  // namespace gdn
}  // namespace xops
