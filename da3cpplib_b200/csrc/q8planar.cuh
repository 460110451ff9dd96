// Planar Q8_0: the resident layout of the ViT block linears.
//
// A GGUF Q8_0 matrix [N][K] is K/32 blocks per row of {f16 d; int8 q[32]} (34 bytes per
// 32 weights; ggml block_q8_0, dequantised as w = d * q). Planar Q8_0 keeps exactly
// those bytes in two planes whose rows a TMA can tile (16-byte aligned, no 34-byte
// stride):
//   q plane  int8 [N][K]          at offset 0
//   d plane  f16  [K/32][N]       at offset N * K (block scales, transposed so that the
//                                  scales of one K block for a run of rows are contiguous)
// Both the per-block f16 staging dequantisation and the GEMM that dequantises its weight
// tiles in shared memory produce w as f16(d * q) through q8x8_to_f16x8, so the two give
// bit-identical f16 weights.
#pragma once

#include <cuda_fp16.h>
#include <stdint.h>

#include "ops.h"

namespace da3b {

// Bytes of a planar Q8_0 matrix (the same as its GGUF Q8_0 bytes).
__host__ __device__ inline size_t q8p_bytes(int N, int K) {
  return static_cast<size_t>(N) * K + static_cast<size_t>(K / 32) * N * 2;
}

// f16(d * q) of eight int8 q (raw, K order from the low byte) with the scale pair d2 =
// (d, d). The int8 -> f16 conversion is exact: with the sign bit flipped a byte u = q + 128
// becomes the f16 1024 + u by placing it under the exponent byte 0x64, and subtracting
// 1152 leaves q. The product of an 11-bit and an 8-bit significand needs at most 19
// bits, so the one rounding of the f16 multiply gives the same value as rounding the
// exact f32 product d * q to f16.
__device__ __forceinline__ uint4 q8x8_to_f16x8(uint2 raw, __half2 d2) {
  const uint32_t x0 = raw.x ^ 0x80808080u, x1 = raw.y ^ 0x80808080u;
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1152
  uint32_t w[4] = {__byte_perm(x0, 0x64646464u, 0x4140), __byte_perm(x0, 0x64646464u, 0x4342),
                   __byte_perm(x1, 0x64646464u, 0x4140), __byte_perm(x1, 0x64646464u, 0x4342)};
  uint4 out;
  uint32_t* o = reinterpret_cast<uint32_t*>(&out);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const __half2 q = __hsub2(*reinterpret_cast<const __half2*>(&w[i]), bias);
    const __half2 v = __hmul2(q, d2);
    o[i] = *reinterpret_cast<const uint32_t*>(&v);
  }
  return out;
}

// Up to four planar Q8_0 matrices -> dense f16, thread `tid` of `nthreads` (grid-stride):
// a thread takes 16 consecutive weights of a row (one 16-byte load of the q plane, its
// block's scale, two 16-byte stores), consecutive threads consecutive pieces, so every
// load and store of a warp is one contiguous run.
__device__ __forceinline__ void q8p_segs_dequant(const Q8Segs& g, long tid, long nthreads) {
  for (int k = 0; k < g.n; ++k) {
    const Q8Seg& sg = g.s[k];
    const int K = sg.nblk * 32, per_row = K / 16;
    const long units = static_cast<long>(sg.rows) * per_row;
    const __half* dplane = reinterpret_cast<const __half*>(sg.q8 + static_cast<size_t>(sg.rows) * K);
    for (long u = tid; u < units; u += nthreads) {
      const int n = static_cast<int>(u / per_row), j = static_cast<int>(u % per_row);
      const uint4 q = __ldg(reinterpret_cast<const uint4*>(sg.q8 + static_cast<size_t>(n) * K + 16 * j));
      const __half d = dplane[static_cast<size_t>(j >> 1) * sg.rows + n];
      const __half2 d2 = __halves2half2(d, d);
      uint4* dst = reinterpret_cast<uint4*>(sg.out + static_cast<size_t>(n) * K + 16 * j);
      dst[0] = q8x8_to_f16x8(make_uint2(q.x, q.y), d2);
      dst[1] = q8x8_to_f16x8(make_uint2(q.z, q.w), d2);
    }
  }
}

// Grid blocks of the staging dequantisation of g (256 threads each).
inline long q8p_segs_blocks(const Q8Segs& g) {
  long units = 0;
  for (int k = 0; k < g.n; ++k) {
    const long u = static_cast<long>(g.s[k].rows) * g.s[k].nblk * 2;
    units = u > units ? u : units;
  }
  long blocks = (units + 255) / 256;
  return blocks > 148 * 8 ? 148 * 8 : blocks;
}

}  // namespace da3b
