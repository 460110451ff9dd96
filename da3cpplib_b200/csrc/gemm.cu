// Persistent warp-specialised tcgen05 GEMM / implicit-GEMM convolution for sm_100a.
//
// Roles (320 threads, one CTA per SM, grid = min(#tiles, #SMs)):
//   warp 0       TMA producer: streams A/B k-blocks into a kStages-deep ring of
//                128B-swizzled shared-memory stages (mbarrier full/empty pairs);
//   warp 1       MMA issuer: one thread issues tcgen05.mma (M=128, N=BN, K=16) into
//                one of two TMEM accumulators, commits stage releases and
//                "accumulator full" events;
//   warps 2..9   epilogue: tcgen05.ld the accumulator (warp w may read TMEM lanes
//                32*(w%4)..+31; two warps share each lane quarter and split the
//                tile's columns), apply the fused epilogue, store to global, and
//                release the accumulator so the MMA of the next tile overlaps.
//                f16 outputs, the QKV split and the f32 residual update go through a
//                per-warp staging buffer so that each store (or read-modify-write)
//                covers 8 rows x 64-128 contiguous bytes; the other kinds store row by
//                row.
// Tiles are visited m-major (all N tiles of one 128-row A panel back to back) so an
// A panel is read from HBM about once while the weights stay resident in L2.
#include <algorithm>
#include <cmath>
#include <atomic>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "gemm.h"
#include "ops.h"
#include "ptx.cuh"
#include "q8planar.cuh"

namespace da3b {

constexpr int kEpiWarps = 8;

template <int BN, bool kQ8 = false>
struct GemmCfg {
  static constexpr int kABytes = 128 * 64 * 2;
  static constexpr int kBBytes = BN * 64 * 2;
  // planar Q8_0 weights (kQ8): per stage the raw int8 tile [BN][64] and its two blocks'
  // scales [2][BN] f16 land next to the f16 B tile the converter warps write
  static constexpr int kQBytes = kQ8 ? BN * 64 : 0;
  static constexpr int kSBytes = kQ8 ? 2 * BN * 2 : 0;
  static constexpr int kTxBytes = kQ8 ? kABytes + kQBytes + kSBytes : kABytes + kBBytes;  // TMA bytes a stage
  static constexpr int kStageBytes = kABytes + kBBytes + kQBytes + kSBytes;
  // per epilogue warp: a [32][32] f32 staging buffer and its bias slice (BN >= 64).
  // They cost one pipeline stage (two at BN = 64); the staged epilogue made the
  // M = 1370 GEMMs of a batch-1 ViT-B 1.14-2.1x faster on a B200 (QKV 27.6 -> 13.1 us,
  // fc1 + GELU 29.1 -> 14.8 us), with bit-identical outputs.
  static constexpr int kEpiBufBytes = BN >= 64 ? 4096 : 0;
  static constexpr int kBiasFloats = BN >= 64 ? BN / 2 : 0;
  static constexpr int kEpiBytes = kEpiWarps * (kEpiBufBytes + kBiasFloats * 4);
  static constexpr int kStages =
      kQ8 ? (BN >= 128 ? 4 : 6) : ((BN >= 256) ? 3 : (BN >= 128 ? 5 : (BN >= 64 ? 6 : 8)));
  static constexpr int kAccCols = (BN < 32) ? 32 : BN;
  static constexpr int kTmemCols = (2 * kAccCols <= 64) ? 64 : (2 * kAccCols <= 128 ? 128 : (2 * kAccCols <= 256 ? 256 : 512));
  // epilogue constants of the fused out2a -> out2b stage (N == 32): bias, LayerNorm
  // gamma/beta, out2b weights [8][32] and biases [8], staged once per CTA
  static constexpr int kConstFloats = 32 * 3 + 8 * 32 + 8;
  static constexpr int kConstBytes = (kConstFloats * 4 + 127) / 128 * 128;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kConstBytes + kEpiBytes + 256;
  // N <= 32: the two epilogue warp halves take alternate tiles (each all columns)
  static constexpr bool kSplitTiles = BN < 64;
};

// erf(z) by Abramowitz & Stegun, Handbook of Mathematical Functions, formula 7.1.26:
// erf(z) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) e^(-z^2), t = 1 / (1 + p z),
// z >= 0, |error| <= 1.5e-7 (odd extension for z < 0). Far below the f16 rounding of
// the GELU output it feeds.
__device__ __forceinline__ float erf_as(float z) {
  const float az = fabsf(z);
  const float t = __fdividef(1.0f, fmaf(0.3275911f, az, 1.0f));
  float y = fmaf(1.061405429f, t, -1.453152027f);
  y = fmaf(y, t, 1.421413741f);
  y = fmaf(y, t, -0.284496736f);
  y = fmaf(y, t, 0.254829592f);
  y *= t;
  const float e = ex2_approx(-az * az * 1.4426950408889634f);
  return copysignf(fmaf(-y, e, 1.0f), z);
}
// Exact-form GELU 0.5 x (1 + erf(x / sqrt 2)) (ggml_gelu_erf, src/ggml_extend.hpp:22-25).
__device__ __forceinline__ float gelu_erf(float v) { return 0.5f * v * (1.0f + erf_as(v * 0.70710678118654752f)); }

// gelu_erf of two values with packed f32x2 arithmetic (sm_100): the same operations in
// the same order as gelu_erf, so each result is bit-identical to the scalar one, in
// about half the instructions.
__device__ __forceinline__ float2 f2c(float c) { return make_float2(c, c); }
__device__ __forceinline__ float2 gelu_erf2(float2 v) {
  const float2 z = __fmul2_rn(v, f2c(0.70710678118654752f));
  const float2 az = make_float2(fabsf(z.x), fabsf(z.y));
  const float2 d = __ffma2_rn(f2c(0.3275911f), az, f2c(1.0f));
  const float2 t = make_float2(__fdividef(1.0f, d.x), __fdividef(1.0f, d.y));
  float2 y = __ffma2_rn(f2c(1.061405429f), t, f2c(-1.453152027f));
  y = __ffma2_rn(y, t, f2c(1.421413741f));
  y = __ffma2_rn(y, t, f2c(-0.284496736f));
  y = __ffma2_rn(y, t, f2c(0.254829592f));
  y = __fmul2_rn(y, t);
  const float2 w = __fmul2_rn(__fmul2_rn(make_float2(-az.x, -az.y), az), f2c(1.4426950408889634f));
  const float2 ex = make_float2(ex2_approx(w.x), ex2_approx(w.y));
  float2 r = __ffma2_rn(make_float2(-y.x, -y.y), ex, f2c(1.0f));
  r = make_float2(copysignf(r.x, z.x), copysignf(r.y, z.y));
  return __fmul2_rn(__fmul2_rn(f2c(0.5f), v), __fadd2_rn(f2c(1.0f), r));
}

// Exact-form GELU with erf from Abramowitz & Stegun formula 7.1.28:
// erf(z) = 1 - (1 + a1 z + a2 z^2 + ... + a6 z^6)^-16, z >= 0, |error| <= 3e-7. With
// r = (1 + ...)^-16, 1 + erf(x / sqrt 2) is 2 - r for x >= 0 and r for x < 0 (no
// cancellation for negative x); one reciprocal (MUFU) and no exponential per value.
__device__ __forceinline__ float gelu_r(float v) {
  const float z = fabsf(v * 0.70710678118654752f);
  float p = fmaf(0.0000430638f, z, 0.0002765672f);
  p = fmaf(p, z, 0.0001520143f);
  p = fmaf(p, z, 0.0092705272f);
  p = fmaf(p, z, 0.0422820123f);
  p = fmaf(p, z, 0.0705230784f);
  p = fmaf(p, z, 1.0f);
  float r = __fdividef(1.0f, p);
  r *= r;
  r *= r;
  r *= r;
  r *= r;
  return 0.5f * v * (v >= 0.0f ? 2.0f - r : r);
}
// gelu_r of two values with packed f32x2 arithmetic, the same operations in the same
// order (bit-identical to the scalar form).
__device__ __forceinline__ float2 gelu_r2(float2 v) {
  const float2 zz = __fmul2_rn(v, f2c(0.70710678118654752f));
  const float2 z = make_float2(fabsf(zz.x), fabsf(zz.y));
  float2 p = __ffma2_rn(f2c(0.0000430638f), z, f2c(0.0002765672f));
  p = __ffma2_rn(p, z, f2c(0.0001520143f));
  p = __ffma2_rn(p, z, f2c(0.0092705272f));
  p = __ffma2_rn(p, z, f2c(0.0422820123f));
  p = __ffma2_rn(p, z, f2c(0.0705230784f));
  p = __ffma2_rn(p, z, f2c(1.0f));
  float2 r = make_float2(__fdividef(1.0f, p.x), __fdividef(1.0f, p.y));
  r = __fmul2_rn(r, r);
  r = __fmul2_rn(r, r);
  r = __fmul2_rn(r, r);
  r = __fmul2_rn(r, r);
  const float2 t = make_float2(v.x >= 0.0f ? 2.0f - r.x : r.x, v.y >= 0.0f ? 2.0f - r.y : r.y);
  return __fmul2_rn(__fmul2_rn(f2c(0.5f), v), t);
}

__device__ __forceinline__ float apply_act(float v, int act) {
  if (act == kActRelu) return fmaxf(v, 0.0f);
  if (act == kActGelu) return gelu_erf(v);
  if (act == kActGeluR) return gelu_r(v);
  return v;
}

__device__ __forceinline__ void load_h8(const __half* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store_h8(__half* p, const float* v) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Q8_0 round trip of one 32-element block with ggml's reference quantiser
// (quantize_row_q8_0_ref: d = amax/127, q = roundf(x * (1/d)), d stored as f16) followed
// by dequantisation d*q: the values a ggml Q8_0 x Q8_0 dot product sees on the
// activation side.
__device__ __forceinline__ void q8_roundtrip32(float (&t)[32]) {
  float amax = 0.f;
#pragma unroll
  for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(t[i]));
  const float d = amax / 127.0f;
  const float id = d != 0.f ? 1.0f / d : 0.0f;
  const float dh = __half2float(__float2half_rn(d));
#pragma unroll
  for (int i = 0; i < 32; ++i) t[i] = dh * roundf(t[i] * id);
}

constexpr int kGemmThreads = 64 + 32 * kEpiWarps;
constexpr int kConvWarps = 4;  // planar Q8_0 weight-tile converters (k_tc_gemm<BN, true>)
constexpr int kGemmThreadsQ8 = kGemmThreads + 32 * kConvWarps;

// 8 consecutive f32 (32-byte aligned) from global memory.
__device__ __forceinline__ void load_f8(const float* p, float* v) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ int remap_row(const EpiArgs& e, int row) {
  return e.rm_div > 0 ? (row / e.rm_div) * e.rm_mul + e.rm_add + row % e.rm_div : row;
}

// Epilogue for 32 accumulator columns [n_base, n_base+32) of one output row.
// `row` is the GEMM row (linear row, or output pixel index in conv mode).
__device__ __forceinline__ void epilogue32(const GemmGeom& g, const EpiArgs& e, int row, int n_base, float (&v)[32]) {
  const int nvalid = min(32, g.N - n_base);
  if (nvalid <= 0) return;
  switch (e.kind) {
    case kEpiF16: {
      const int orow = remap_row(e, row);
      if (e.q8) {  // full 32-column block (host enforces N % 32 == 0, no addends)
        float t[32];
        if (e.bias) {
#pragma unroll
          for (int j0 = 0; j0 < 32; j0 += 8) load_f8(e.bias + n_base + j0, t + j0);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) t[i] = 0.f;
        }
#pragma unroll
        for (int i = 0; i < 32; ++i) t[i] = apply_act(v[i] + t[i], e.act);
        q8_roundtrip32(t);
#pragma unroll
        for (int j0 = 0; j0 < 32; j0 += 8) store_h8(e.out + static_cast<size_t>(orow) * e.ld_out + n_base + j0, t + j0);
        break;
      }
      for (int j0 = 0; j0 < nvalid; j0 += 8) {  // N % 8 == 0 is enforced by the host
        float t[8];
        if (e.bias) {
          load_f8(e.bias + n_base + j0, t);
#pragma unroll
          for (int i = 0; i < 8; ++i) t[i] += v[j0 + i];
        } else {
#pragma unroll
          for (int i = 0; i < 8; ++i) t[i] = v[j0 + i];
        }
        if (e.res1) {
          const int r1 = e.res1_mod > 0 ? orow % e.res1_mod : orow;
          float s[8];
          load_h8(e.res1 + static_cast<size_t>(r1) * e.ld_res1 + n_base + j0, s);
#pragma unroll
          for (int i = 0; i < 8; ++i) t[i] += s[i];
        }
        if (e.res2) {
          float s[8];
          load_h8(e.res2 + static_cast<size_t>(orow) * e.ld_res2 + n_base + j0, s);
#pragma unroll
          for (int i = 0; i < 8; ++i) t[i] += s[i];
        }
        if (e.out_relu) {
          float q[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) q[i] = fmaxf(t[i], 0.0f);
          store_h8(e.out_relu + static_cast<size_t>(orow) * e.ld_out + n_base + j0, q);
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] = apply_act(t[i], e.act);
        store_h8(e.out + static_cast<size_t>(orow) * e.ld_out + n_base + j0, t);
      }
      break;
    }
    case kEpiResid: {
      const int orow = remap_row(e, row);
      float* p = e.resid + static_cast<size_t>(orow) * e.ld_resid + n_base;
      for (int j0 = 0; j0 < nvalid; j0 += 8) {
        float bb[8], sc[8];
        if (e.bias) load_f8(e.bias + n_base + j0, bb);
        else {
#pragma unroll
          for (int i = 0; i < 8; ++i) bb[i] = 0.f;
        }
        if (e.scale) load_f8(e.scale + n_base + j0, sc);
        else {
#pragma unroll
          for (int i = 0; i < 8; ++i) sc[i] = 1.f;
        }
        float4 x0 = *reinterpret_cast<float4*>(p + j0);
        float4 x1 = *reinterpret_cast<float4*>(p + j0 + 4);
        x0.x += sc[0] * (v[j0 + 0] + bb[0]); x0.y += sc[1] * (v[j0 + 1] + bb[1]);
        x0.z += sc[2] * (v[j0 + 2] + bb[2]); x0.w += sc[3] * (v[j0 + 3] + bb[3]);
        x1.x += sc[4] * (v[j0 + 4] + bb[4]); x1.y += sc[5] * (v[j0 + 5] + bb[5]);
        x1.z += sc[6] * (v[j0 + 6] + bb[6]); x1.w += sc[7] * (v[j0 + 7] + bb[7]);
        *reinterpret_cast<float4*>(p + j0) = x0;
        *reinterpret_cast<float4*>(p + j0 + 4) = x1;
      }
      break;
    }
    case kEpiTokens: {
      const int orow = remap_row(e, row);
      const int prow = 1 + row % e.rm_div;
      float* p = e.resid + static_cast<size_t>(orow) * e.ld_resid + n_base;
      const float* pp = e.pos + static_cast<size_t>(prow) * g.N + n_base;
      for (int j0 = 0; j0 < nvalid; j0 += 4) {
        float4 x;
        x.x = v[j0 + 0] + __ldg(e.bias + n_base + j0 + 0) + __ldg(pp + j0 + 0);
        x.y = v[j0 + 1] + __ldg(e.bias + n_base + j0 + 1) + __ldg(pp + j0 + 1);
        x.z = v[j0 + 2] + __ldg(e.bias + n_base + j0 + 2) + __ldg(pp + j0 + 2);
        x.w = v[j0 + 3] + __ldg(e.bias + n_base + j0 + 3) + __ldg(pp + j0 + 3);
        *reinterpret_cast<float4*>(p + j0) = x;
      }
      break;
    }
    case kEpiConvT: {
      const int hw = e.ct_hin * e.ct_win;
      const int b = row / hw, rem = row % hw;
      const int y = rem / e.ct_win, x = rem % e.ct_win;
      const int S = e.ct_s;
      const int hout = e.ct_hin * S, wout = e.ct_win * S;
      for (int j0 = 0; j0 < nvalid; j0 += 8) {
        const int n = n_base + j0;
        const int grp = n / e.ct_oc, oc = n % e.ct_oc;
        const int ky = grp / S, kx = grp % S;
        const size_t opix = (static_cast<size_t>(b) * hout + (S * y + ky)) * wout + (S * x + kx);
        float t[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) t[i] = v[j0 + i] + (e.bias ? __ldg(e.bias + oc + i) : 0.0f);
        store_h8(e.out + opix * e.ld_out + oc, t);
      }
      break;
    }
    case kEpiQKV: {
      // q | k thirds: plain f16 rows; v third: transposed store vt[seq][h][d][tok]
      // (a warp's 32 rows are 32 consecutive tokens: each d is one 64-byte run).
      if (n_base < 2 * e.vt_d) {
        for (int j0 = 0; j0 < nvalid; j0 += 8) {
          float t[8];
          if (e.bias) {
            load_f8(e.bias + n_base + j0, t);
#pragma unroll
            for (int i = 0; i < 8; ++i) t[i] += v[j0 + i];
          } else {
#pragma unroll
            for (int i = 0; i < 8; ++i) t[i] = v[j0 + i];
          }
          store_h8(e.out + static_cast<size_t>(row) * e.ld_out + n_base + j0, t);
        }
      } else {
        const int seq = row / e.vt_seqlen, tok = row % e.vt_seqlen;
        const int c0 = n_base - 2 * e.vt_d;  // 32 columns within one head (64 | c0 + 32)
        const int nh = e.vt_d / 64;
        __half* dst = e.vt + (static_cast<size_t>(seq) * nh * 64 + c0) * e.vt_ld + tok;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const float b = e.bias ? __ldg(e.bias + n_base + i) : 0.0f;
          dst[static_cast<size_t>(i) * e.vt_ld] = __float2half_rn(v[i] + b);
        }
      }
      break;
    }
    case kEpiOut2: {
      // out2a channels (N == 32) -> [channels-last LayerNorm] -> relu -> out2b 1x1 -> activation
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += e.bias ? __ldg(e.bias + j) : 0.0f;
      if (e.o2_ln_g) {
        float mean = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) mean += v[j];
        mean *= (1.0f / 32.0f);
        float var = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) { const float d = v[j] - mean; var += d * d; }
        var *= (1.0f / 32.0f);
        const float rstd = rsqrtf(var + e.o2_ln_eps);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = (v[j] - mean) * rstd * __ldg(e.o2_ln_g + j) + __ldg(e.o2_ln_b + j);
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.0f);
      for (int od = 0; od < e.o2_dim; ++od) {
        float l = __ldg(e.o2_b + od);
        const float* w = e.o2_w + od * 32;
#pragma unroll
        for (int j = 0; j < 32; ++j) l = fmaf(v[j], __ldg(w + j), l);
        e.o2_out[od][row] = out_act(l, e.o2_act[od], e.o2_scale);
      }
      break;
    }
    default: break;
  }
}

// Fused out2a -> [LayerNorm] -> relu -> out2b -> output activation of one pixel (the
// kEpiOut2 case of epilogue32) with its constants read from shared memory (c, staged
// once per CTA) instead of global memory per row.
__device__ __forceinline__ void epi_out2_smem(const EpiArgs& e, int row, float (&v)[32], const float* c) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] += c[j];
  if (e.o2_ln_g) {
    float mean = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) mean += v[j];
    mean *= (1.0f / 32.0f);
    float var = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) { const float d = v[j] - mean; var += d * d; }
    var *= (1.0f / 32.0f);
    const float rstd = rsqrtf(var + e.o2_ln_eps);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = (v[j] - mean) * rstd * c[32 + j] + c[64 + j];
  }
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.0f);
  for (int od = 0; od < e.o2_dim; ++od) {
    float l = c[352 + od];
    const float* w = c + 96 + od * 32;
#pragma unroll
    for (int j = 0; j < 32; ++j) l = fmaf(v[j], w[j], l);
    e.o2_out[od][row] = out_act(l, e.o2_act[od], e.o2_scale);
  }
}

// Transposed epilogue of one warp: its 32 accumulator rows (TMEM lanes; `row` is
// this lane's output row or -1) x columns [c_begin, c_end) of the tile at column n_tile.
// Each 32x32 f32 chunk is written row-per-lane into the warp's staging buffer (16-byte
// pieces XOR-swizzled by row & 7: conflict-free both ways) and read back so that lane
// l holds columns 8*(l&3) .. +7 of row 8k + (l>>2), k = 0..3. All per-element work then
// runs in that layout, and each global store instruction covers 8 rows x 64 contiguous
// bytes. kEpiF16 with res1/res2/out_relu: bias, residual addends, relu copy, activation
// in that layout; kEpiF16 without them and the q|k thirds of kEpiQKV: the row-layout
// path (bias and activation per row, f16 staging); the v third of kEpiQKV transposed per
// (sequence, head) into vt.
// bsm: this warp's bias slice [c_end - c_begin] in shared memory (zeros without bias).
template <int BN>
__device__ __forceinline__ void epi_transposed(const GemmGeom& g, const EpiArgs& e, uint32_t tbase, int c_begin,
                                               int c_end, int n_tile, int row, int lane, float* stg,
                                               const float* bsm) {
  const int s = lane & 3, rsub = lane >> 2;
  const int orow = (row >= 0 && e.kind == kEpiF16) ? remap_row(e, row) : row;
#pragma unroll 1
  for (int c = c_begin; c < c_end; c += 32) {
    uint32_t raw[32];
    tmem_ld32(tbase + c, raw);
    tmem_wait_ld();
    const int n_base = n_tile + c;
    if (n_base >= g.N) continue;  // warp-uniform
    if (e.kind == kEpiQKV ? n_base < 2 * e.vt_d : (e.kind == kEpiF16 && !e.res1 && !e.res2 && !e.out_relu)) {
      // Plain f16 output: bias and activation while the lane holds its own row (columns
      // c .. c+31), then f16 staging: each lane writes its row's 64 bytes (16-byte pieces
      // swizzled by (row >> 1) & 3) and reads back 8 consecutive columns of row
      // 8k + (lane >> 2); both phases are conflict-free, and each store still covers
      // 8 rows x 64 contiguous bytes. Half the staged bytes of the f32 path below and
      // about a third of its shared-memory instructions: the tensor pipe runs measurably
      // slower while epilogue warps issue, so the epilogue is kept short.
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; j += 4) {
        const float4 bb = *reinterpret_cast<const float4*>(bsm + (c - c_begin) + j);
        v[j] = __uint_as_float(raw[j]) + bb.x;
        v[j + 1] = __uint_as_float(raw[j + 1]) + bb.y;
        v[j + 2] = __uint_as_float(raw[j + 2]) + bb.z;
        v[j + 3] = __uint_as_float(raw[j + 3]) + bb.w;
      }
      if (e.kind == kEpiF16) {
        if (e.act == kActGelu) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 gv = gelu_erf2(make_float2(v[i], v[i + 1]));
            v[i] = gv.x;
            v[i + 1] = gv.y;
          }
        } else if (e.act == kActGeluR) {
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float2 gv = gelu_r2(make_float2(v[i], v[i + 1]));
            v[i] = gv.x;
            v[i + 1] = gv.y;
          }
        } else if (e.act == kActRelu) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = fmaxf(v[i], 0.0f);
        }
      }
      uint32_t h[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        __half2 hh = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
        h[i] = *reinterpret_cast<uint32_t*>(&hh);
      }
      uint4* srow = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(stg) + lane * 64);
      const int wsw = (lane >> 1) & 3;
#pragma unroll
      for (int q = 0; q < 4; ++q) srow[q ^ wsw] = make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
      __syncwarp();
      uint4 o[4];
      int rr[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int r = 8 * k + rsub;
        rr[k] = __shfl_sync(0xffffffffu, orow, r);
        o[k] = reinterpret_cast<const uint4*>(reinterpret_cast<const uint8_t*>(stg) + r * 64)[s ^ ((r >> 1) & 3)];
      }
      __syncwarp();  // every lane has read the staging buffer before the next chunk overwrites it
      const int n = n_base + 8 * s;
      if (n < g.N) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
          if (rr[k] >= 0) *reinterpret_cast<uint4*>(e.out + static_cast<size_t>(rr[k]) * e.ld_out + n) = o[k];
      }
      continue;
    }
    if (e.kind == kEpiQKV && n_base >= 2 * e.vt_d) {
      // v third: lanes are consecutive tokens, so each of the 32 columns is one
      // contiguous run of the transposed row
      if (row >= 0) {
        const int seq = row / e.vt_seqlen, tok = row % e.vt_seqlen;
        const int c0 = n_base - 2 * e.vt_d;
        __half* dst = e.vt + (static_cast<size_t>(seq) * (e.vt_d / 64) * 64 + c0) * e.vt_ld + tok;
#pragma unroll
        for (int i = 0; i < 32; ++i)
          dst[static_cast<size_t>(i) * e.vt_ld] = __float2half_rn(__uint_as_float(raw[i]) + bsm[c - c_begin + i]);
      }
      continue;
    }
    uint4* wrow = reinterpret_cast<uint4*>(stg + lane * 32);
#pragma unroll
    for (int j = 0; j < 8; ++j)
      wrow[j ^ (lane & 7)] = make_uint4(raw[4 * j], raw[4 * j + 1], raw[4 * j + 2], raw[4 * j + 3]);
    __syncwarp();
    const int n = n_base + 8 * s;
    const bool col_ok = n < g.N;
    const float4 b0 = *reinterpret_cast<const float4*>(bsm + (c - c_begin) + 8 * s);
    const float4 b1 = *reinterpret_cast<const float4*>(bsm + (c - c_begin) + 8 * s + 4);
    // gather all four row groups first: 32 independent values per lane for the math
    float t[4][8];
    int rr[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = 8 * k + rsub;
      rr[k] = __shfl_sync(0xffffffffu, orow, r);
      const uint4* rrow = reinterpret_cast<const uint4*>(stg + r * 32);
      const uint4 a = rrow[(2 * s) ^ (r & 7)], b = rrow[(2 * s + 1) ^ (r & 7)];
      t[k][0] = __uint_as_float(a.x) + b0.x;
      t[k][1] = __uint_as_float(a.y) + b0.y;
      t[k][2] = __uint_as_float(a.z) + b0.z;
      t[k][3] = __uint_as_float(a.w) + b0.w;
      t[k][4] = __uint_as_float(b.x) + b1.x;
      t[k][5] = __uint_as_float(b.y) + b1.y;
      t[k][6] = __uint_as_float(b.z) + b1.z;
      t[k][7] = __uint_as_float(b.w) + b1.w;
    }
    __syncwarp();  // every lane has read the staging buffer before the next chunk overwrites it
    if (e.kind == kEpiF16) {
      if (e.res1) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (rr[k] < 0 || !col_ok) continue;
          const int r1 = e.res1_mod > 0 ? rr[k] % e.res1_mod : rr[k];
          float a1[8];
          load_h8(e.res1 + static_cast<size_t>(r1) * e.ld_res1 + n, a1);
#pragma unroll
          for (int i = 0; i < 8; ++i) t[k][i] += a1[i];
        }
      }
      if (e.res2) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (rr[k] < 0 || !col_ok) continue;
          float a2[8];
          load_h8(e.res2 + static_cast<size_t>(rr[k]) * e.ld_res2 + n, a2);
#pragma unroll
          for (int i = 0; i < 8; ++i) t[k][i] += a2[i];
        }
      }
      if (e.out_relu) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (rr[k] < 0 || !col_ok) continue;
          float rl[8];
#pragma unroll
          for (int i = 0; i < 8; ++i) rl[i] = fmaxf(t[k][i], 0.0f);
          store_h8(e.out_relu + static_cast<size_t>(rr[k]) * e.ld_out + n, rl);
        }
      }
      if (e.act == kActGelu) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            const float2 gv = gelu_erf2(make_float2(t[k][i], t[k][i + 1]));
            t[k][i] = gv.x;
            t[k][i + 1] = gv.y;
          }
      } else if (e.act == kActGeluR) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int i = 0; i < 8; i += 2) {
            const float2 gv = gelu_r2(make_float2(t[k][i], t[k][i + 1]));
            t[k][i] = gv.x;
            t[k][i + 1] = gv.y;
          }
      } else if (e.act == kActRelu) {
#pragma unroll
        for (int k = 0; k < 4; ++k)
#pragma unroll
          for (int i = 0; i < 8; ++i) t[k][i] = fmaxf(t[k][i], 0.0f);
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (rr[k] >= 0 && col_ok) store_h8(e.out + static_cast<size_t>(rr[k]) * e.ld_out + n, t[k]);
  }
}


// kEpiResid through the same staging: each 32x32 f32 chunk is read back so that lane
// l holds columns 8*(l&3)..+7 of row 8k + (l>>2); the read-modify-write of the f32
// residual then covers 8 rows x 128 contiguous bytes per instruction.
__device__ __forceinline__ void epi_resid_transposed(const GemmGeom& g, const EpiArgs& e, uint32_t tbase, int c_begin,
                                                     int c_end, int n_tile, int row, int lane, float* stg) {
  const int s = lane & 3, rsub = lane >> 2;
  const int orow = row >= 0 ? remap_row(e, row) : -1;
  int rr[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) rr[k] = __shfl_sync(0xffffffffu, orow, 8 * k + rsub);
#pragma unroll 1
  for (int c = c_begin; c < c_end; c += 32) {
    uint32_t raw[32];
    tmem_ld32(tbase + c, raw);
    tmem_wait_ld();
    const int n_base = n_tile + c;
    if (n_base >= g.N) continue;  // warp-uniform
    uint4* wrow = reinterpret_cast<uint4*>(stg + lane * 32);
#pragma unroll
    for (int j = 0; j < 8; ++j) wrow[j ^ (lane & 7)] = make_uint4(raw[4 * j], raw[4 * j + 1], raw[4 * j + 2], raw[4 * j + 3]);
    __syncwarp();
    float t[4][8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int r = 8 * k + rsub;
      const uint4* rrow = reinterpret_cast<const uint4*>(stg + r * 32);
      const uint4 a = rrow[(2 * s) ^ (r & 7)], b = rrow[(2 * s + 1) ^ (r & 7)];
      t[k][0] = __uint_as_float(a.x); t[k][1] = __uint_as_float(a.y); t[k][2] = __uint_as_float(a.z);
      t[k][3] = __uint_as_float(a.w); t[k][4] = __uint_as_float(b.x); t[k][5] = __uint_as_float(b.y);
      t[k][6] = __uint_as_float(b.z); t[k][7] = __uint_as_float(b.w);
    }
    __syncwarp();
    const int n = n_base + 8 * s;
    if (n >= g.N) continue;
    float bb[8], sc[8];
    if (e.bias) load_f8(e.bias + n, bb);
    else {
#pragma unroll
      for (int i = 0; i < 8; ++i) bb[i] = 0.f;
    }
    if (e.scale) load_f8(e.scale + n, sc);
    else {
#pragma unroll
      for (int i = 0; i < 8; ++i) sc[i] = 1.f;
    }
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      if (rr[k] < 0) continue;
      float* p = e.resid + static_cast<size_t>(rr[k]) * e.ld_resid + n;
      float4 x0 = *reinterpret_cast<float4*>(p);
      float4 x1 = *reinterpret_cast<float4*>(p + 4);
      x0.x += sc[0] * (t[k][0] + bb[0]); x0.y += sc[1] * (t[k][1] + bb[1]);
      x0.z += sc[2] * (t[k][2] + bb[2]); x0.w += sc[3] * (t[k][3] + bb[3]);
      x1.x += sc[4] * (t[k][4] + bb[4]); x1.y += sc[5] * (t[k][5] + bb[5]);
      x1.z += sc[6] * (t[k][6] + bb[6]); x1.w += sc[7] * (t[k][7] + bb[7]);
      *reinterpret_cast<float4*>(p) = x0;
      *reinterpret_cast<float4*>(p + 4) = x1;
    }
  }
}

// kQ8: the weights are planar Q8_0 (q8planar.cuh): tmB maps the int8 plane (box [BN][64],
// no swizzle), tmS the f16 scale plane (box [2][BN]); four more warps (10-13) turn each
// stage's raw tile into the f16 B tile, 128B-swizzled as a TMA would have written it,
// and release it to the MMA warp. Otherwise tmB maps f16 weights and tmS is unused.
template <int BN, bool kQ8>
__global__ void __launch_bounds__(kQ8 ? kGemmThreadsQ8 : kGemmThreads, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmS, const GemmGeom g, const EpiArgs e, int* status) {
  using Cfg = GemmCfg<BN, kQ8>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + Cfg::kStages * Cfg::kABytes;
  uint8_t* sQ = sB + Cfg::kStages * Cfg::kBBytes;  // kQ8: raw int8 tiles
  uint8_t* sS = sQ + Cfg::kStages * Cfg::kQBytes;  // kQ8: their scales
  float* sConst = reinterpret_cast<float*>(smem + Cfg::kStages * Cfg::kStageBytes);
  uint8_t* sEpi = smem + Cfg::kStages * Cfg::kStageBytes + Cfg::kConstBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + Cfg::kStages * Cfg::kStageBytes + Cfg::kConstBytes + Cfg::kEpiBytes);
  uint64_t* empty = full + Cfg::kStages;
  uint64_t* tfull = empty + Cfg::kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* conv = tempty + 2;  // kQ8: [kStages] the stage's f16 B tile is written
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(conv + (kQ8 ? Cfg::kStages : 0));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int num_tiles = g.num_m_tiles * g.num_n_tiles;
  // K split (g.ksplit > 1, BN >= 64): a cluster of ks CTAs shares one tile, CTA `split`
  // (its cluster rank) taking k-blocks [kb0, kb1); the partial accumulators are summed
  // into the first CTA's TMEM in rank order before its epilogue. Otherwise the grid is
  // persistent over tiles and one CTA takes all k-blocks.
  const int ks = (!kQ8 && g.ksplit > 1) ? g.ksplit : 1;  // not with the Q8_0 converters
  const int split = static_cast<int>(blockIdx.x) % ks;
  const int t_first = static_cast<int>(blockIdx.x) / ks, t_step = static_cast<int>(gridDim.x) / ks;
  const int kb0 = split * g.num_kb / ks, kb1 = (split + 1) * g.num_kb / ks;

  if (e.kind == kEpiOut2) {
    // [0,32) bias, [32,64) LN gamma, [64,96) LN beta, [96,352) out2b weights, [352,360) out2b bias
    for (int i = threadIdx.x; i < Cfg::kConstFloats; i += blockDim.x) {
      float v = 0.f;
      if (i < 32) v = e.bias ? e.bias[i] : 0.f;
      else if (i < 64) v = e.o2_ln_g ? e.o2_ln_g[i - 32] : 1.f;
      else if (i < 96) v = e.o2_ln_b ? e.o2_ln_b[i - 64] : 0.f;
      else if (i < 352) v = (i - 96) < e.o2_dim * 32 ? e.o2_w[i - 96] : 0.f;
      else v = (i - 352) < e.o2_dim ? e.o2_b[i - 352] : 0.f;
      sConst[i] = v;
    }
  }

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], Cfg::kSplitTiles ? kEpiWarps / 2 : kEpiWarps);
    }
    if (kQ8)
      for (int st = 0; st < Cfg::kStages; ++st) mbar_init(&conv[st], kConvWarps);
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    if (kQ8) prefetch_tmap(&tmS);
  }
  if (warp == 1) tmem_alloc(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = t_first; t < num_tiles && ok; t += t_step) {
        const int mt = t / g.num_n_tiles, nt = t % g.num_n_tiles;
        const int n0 = nt * BN;
        int cb = 0, cx = 0, cy = 0;
        if (g.mode == kModeConv) {
          const int per_img = g.tiles_x * g.tiles_y;
          cb = mt / per_img;
          const int rem = mt % per_img;
          cy = (rem / g.tiles_x) * g.bh;
          cx = (rem % g.tiles_x) * g.bw;
        }
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, status, kStatusTimeoutEmpty)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[stage], Cfg::kTxBytes);
          uint8_t* a_dst = sA + stage * Cfg::kABytes;
          uint8_t* b_dst = sB + stage * Cfg::kBBytes;
          if (kQ8) {
            tma_load_2d(a_dst, &tmA, &full[stage], kb * 64, mt * 128);
            tma_load_2d(sQ + stage * Cfg::kQBytes, &tmB, &full[stage], kb * 64, n0);
            tma_load_2d(sS + stage * Cfg::kSBytes, &tmS, &full[stage], n0, kb * 2);
          } else if (g.mode == kModeConv) {
            const int tap = kb / g.ic_chunks;
            const int ic0 = (kb % g.ic_chunks) * 64;
            const int dy = tap / g.ksize - g.pad, dx = tap % g.ksize - g.pad;
            tma_load_4d(a_dst, &tmA, &full[stage], ic0, cx + dx, cy + dy, cb);
            tma_load_2d(b_dst, &tmB, &full[stage], tap * g.icp + ic0, n0);
          } else {
            tma_load_2d(a_dst, &tmA, &full[stage], kb * 64, mt * 128);
            tma_load_2d(b_dst, &tmB, &full[stage], kb * 64, n0);
          }
          if (++stage == Cfg::kStages) { stage = 0; phase ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t idesc = umma_idesc_f16(128, BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = t_first; t < num_tiles && ok; t += t_step, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, status, kStatusTimeoutAccumFree)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kAccCols;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, status, kStatusTimeoutFull)) { ok = false; break; }
          if (kQ8 && !mbar_wait(&conv[stage], phase, status, kStatusTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(sA + stage * Cfg::kABytes));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + stage * Cfg::kBBytes));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > kb0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
          if (++stage == Cfg::kStages) { stage = 0; phase ^= 1u; }
        }
        if (ok) umma_commit(&tfull[acc]);
      }
    }
    __syncwarp();
  } else if (kQ8 && warp >= 2 + kEpiWarps) {
    // ------------------------------------------------------------ weight-tile dequantisation
    // 128 threads, 16-byte pieces (8 weights): thread ct takes column chunk c = ct % 8 of
    // rows ct / 8 + 16 i, so a warp reads 4 raw rows (256 contiguous bytes) and writes 4
    // swizzled f16 rows (512 contiguous bytes) per step; chunk c of row n goes to
    // 16-byte slot c ^ (n % 8) of the row, where the 128B swizzle of a TMA load puts it.
    const int ct = threadIdx.x - 32 * (2 + kEpiWarps);
    const int c = ct & 7, n_lo = ct >> 3;
    const int swz = (c ^ (n_lo & 7)) << 4;
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int t = t_first; t < num_tiles && ok; t += t_step) {
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!mbar_wait_warp(&full[stage], phase, status, kStatusTimeoutFull)) { ok = false; break; }
        const uint8_t* qt = sQ + stage * Cfg::kQBytes;
        const __half* sc = reinterpret_cast<const __half*>(sS + stage * Cfg::kSBytes) + (c >> 2) * BN;
        uint8_t* bt = sB + stage * Cfg::kBBytes;
#pragma unroll
        for (int i = 0; i < BN / 16; ++i) {
          const int n = n_lo + 16 * i;
          const uint2 raw = *reinterpret_cast<const uint2*>(qt + n * 64 + c * 8);
          const __half d = sc[n];
          *reinterpret_cast<uint4*>(bt + n * 128 + swz) = q8x8_to_f16x8(raw, __halves2half2(d, d));
        }
        fence_proxy_async_smem();  // the tensor core reads the tile through the async proxy
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[stage]);
        if (++stage == Cfg::kStages) { stage = 0; phase ^= 1u; }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int r = q * 32 + lane;
    // column range of this warp: halves of the tile when BN >= 64
    const int half = (warp - 2) / 4;
    const int c_begin = Cfg::kSplitTiles ? 0 : half * (BN / 2);
    const int c_end = Cfg::kSplitTiles ? BN : c_begin + BN / 2;
    bool split_ok = false;
    // the epilogue of tile t from accumulator buffer acc (after tfull when wait_full)
    auto epi_tile = [&](int t, int acc, bool wait_full, uint32_t acc_phase) -> bool {
      const int mt = t / g.num_n_tiles, nt = t % g.num_n_tiles;
      int row = -1;
      if (g.mode == kModeConv) {
        const int per_img = g.tiles_x * g.tiles_y;
        const int b = mt / per_img, rem = mt % per_img;
        const int y = (rem / g.tiles_x) * g.bh + r / g.bw;
        const int x = (rem % g.tiles_x) * g.bw + r % g.bw;
        if (y < g.H && x < g.W) row = (b * g.H + y) * g.W + x;
      } else {
        const int m = mt * 128 + r;
        if (m < g.M) row = m;
      }
      const bool staged = BN >= 64 && ((e.kind == kEpiF16 && !e.q8) || e.kind == kEpiQKV || e.kind == kEpiResid);
      float4 bq = make_float4(0.f, 0.f, 0.f, 0.f);
      const int bcol = nt * BN + c_begin + 4 * lane;
      if (staged && e.kind != kEpiResid && e.bias && 4 * lane < c_end - c_begin && bcol < g.N)
        bq = __ldg(reinterpret_cast<const float4*>(e.bias + bcol));
      if (wait_full && !mbar_wait_warp(&tfull[acc], acc_phase, status, kStatusTimeoutAccum)) return false;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * Cfg::kAccCols;
      if (staged) {
        uint8_t* ebuf = sEpi + (warp - 2) * Cfg::kEpiBufBytes;
        float* ebias = reinterpret_cast<float*>(sEpi + 8 * Cfg::kEpiBufBytes) + (warp - 2) * Cfg::kBiasFloats;
        if (e.kind == kEpiResid) {
          epi_resid_transposed(g, e, tbase, c_begin, c_end, nt * BN, row, lane, reinterpret_cast<float*>(ebuf));
        } else {
          if (4 * lane < c_end - c_begin) *reinterpret_cast<float4*>(ebias + 4 * lane) = bq;
          __syncwarp();
          epi_transposed<BN>(g, e, tbase, c_begin, c_end, nt * BN, row, lane, reinterpret_cast<float*>(ebuf), ebias);
        }
      } else
#pragma unroll 1
      for (int c = c_begin; c < c_end; c += 32) {
        uint32_t raw[32];
        tmem_ld32(tbase + c, raw);
        tmem_wait_ld();
        if (row >= 0) {
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]);
          if (e.kind == kEpiOut2) epi_out2_smem(e, row, v, sConst);
          else epilogue32(g, e, row, nt * BN + c, v);
        }
      }
      return true;
    };
    if (ks > 1) {
      // one tile per cluster: the other CTAs hand their partial accumulator (this
      // warp's columns) to the first through their idle A / B ring, column-chunk-major
      // (float4 chunk j of row r at [j][r]), so that a warp's remote load reads 512
      // contiguous bytes
      if (t_first < num_tiles && mbar_wait_warp(&tfull[0], 0, status, kStatusTimeoutAccum)) {
        tc_fence_after();
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        if (split != 0) {
          float4* share = reinterpret_cast<float4*>(smem);
#pragma unroll 1
          for (int c = c_begin; c < c_end; c += 32) {
            uint32_t raw[32];
            tmem_ld32(tbase + c, raw);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 8; ++i)
              share[((c >> 2) + i) * 128 + r] = make_float4(__uint_as_float(raw[4 * i]), __uint_as_float(raw[4 * i + 1]),
                                                            __uint_as_float(raw[4 * i + 2]), __uint_as_float(raw[4 * i + 3]));
          }
        }
        split_ok = true;
      }
    } else {
      int it = 0;
      for (int t = t_first; t < num_tiles; t += t_step, ++it) {
        if (Cfg::kSplitTiles && (it & 1) != half) continue;  // the other half takes this tile
        const int acc = it & 1;
        if (!epi_tile(t, acc, true, (it >> 1) & 1)) break;
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[acc]);
      }
    }
    if (ks > 1) {
      cluster_sync();  // every partial accumulator is in its CTA's shared memory
      if (split == 0 && split_ok) {
        // sum the shares into this CTA's accumulator in rank order, then the epilogue
        const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16);
        const uint32_t share = smem_u32(smem);
#pragma unroll 1
        for (int c = c_begin; c < c_end; c += 32) {
          uint32_t raw[32];
          tmem_ld32(tbase + c, raw);
          tmem_wait_ld();
          for (int sp = 1; sp < ks; ++sp) {
            float4 v[8];
            const uint32_t peer = mapa_shared(share + static_cast<uint32_t>(((c >> 2) * 128 + r) * 16), static_cast<uint32_t>(sp));
#pragma unroll
            for (int i = 0; i < 8; ++i) v[i] = ld_dsmem_f4(peer + static_cast<uint32_t>(i * 128 * 16));
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              raw[4 * i] = __float_as_uint(__uint_as_float(raw[4 * i]) + v[i].x);
              raw[4 * i + 1] = __float_as_uint(__uint_as_float(raw[4 * i + 1]) + v[i].y);
              raw[4 * i + 2] = __float_as_uint(__uint_as_float(raw[4 * i + 2]) + v[i].z);
              raw[4 * i + 3] = __float_as_uint(__uint_as_float(raw[4 * i + 3]) + v[i].w);
            }
          }
          tmem_st32(tbase + c, raw);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        epi_tile(t_first, 0, false, 0);
      }
    }
  }
  // the K-split cluster's second barrier: no CTA leaves while the first may still read
  // its share (every thread of every CTA of the cluster takes both barriers)
  if (ks > 1) {
    if (warp < 2 || (kQ8 && warp >= 2 + kEpiWarps)) cluster_sync();
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::kTmemCols);
  }
}


// ---------------------------------------------------------------- 2-SM variant
// Same roles over a CTA pair (cluster of 2, cta_group::2): a tile is 256 rows x BN;
// each CTA TMA-loads its own 128 rows of A and BN/2 rows of B (no multicast) and
// both loads complete on the leader's (rank 0) stage barrier; the leader's single
// MMA thread issues M=256 tcgen05.mma over both CTAs' shared memory, which leaves
// each CTA's 128 rows of the accumulator in its own TMEM; commits are multicast to
// both CTAs; the peer's epilogue releases the accumulator with a remote arrive on
// the leader's barrier. Per SM the operand traffic per MMA is 3/4 of the 1-SM tile's.
// kStaged: the epilogue writes through shared memory and TMA stores / reduces (one
// [32 rows][128 B] staging buffer per epilogue warp), otherwise straight from registers.
// Both variants keep the CTA near 198 KB of shared memory: more would shrink the L1
// that serves the epilogue's bias loads and direct stores.
template <int BN, bool kStaged>
struct Gemm2Cfg {
  static constexpr int kABytes = 128 * 64 * 2;
  static constexpr int kBBytes = (BN / 2) * 64 * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kEpiBufBytes = 4096;
  static constexpr int kBiasBytes = (BN / 2) * 4;  // one warp's bias slice (transposed epilogue)
  static constexpr int kEpiBytes = kStaged ? kEpiWarps * (kEpiBufBytes + kBiasBytes) : 0;
  static constexpr int kStages = (196 * 1024 - kEpiBytes) / kStageBytes > 6 ? 6 : (196 * 1024 - kEpiBytes) / kStageBytes;
  static constexpr int kAccCols = (BN < 32) ? 32 : BN;
  static constexpr int kTmemCols = (2 * kAccCols <= 64) ? 64 : (2 * kAccCols <= 128 ? 128 : (2 * kAccCols <= 256 ? 256 : 512));
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kEpiBytes + 256;
};

// Stores one warp's [32 rows][128 B] slice through its 128B-swizzled staging buffer and
// a TMA store (f16, 64 columns) or TMA reduce-add (f32, 32 columns). Lane = tile row.
__device__ __forceinline__ void stage_and_store(uint8_t* buf, const uint32_t (&words)[32], int lane,
                                                const CUtensorMap* map, int x, int y, bool reduce) {
  if (lane == 0) bulk_wait_read<0>();  // the previous store of this warp has read the buffer
  __syncwarp();
  uint8_t* rowp = buf + lane * 128;
#pragma unroll
  for (int c = 0; c < 8; ++c)
    *reinterpret_cast<uint4*>(rowp + ((c ^ (lane & 7)) << 4)) =
        make_uint4(words[4 * c], words[4 * c + 1], words[4 * c + 2], words[4 * c + 3]);
  fence_proxy_async_smem();
  __syncwarp();
  if (lane == 0) {
    if (reduce) tma_reduce_add_2d(map, buf, x, y);
    else tma_store_2d(map, buf, x, y);
    bulk_commit();
  }
}

template <int BN, bool kStaged>
__global__ void __launch_bounds__(kGemmThreads, 1)
    k_tc_gemm2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmC, const GemmGeom g, const EpiArgs e, int* status) {
  using Cfg = Gemm2Cfg<BN, kStaged>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + Cfg::kStages * Cfg::kABytes;
  uint8_t* sEpi = smem + Cfg::kStages * Cfg::kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sEpi + Cfg::kEpiBytes);
  uint64_t* empty = full + Cfg::kStages;
  uint64_t* tfull = empty + Cfg::kStages;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int m_pairs = (g.num_m_tiles + 1) >> 1;
  const int num_tiles = m_pairs * g.num_n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&tfull[a], 1);
      mbar_init(&tempty[a], 2 * kEpiWarps);
    }
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) tmem_alloc2(tmem_slot, Cfg::kTmemCols);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------ TMA producer (both CTAs)
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs) {
        const int mp = t / g.num_n_tiles, nt = t % g.num_n_tiles;
        const int mt = 2 * mp + static_cast<int>(rank);  // this CTA's 128-row tile
        const int n0 = nt * BN + static_cast<int>(rank) * (BN / 2);
        int cb = 0, cx = 0, cy = 0;
        if (g.mode == kModeConv) {
          const int per_img = g.tiles_x * g.tiles_y;
          cb = mt / per_img;  // may be == B for the odd tail tile: zero-filled
          const int rem = mt % per_img;
          cy = (rem / g.tiles_x) * g.bh;
          cx = (rem % g.tiles_x) * g.bw;
        }
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, status, kStatusTimeoutEmpty)) { ok = false; break; }
          if (rank == 0) mbar_arrive_expect_tx(&full[stage], 2 * Cfg::kStageBytes);
          const uint32_t fb = mapa_shared(smem_u32(&full[stage]), 0);
          uint8_t* a_dst = sA + stage * Cfg::kABytes;
          uint8_t* b_dst = sB + stage * Cfg::kBBytes;
          if (g.mode == kModeConv) {
            const int tap = kb / g.ic_chunks;
            const int ic0 = (kb % g.ic_chunks) * 64;
            const int dy = tap / g.ksize - g.pad, dx = tap % g.ksize - g.pad;
            tma2_load_4d(a_dst, &tmA, fb, ic0, cx + dx, cy + dy, cb);
            tma2_load_2d(b_dst, &tmB, fb, tap * g.icp + ic0, n0);
          } else {
            tma2_load_2d(a_dst, &tmA, fb, kb * 64, mt * 128);
            tma2_load_2d(b_dst, &tmB, fb, kb * 64, n0);
          }
          if (++stage == Cfg::kStages) { stage = 0; phase ^= 1u; }
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ------------------------------------------------------------ MMA issuer (leader only)
      constexpr uint32_t idesc = umma_idesc_f16(256, BN);
      int stage = 0;
      uint32_t phase = 0;
      int it = 0;
      bool ok = true;
      for (int t = pair; t < num_tiles && ok; t += npairs, ++it) {
        const int acc = it & 1;
        const uint32_t acc_phase = (it >> 1) & 1;
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1u, status, kStatusTimeoutAccumFree)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * Cfg::kAccCols;
        for (int kb = 0; kb < g.num_kb; ++kb) {
          if (!mbar_wait(&full[stage], phase, status, kStatusTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(sA + stage * Cfg::kABytes));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + stage * Cfg::kBBytes));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma2_f16(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb > 0 || k > 0) ? 1u : 0u);
          umma2_commit_mc(&empty[stage], 0x3);
          if (++stage == Cfg::kStages) { stage = 0; phase ^= 1u; }
        }
        if (ok) umma2_commit_mc(&tfull[acc], 0x3);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const int half = (warp - 2) / 4;
    const int c_begin = BN >= 64 ? half * (BN / 2) : (half == 0 ? 0 : BN);
    const int c_end = BN >= 64 ? c_begin + BN / 2 : (half == 0 ? BN : BN);
    const uint32_t tempty_leader0 = mapa_shared(smem_u32(&tempty[0]), 0);
    const uint32_t tempty_leader1 = mapa_shared(smem_u32(&tempty[1]), 0);
    uint8_t* ebuf = sEpi + (warp - 2) * Cfg::kEpiBufBytes;
    float* ebias = reinterpret_cast<float*>(sEpi + kEpiWarps * Cfg::kEpiBufBytes) + (warp - 2) * (BN / 2);
    int it = 0;
    for (int t = pair; t < num_tiles; t += npairs, ++it) {
      const int acc = it & 1;
      const uint32_t acc_phase = (it >> 1) & 1;
      const int mp = t / g.num_n_tiles, nt = t % g.num_n_tiles;
      const int mt = 2 * mp + static_cast<int>(rank);
      int row = -1;
      if (g.mode == kModeConv) {
        const int per_img = g.tiles_x * g.tiles_y;
        const int b = mt / per_img, rem = mt % per_img;
        const int y = (rem / g.tiles_x) * g.bh + r / g.bw;
        const int x = (rem % g.tiles_x) * g.bw + r % g.bw;
        if (b < g.B && y < g.H && x < g.W) row = (b * g.H + y) * g.W + x;
      } else {
        const int m = mt * 128 + r;
        if (m < g.M) row = m;
      }
      // transposed epilogue: this tile's bias slice is fetched before the accumulator
      // wait, so its latency hides behind the MMA
      float4 bq = make_float4(0.f, 0.f, 0.f, 0.f);
      const int bcol = nt * BN + c_begin + 4 * lane;
      if (kStaged && e.tma_store == 3 && e.bias && 4 * lane < c_end - c_begin && bcol < g.N)
        bq = __ldg(reinterpret_cast<const float4*>(e.bias + bcol));
      if (!mbar_wait_warp(&tfull[acc], acc_phase, status, kStatusTimeoutAccum)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + acc * Cfg::kAccCols;
      if (kStaged && e.tma_store == 3) {
        if (4 * lane < c_end - c_begin) *reinterpret_cast<float4*>(ebias + 4 * lane) = bq;
        __syncwarp();
        epi_transposed<BN>(g, e, tbase, c_begin, c_end, nt * BN, row, lane, reinterpret_cast<float*>(ebuf), ebias);
      } else if (kStaged && e.tma_store == 1) {
        // f16 out: 64-column slices -> staging -> TMA store (rows / columns past the
        // tensor are clipped by the TMA unit)
#pragma unroll 1
        for (int c = c_begin; c < c_end; c += 64) {
          uint32_t ra[32], rb[32];
          tmem_ld32(tbase + c, ra);
          tmem_ld32(tbase + c + 32, rb);
          tmem_wait_ld();
          const int n0 = nt * BN + c;
          float v[32], w[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            v[j] = __uint_as_float(ra[j]);
            w[j] = __uint_as_float(rb[j]);
          }
          if (e.bias) {
#pragma unroll
            for (int j0 = 0; j0 < 32; j0 += 8) {
              float bb[8], bc[8];
              load_f8(e.bias + n0 + j0, bb);
              load_f8(e.bias + n0 + 32 + j0, bc);
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                v[j0 + i] += bb[i];
                w[j0 + i] += bc[i];
              }
            }
          }
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            v[j] = apply_act(v[j], e.act);
            w[j] = apply_act(w[j], e.act);
          }
          if (e.q8) {
            q8_roundtrip32(v);
            q8_roundtrip32(w);
          }
          uint32_t words[32];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            __half2 h0 = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
            __half2 h1 = __floats2half2_rn(w[2 * j], w[2 * j + 1]);
            words[j] = *reinterpret_cast<uint32_t*>(&h0);
            words[16 + j] = *reinterpret_cast<uint32_t*>(&h1);
          }
          if (n0 < g.N && mt * 128 + q * 32 < g.M) {  // warp-uniform: no store starts past the tensor
            stage_and_store(ebuf, words, lane, &tmC, n0, mt * 128 + q * 32, false);
          }
        }
      } else if (kStaged && e.tma_store == 2) {
        // f32 residual: delta = scale * (acc + bias), added in place by a TMA reduce
#pragma unroll 1
        for (int c = c_begin; c < c_end; c += 32) {
          uint32_t raw[32];
          tmem_ld32(tbase + c, raw);
          tmem_wait_ld();
          const int n0 = nt * BN + c;
          uint32_t words[32];
#pragma unroll
          for (int j0 = 0; j0 < 32; j0 += 8) {
            float bb[8], sc[8];
            if (e.bias) load_f8(e.bias + n0 + j0, bb);
            else {
#pragma unroll
              for (int i = 0; i < 8; ++i) bb[i] = 0.f;
            }
            if (e.scale) load_f8(e.scale + n0 + j0, sc);
            else {
#pragma unroll
              for (int i = 0; i < 8; ++i) sc[i] = 1.f;
            }
#pragma unroll
            for (int i = 0; i < 8; ++i) words[j0 + i] = __float_as_uint(sc[i] * (__uint_as_float(raw[j0 + i]) + bb[i]));
          }
          if (n0 < g.N && mt * 128 + q * 32 < g.M) {
            stage_and_store(ebuf, words, lane, &tmC, n0, mt * 128 + q * 32, true);
          }
        }
      } else {
#pragma unroll 1
        for (int c = c_begin; c < c_end; c += 32) {
          uint32_t raw[32];
          tmem_ld32(tbase + c, raw);
          tmem_wait_ld();
          if (row >= 0) {
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(raw[j]);
            epilogue32(g, e, row, nt * BN + c, v);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote_relaxed(acc ? tempty_leader1 : tempty_leader0);
    }
    if (kStaged) {
      if (lane == 0) bulk_wait_all();  // every TMA store of this warp has completed
      __syncwarp();
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem_base, Cfg::kTmemCols);
  }
}

// ---------------------------------------------------------------- host side

typedef CUresult (*PFN_tmapEncodeTiled)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                        const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                        CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                        CUtensorMapFloatOOBfill);

static PFN_tmapEncodeTiled tmap_encoder() {
  static PFN_tmapEncodeTiled fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_tmapEncodeTiled>(p);
  }
  return fn;
}

// 2-D f16 tensor map over a row-major [rows][cols] matrix with leading dimension ld
// (elements), box = 64 columns x box_rows rows, 128B swizzle, zero fill out of range.
int make_tmap_2d(CUtensorMap* map, const void* ptr, int rows, int cols, int ld, int box_rows) {
  PFN_tmapEncodeTiled enc = tmap_encoder();
  if (!enc) return -1;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (ld * 2) % 16 || box_rows > 256 || box_rows < 1) return -2;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

// 2-D tensor map of any element type over a row-major [rows][cols] matrix (ld elements
// between rows), box = box_cols x box_rows, the given swizzle, zero fill out of range.
int make_tmap_2d_typed(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes, int rows,
                       int cols, int ld, int box_cols, int box_rows, CUtensorMapSwizzle swz) {
  PFN_tmapEncodeTiled enc = tmap_encoder();
  if (!enc) return -1;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (static_cast<long>(ld) * elem_bytes) % 16 || box_rows > 256 ||
      box_rows < 1 || box_cols > 256 || box_cols < 1 || (box_cols * elem_bytes) % 16)
    return -2;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * elem_bytes};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(box_cols), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, dtype, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

// 4-D f16 tensor map over an NHWC tensor [B][H][W][C] (row pitch C), box =
// 64 channels x bw x bh x 1, 128B swizzle, zero fill out of range (conv padding).
int make_tmap_nhwc(CUtensorMap* map, const void* ptr, int B, int H, int W, int C, int bw, int bh) {
  PFN_tmapEncodeTiled enc = tmap_encoder();
  if (!enc) return -1;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || (C * 2) % 16) return -2;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(C), static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(C) * 2, static_cast<cuuint64_t>(C) * 2 * W,
                           static_cast<cuuint64_t>(C) * 2 * W * H};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(bw), static_cast<cuuint32_t>(bh), 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

// 5-D f16 tensor map over an NHWC tensor [B][H][W][C] (C % 64 == 0) whose box lands
// channel-chunk-major: dims (8 channels, W, H, C/8 chunks, B), box = 8 channels x bw x
// bh x 8 chunks x 1, no swizzle, zero fill out of range. In shared memory a box is
// [chunk][y][x][8 halves]: the K-major no-swizzle MMA operand layout with one 16-byte
// core-matrix row per pixel, so a shifted pixel window is a shifted descriptor start.
int make_tmap_nhwc_planes(CUtensorMap* map, const void* ptr, int B, int H, int W, int C, int bw, int bh) {
  PFN_tmapEncodeTiled enc = tmap_encoder();
  if (!enc) return -1;
  if ((reinterpret_cast<uintptr_t>(ptr) & 15) || C % 64 || bw < 1 || bw > 256 || bh < 1 || bh > 256) return -2;
  cuuint64_t dims[5] = {8, static_cast<cuuint64_t>(W), static_cast<cuuint64_t>(H), static_cast<cuuint64_t>(C / 8),
                        static_cast<cuuint64_t>(B)};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(C) * 2, static_cast<cuuint64_t>(C) * 2 * W, 16,
                           static_cast<cuuint64_t>(C) * 2 * W * H};
  cuuint32_t box[5] = {8, static_cast<cuuint32_t>(bw), static_cast<cuuint32_t>(bh), 8, 1};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 5, const_cast<void*>(ptr), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : -3;
}

static int g_num_sms = 0;
static int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

// kQ8: tb maps the planar Q8_0 int8 plane and ts its scale plane; otherwise ts is unused.
template <int BN, bool kQ8>
static int launch_bn(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& ts, const GemmGeom& g,
                     const EpiArgs& e, int* status, cudaStream_t stream, int max_ctas) {
  using Cfg = GemmCfg<BN, kQ8>;
  static std::atomic<uint64_t> attr_set{0};  // one bit per device; first calls may race
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((attr_set.load() >> (dev & 63)) & 1)) {
    if (cudaFuncSetAttribute(k_tc_gemm<BN, kQ8>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) !=
        cudaSuccess)
      return -10;
    attr_set.fetch_or(uint64_t(1) << (dev & 63));
  }
  const int tiles = g.num_m_tiles * g.num_n_tiles;
  if (g.ksplit > 1) {
    // one tile per cluster of g.ksplit CTAs
    cudaLaunchConfig_t cfg;
    memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(static_cast<unsigned>(tiles * g.ksplit), 1, 1);
    cfg.blockDim = dim3(kQ8 ? kGemmThreadsQ8 : kGemmThreads, 1, 1);
    cfg.dynamicSmemBytes = Cfg::kSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(g.ksplit);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, k_tc_gemm<BN, kQ8>, ta, tb, ts, g, e, status) != cudaSuccess) return -11;
    return cudaGetLastError() == cudaSuccess ? 0 : -11;
  }
  int grid = num_sms();
  if (max_ctas > 0 && max_ctas < grid) grid = max_ctas;
  if (tiles < grid) grid = tiles;
  if (grid <= 0) return 0;
  k_tc_gemm<BN, kQ8><<<grid, kQ8 ? kGemmThreadsQ8 : kGemmThreads, Cfg::kSmemBytes, stream>>>(ta, tb, ts, g, e, status);
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

template <int BN, bool kStaged>
static int launch_bn2(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmGeom& g,
                      const EpiArgs& e, int* status, cudaStream_t stream) {
  using Cfg = Gemm2Cfg<BN, kStaged>;
  static std::atomic<uint64_t> attr_set{0};  // one bit per device; first calls may race
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((attr_set.load() >> (dev & 63)) & 1)) {
    if (cudaFuncSetAttribute(k_tc_gemm2<BN, kStaged>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmemBytes) !=
        cudaSuccess)
      return -10;
    attr_set.fetch_or(uint64_t(1) << (dev & 63));
  }
  const int tiles = ((g.num_m_tiles + 1) / 2) * g.num_n_tiles;
  int pairs = num_sms() / 2;
  if (tiles < pairs) pairs = tiles;
  if (pairs <= 0) return 0;
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, k_tc_gemm2<BN, kStaged>, ta, tb, tc, g, e, status) != cudaSuccess) return -11;
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

// 1 = use the 2-SM kernel for problems with enough 256-row tiles (default);
// the environment variable DA3B_GEMM_2SM=0 keeps every launch on the 1-SM kernel.
static int use_2sm() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("DA3B_GEMM_2SM");
    v = (s && s[0] == '0') ? 0 : 1;
  }
  return v;
}

// 2-SM launch (B tensor map box of bn/2 rows). BN in {64, 128, 256}.
static int gemm_launch2(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& tc, const GemmGeom& g,
                        const EpiArgs& e, int* status, cudaStream_t stream) {
  if (e.tma_store) {
    switch (bn) {
      case 64: return launch_bn2<64, true>(ta, tb, tc, g, e, status, stream);
      case 128: return launch_bn2<128, true>(ta, tb, tc, g, e, status, stream);
      case 256: return launch_bn2<256, true>(ta, tb, tc, g, e, status, stream);
      default: return -12;
    }
  }
  switch (bn) {
    case 64: return launch_bn2<64, false>(ta, tb, tc, g, e, status, stream);
    case 128: return launch_bn2<128, false>(ta, tb, tc, g, e, status, stream);
    case 256: return launch_bn2<256, false>(ta, tb, tc, g, e, status, stream);
    default: return -12;
  }
}

typedef CUresult (*PFN_tmapEncodeTiled2)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                         const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                         CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                         CUtensorMapFloatOOBfill);

// Output map of a TMA-store epilogue: row-major [rows][cols] of f16 (box 64 x 32) or
// f32 (box 32 x 32), 128-byte swizzle. Returns false when the layout does not qualify.
static bool make_out_map(CUtensorMap* map, void* ptr, bool f32, int rows, int cols, int ld) {
  PFN_tmapEncodeTiled enc = tmap_encoder();
  const int eb = f32 ? 4 : 2;
  if (!enc || (reinterpret_cast<uintptr_t>(ptr) & 15) || (static_cast<long>(ld) * eb) % 16) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * eb};
  cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / eb), 32};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ptr, dims, strides, box,
             estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// The 2-SM kernel pays off once every CTA pair gets at least one 256-row tile.
// Epilogue of the 2-SM kernel for f16 outputs: 0 (default) = transposed epilogue with
// coalesced stores; 1 = the earlier selection (GELU via staged TMA store, others direct
// per-row stores). DA3B_GEMM_EPI=1 selects the latter, for A/B timing.
static int epi_mode_override() {
  static int v = -1;
  if (v < 0) {
    const char* s = getenv("DA3B_GEMM_EPI");
    v = (s && s[0] == '1') ? 1 : 0;
  }
  return v;
}

static bool want_2sm(const GemmGeom& g, int bn) {
  return use_2sm() && bn >= 64 && ((g.num_m_tiles + 1) / 2) * g.num_n_tiles >= num_sms() / 2;
}

// Launch with a validated geometry. BN in {32, 64, 128, 256}.
int gemm_launch(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmGeom& g, const EpiArgs& e,
                int* status, cudaStream_t stream, int max_ctas) {
  CUtensorMap unused;
  memset(&unused, 0, sizeof(unused));
  switch (bn) {
    case 32: return launch_bn<32, false>(ta, tb, unused, g, e, status, stream, max_ctas);
    case 64: return launch_bn<64, false>(ta, tb, unused, g, e, status, stream, max_ctas);
    case 128: return launch_bn<128, false>(ta, tb, unused, g, e, status, stream, max_ctas);
    case 256: return launch_bn<256, false>(ta, tb, unused, g, e, status, stream, max_ctas);
    default: return -12;
  }
}

EpiArgs epi_default() {
  EpiArgs e;
  memset(&e, 0, sizeof(e));
  e.kind = kEpiF16;
  e.o2_ln_eps = 1e-5f;
  e.o2_scale = 1.0f;
  return e;
}

int pick_bn(int N) {
  if (N <= 32) return 32;
  if (N <= 64) return 64;
  if (N <= 128) return 128;
  return 256;
}

static int check_epi(const EpiArgs& e, int N) {
  if ((reinterpret_cast<uintptr_t>(e.bias) & 15) || (reinterpret_cast<uintptr_t>(e.scale) & 15)) return -19;
  if (e.kind == kEpiF16 || e.kind == kEpiConvT) {
    if (N % 8 || !e.out || e.ld_out % 8 || (reinterpret_cast<uintptr_t>(e.out) & 15)) return -20;
    if (e.out_relu && (reinterpret_cast<uintptr_t>(e.out_relu) & 15)) return -21;
    if (e.res1 && (e.ld_res1 % 8 || (reinterpret_cast<uintptr_t>(e.res1) & 15))) return -22;
    if (e.res2 && (e.ld_res2 % 8 || (reinterpret_cast<uintptr_t>(e.res2) & 15))) return -23;
    if (e.q8 && (N % 32 || e.res1 || e.res2 || e.out_relu || e.kind != kEpiF16)) return -29;
  }
  if (e.kind == kEpiResid || e.kind == kEpiTokens) {
    if (N % 8 || !e.resid || e.ld_resid % 4 || (reinterpret_cast<uintptr_t>(e.resid) & 15)) return -24;
    if (e.kind == kEpiTokens && (!e.pos || !e.bias || e.rm_div <= 0)) return -25;
  }
  if (e.kind == kEpiConvT && (e.ct_oc % 8 || e.ct_s <= 0 || e.ct_hin <= 0 || e.ct_win <= 0)) return -26;
  if (e.kind == kEpiQKV && (!e.out || !e.vt || e.ld_out % 8 || N != 3 * e.vt_d || e.vt_d % 64 || e.vt_seqlen <= 0 ||
                            e.vt_ld < e.vt_seqlen || e.vt_ld % 8))
    return -18;
  if (e.kind == kEpiOut2) {
    if (N != 32 || e.o2_dim < 1 || e.o2_dim > 8 || !e.o2_w || !e.o2_b) return -27;
    for (int i = 0; i < e.o2_dim; ++i)
      if (!e.o2_out[i]) return -28;
  }
  return 0;
}

// Few rows (one image: M = 1370): with too few CTA-pair tiles for the SMs the GEMM runs
// on one-CTA tiles, narrowed until they outnumber the SMs or are 64 wide. The K split's
// few-tile rule starts from this width; otherwise the fitted model below picks the tiles.
static int narrow_1sm_bn(int m_tiles, int N, int bn) {
  while (bn > 64 && static_cast<long>(m_tiles) * ((N + bn - 1) / bn) < num_sms()) bn /= 2;
  return bn;
}

// $DA3B_GEMM_KSPLIT=0 (read once per process) keeps every 1-SM launch at one CTA per tile.
static bool ksplit_enabled() {
  static const bool on = [] {
    const char* s = getenv("DA3B_GEMM_KSPLIT");
    return !(s && s[0] == '0');
  }();
  return on;
}

// K split of the 1-SM kernel: when the tiles fill at most half the SMs and the reduction
// is long, a cluster of up to 4 CTAs takes each tile, each at least 8 k-blocks, and the
// first sums the others' partial accumulators (one image's stride-2 conv: 36 tiles of
// 108 k-blocks).
static int pick_ksplit(long tiles, int num_kb, int bn) {
  if (bn < 64 || tiles <= 0 || !ksplit_enabled()) return 1;
  const int sms = num_sms();
  if (tiles * 2 > sms) return 1;
  long ks = std::min<long>(4, sms / tiles);
  ks = std::min<long>(ks, num_kb / 8);
  return ks >= 2 ? static_cast<int>(ks) : 1;
}

// Tile width and K split of a linear on the 1-SM kernel: the candidates (64, 1),
// (128, 1), (256, 1) and, with at least 32 k-blocks, (128, 2), scored by a model fitted
// to B200 measurements at a few images' rows, where each SM's operand stream (its TMA
// ring against the latency of L2 reads) bounds these GEMMs: waves x the larger of a
// CTA's operand bytes at 75 GB/s and its MMA time, against all operand bytes at 7.5
// TB/s, plus about 2.9 us for summing a 128 x 128 f32 share. The rates are fitted to
// timings, not hardware limits (ncu at fc2's shape: L2 throughput 17%, tensor pipe 14%). One ViT-B image: QKV (N = 2304) 256-wide tiles 10.4 us against 13.2 for 128 (198
// tiles are two waves), fc1 + GELU 13.6 against 15.2, proj 64-wide 8.1 against 10.2 for
// 256; fc2 (K = 3072) (128, 2) 16.7 against 20.4 for (64, 1); ViT-L fc2 (K = 4096) (128,
// 1) 27.1 against 44.3; two ViT-B images' fc2 (128, 1) 22.9 against 35.2.
static void model_1sm_tile(int m_tiles, int N, int num_kb, int* bn_out, int* ks_out) {
  const int cand[4][2] = {{64, 1}, {128, 1}, {256, 1}, {128, 2}};
  const double sms = num_sms();
  double best = 1e30;
  for (const auto& c : cand) {
    const int bn = c[0], ks = c[1];
    if (ks > 1 && (num_kb < 32 || !ksplit_enabled())) continue;
    const double ctas = static_cast<double>(m_tiles) * ((N + bn - 1) / bn) * ks;
    const double waves = std::ceil(ctas / sms);
    const double kbs = static_cast<double>(num_kb / ks);
    const double cta_bytes = kbs * (16384.0 + 128.0 * bn);
    const double mma = kbs * 4 * (bn >= 256 ? 128 : 64) / 1.9e9;
    double t = std::max(waves * std::max(cta_bytes / 75e9, mma), ctas * cta_bytes / 7.5e12);
    if (ks > 1) t += 2.9e-6 * (bn / 128.0) * (ks - 1);
    if (t < best * 0.98) {
      best = t;
      *bn_out = bn;
      *ks_out = ks;
    }
  }
}

// The automatic tiles of a linear (f16 or fused-Q8_0 weights, not the out2 stage):
// false for the CTA-pair kernel (bn = its tile width), true for the 1-SM kernel with
// tile width bn and K split ks.
static bool auto_linear_tile(int M, int N, int K, int* bn_out, int* ks_out) {
  GemmGeom g;
  memset(&g, 0, sizeof(g));
  g.num_kb = (K + 63) / 64;
  g.num_m_tiles = (M + 127) / 128;
  int bn = pick_bn(N);
  g.num_n_tiles = (N + bn - 1) / bn;
  *ks_out = 1;
  if (want_2sm(g, bn)) {
    *bn_out = bn;
    return false;
  }
  // few tiles with a long reduction: the narrowest tiles and the cluster K split
  // (measured on one image's stride-2 conv); otherwise the fitted model
  bn = narrow_1sm_bn(g.num_m_tiles, N, bn);
  int ks = pick_ksplit(static_cast<long>(g.num_m_tiles) * ((N + bn - 1) / bn), g.num_kb, bn);
  if (ks <= 1) model_1sm_tile(g.num_m_tiles, N, g.num_kb, &bn, &ks);
  *bn_out = bn;
  *ks_out = ks;
  return true;
}

int gemm_linear(const __half* A, int M, int K, int lda, const __half* W, int N, int ldw, int bn, const EpiArgs& e,
                int* status, cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return M == 0 ? 0 : -30;
  if (lda < K || ldw < K || lda % 8 || ldw % 8) return -31;
  const bool auto_bn = bn <= 0;
  if (auto_bn) bn = pick_bn(N);
  if (e.kind == kEpiOut2) bn = 32;
  int rc = check_epi(e, N);
  if (rc) return rc;
  GemmGeom g;
  memset(&g, 0, sizeof(g));
  g.mode = kModeLinear;
  g.M = M;
  g.N = N;
  g.K = K;
  g.num_kb = (K + 63) / 64;
  g.num_m_tiles = (M + 127) / 128;
  g.num_n_tiles = (N + bn - 1) / bn;
  bool two = want_2sm(g, bn);
  if (e.kind != kEpiOut2) {
    if (auto_bn) {
      int ks = 1;
      two = !auto_linear_tile(M, N, K, &bn, &ks);
      g.ksplit = ks;
    } else if (!two) {
      g.ksplit = pick_ksplit(static_cast<long>(g.num_m_tiles) * g.num_n_tiles, g.num_kb, bn);
    }
    g.num_n_tiles = (N + bn - 1) / bn;
  }
  CUtensorMap ta, tb, tc;
  if ((rc = make_tmap_2d(&ta, A, M, K, lda, 128))) return rc - 100;
  if ((rc = make_tmap_2d(&tb, W, N, K, ldw, two ? bn / 2 : bn))) return rc - 200;
  if (!two) return gemm_launch(bn, ta, tb, g, e, status, stream, 0);
  EpiArgs e2 = e;
  e2.tma_store = 0;
  memset(&tc, 0, sizeof(tc));
  // Measured on B200 (C3 shapes): the staged TMA store wins for the GELU epilogue and
  // the TMA reduce-add for residual updates; plain f16 outputs are faster stored directly.
  const int epi_mode = epi_mode_override();
  if ((e.kind == kEpiF16 && !e.q8) || e.kind == kEpiQKV) {
    if (epi_mode != 1) e2.tma_store = 3;
    else if (bn >= 128 && e.rm_div == 0 && e.kind == kEpiF16 && (e.act == kActGelu || e.act == kActGeluR) &&
             !e.res1 && !e.res2 &&
             !e.out_relu && make_out_map(&tc, e.out, false, M, N, e.ld_out))
      e2.tma_store = 1;
  } else if (bn >= 128 && e.rm_div == 0 && e.kind == kEpiResid &&
             make_out_map(&tc, e.resid, true, M, N, e.ld_resid)) {
    e2.tma_store = 2;
  }
  return gemm_launch2(bn, ta, tb, tc, g, e2, status, stream);
}

// Tile width the planar Q8_0 GEMM (k_tc_gemm<BN, true>) takes for an M x N linear, or 0
// when the problem is one for the CTA-pair kernel (many rows), whose weights are then
// better dequantised once per ViT block into f16 than once per 256-row tile pair.
int gemm_linear_tiles(int M, int N, int K, int* bn, int* ksplit) {
  if (M <= 0 || N <= 0 || K <= 0 || !bn || !ksplit) return -1;
  return auto_linear_tile(M, N, K, bn, ksplit) ? 1 : 0;
}

int gemm_q8p_bn(int M, int N, int K) {
  if (M <= 0 || N <= 0 || K <= 0 || N % 8) return 0;
  int bn = 0, ks = 1;
  if (!auto_linear_tile(M, N, K, &bn, &ks)) return 0;  // CTA pairs
  // the same tiles as the f16 route (so the two give the same bits); no K split there
  return ks == 1 && (bn == 64 || bn == 128) ? bn : 0;
}

int gemm_linear_q8p(const __half* A, int M, int K, int lda, const uint8_t* Wq, int N, const EpiArgs& e, int* status,
                    cudaStream_t stream) {
  if (M <= 0 || N <= 0 || K <= 0) return M == 0 ? 0 : -30;
  if (lda < K || lda % 8 || K % 32 || N % 8 || (reinterpret_cast<uintptr_t>(Wq) & 15) || e.kind == kEpiOut2)
    return -31;
  const int bn = gemm_q8p_bn(M, N, K);
  if (!bn) return 1;
  int rc = check_epi(e, N);
  if (rc) return rc;
  GemmGeom g;
  memset(&g, 0, sizeof(g));
  g.mode = kModeLinear;
  g.M = M;
  g.N = N;
  g.K = K;
  g.num_kb = (K + 63) / 64;
  g.num_m_tiles = (M + 127) / 128;
  g.num_n_tiles = (N + bn - 1) / bn;
  CUtensorMap ta, tq, ts;
  if ((rc = make_tmap_2d(&ta, A, M, K, lda, 128))) return rc - 100;
  if ((rc = make_tmap_2d_typed(&tq, Wq, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K, K, 64, bn, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc - 200;
  if ((rc = make_tmap_2d_typed(&ts, Wq + static_cast<size_t>(N) * K, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, K / 32, N, N,
                               bn, 2, CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc - 300;
  return bn == 64 ? launch_bn<64, true>(ta, tq, ts, g, e, status, stream, 0)
                  : launch_bn<128, true>(ta, tq, ts, g, e, status, stream, 0);
}

// Pixel block of one 128-row M tile: the (bw, bh) with bw * bh == 128 that wastes
// the fewest padded pixels on an H x W map.
static void pick_block(int H, int W, int* bw, int* bh) {
  static const int cand[6][2] = {{16, 8}, {8, 16}, {32, 4}, {4, 32}, {64, 2}, {128, 1}};
  long best = -1;
  for (auto& c : cand) {
    const long cover = static_cast<long>((W + c[0] - 1) / c[0]) * c[0] * ((H + c[1] - 1) / c[1]) * c[1];
    if (best < 0 || cover < best) {
      best = cover;
      *bw = c[0];
      *bh = c[1];
    }
  }
}

int conv_nhwc(const __half* X, int B, int H, int W, int IC, const __half* Wp, int OC, int ksize, int bn,
              const EpiArgs& e, int* status, cudaStream_t stream) {
  if (B <= 0 || H <= 0 || W <= 0 || IC <= 0 || OC <= 0 || (ksize != 1 && ksize != 3)) return -40;
  if (IC % 8) return -41;
  if (bn <= 0) bn = pick_bn(OC);
  if (e.kind == kEpiOut2) bn = 32;
  int rc = check_epi(e, OC);
  if (rc) return rc;
  if (ksize == 3) {
    // The halo-box kernel reads each input pixel once per 64-channel chunk instead of
    // once per tap: 128 output channels (one CTA), or groups of 256 (CTA pairs).
    // $DA3B_CONV_HALO=0 never takes it, =1 also for other multiples of 128.
    const char* ev = getenv("DA3B_CONV_HALO");
    const int mode = ev && ev[0] == '0' ? 0 : (ev && ev[0] == '1' ? 2 : 1);
    if (mode == 2 || (mode == 1 && (OC == 64 || OC == 128 || OC % 256 == 0))) {
      rc = conv3_halo(X, B, H, W, IC, Wp, OC, e, status, stream);
      if (rc != 1) return rc;
    }
  }
  int bw = 16, bh = 8;
  pick_block(H, W, &bw, &bh);
  const int icp = conv_icp(IC);
  GemmGeom g;
  memset(&g, 0, sizeof(g));
  g.mode = kModeConv;
  g.M = B * H * W;
  g.N = OC;
  g.K = IC;
  g.ic_chunks = icp / 64;
  g.icp = icp;
  g.ksize = ksize;
  g.pad = ksize / 2;
  g.num_kb = ksize * ksize * g.ic_chunks;
  g.B = B;
  g.H = H;
  g.W = W;
  g.bw = bw;
  g.bh = bh;
  g.tiles_x = (W + bw - 1) / bw;
  g.tiles_y = (H + bh - 1) / bh;
  g.num_m_tiles = B * g.tiles_x * g.tiles_y;
  g.num_n_tiles = (OC + bn - 1) / bn;
  const bool two = want_2sm(g, bn);
  if (!two && e.kind != kEpiOut2) g.ksplit = pick_ksplit(static_cast<long>(g.num_m_tiles) * g.num_n_tiles, g.num_kb, bn);
  CUtensorMap ta, tb, tc;
  if ((rc = make_tmap_nhwc(&ta, X, B, H, W, IC, bw, bh))) return rc - 100;
  if ((rc = make_tmap_2d(&tb, Wp, OC, ksize * ksize * icp, ksize * ksize * icp, two ? bn / 2 : bn))) return rc - 200;
  if (!two) return gemm_launch(bn, ta, tb, g, e, status, stream, 0);
  memset(&tc, 0, sizeof(tc));
  EpiArgs e2 = e;
  e2.tma_store = (e.kind == kEpiF16 && !e.q8 && epi_mode_override() != 1) ? 3 : 0;
  return gemm_launch2(bn, ta, tb, tc, g, e2, status, stream);
}

}  // namespace da3b
