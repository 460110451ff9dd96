// Memory-bound kernels of the depth path (coalesced, vectorised, one pass each).
#include <atomic>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "kernels.h"
#include "q8planar.cuh"

namespace da3b {

static inline unsigned grid_for(long n, int threads, long cap = 1L << 20) {
  long b = (n + threads - 1) / threads;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return static_cast<unsigned>(b);
}

// x[b*ntok + 0][:] = cls + pos[0]  (token 0 of every image; src/dino_backbone.cpp:123-126)
__global__ void k_cls_rows(float* __restrict__ x, int B, int ntok, int D, const float* __restrict__ cls,
                           const float* __restrict__ pos) {
  const long total = static_cast<long>(B) * D;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int b = static_cast<int>(i / D), e = static_cast<int>(i % D);
    x[static_cast<size_t>(b) * ntok * D + e] = cls[e] + pos[e];
  }
}
int cls_rows(float* x, int B, int ntok, int D, const float* cls, const float* pos, cudaStream_t s) {
  k_cls_rows<<<grid_for(static_cast<long>(B) * D, 256), 256, 0, s>>>(x, B, ntok, D, cls, pos);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Token 0 of every view := camera_token[slot] with slot 0 for the first view of
// each scene and slot 1 for the others (src/dino_backbone.cpp:533-546).
__global__ void k_cam_rows(float* __restrict__ x, int nviews_total, int views_per_scene, int ntok, int D,
                           const float* __restrict__ cam) {
  const long total = static_cast<long>(nviews_total) * D;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int v = static_cast<int>(i / D), e = static_cast<int>(i % D);
    const int slot = (v % views_per_scene) == 0 ? 0 : 1;
    x[static_cast<size_t>(v) * ntok * D + e] = cam[slot * D + e];
  }
}
int cam_rows(float* x, int nviews_total, int views_per_scene, int ntok, int D, const float* cam, cudaStream_t s) {
  k_cam_rows<<<grid_for(static_cast<long>(nviews_total) * D, 256), 256, 0, s>>>(x, nviews_total, views_per_scene,
                                                                                ntok, D, cam);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ---------------------------------------------------------------- LayerNorm
// One warp per output row; VPL = D / 32 values per lane held in registers.
// Two-pass mean / variance in f32, y = (x - mean) * rsqrt(var + eps) * g + b
// (ggml_norm + mul + add, src/ggml_extend.hpp:12-17).
template <typename Tin, int VPL>
__global__ void k_layernorm(const Tin* __restrict__ in, int ld_in, int rows, int D, const float* __restrict__ g,
                            const float* __restrict__ bta, float eps, __half* __restrict__ out, int ld_out, int col_off,
                            int rm_div, int rm_mul, int rm_add, int q8) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int in_row = rm_div > 0 ? (warp / rm_div) * rm_mul + rm_add + warp % rm_div : warp;
  const Tin* src = in + static_cast<size_t>(in_row) * ld_in;
  float v[VPL];
  // element j of lane: index = (j / 4) * 128 + lane * 4 + (j % 4)   (vectors of 4)
#pragma unroll
  for (int j = 0; j < VPL; j += 4) {
    const int idx = (j / 4) * 128 + lane * 4;
    if (sizeof(Tin) == 4) {
      const float4 f = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + idx);
      v[j] = f.x; v[j + 1] = f.y; v[j + 2] = f.z; v[j + 3] = f.w;
    } else {
      const uint2 u = *reinterpret_cast<const uint2*>(reinterpret_cast<const __half*>(src) + idx);
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
      v[j] = a.x; v[j + 1] = a.y; v[j + 2] = b.x; v[j + 3] = b.y;
    }
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) s += v[j];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / D;
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const float d = v[j] - mean;
    q += d * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q / D + eps);
  __half* dst = out + static_cast<size_t>(warp) * ld_out + col_off;
#pragma unroll
  for (int j = 0; j < VPL; j += 4) {
    const int idx = (j / 4) * 128 + lane * 4;
    float r[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) r[i] = (v[j + i] - mean) * rstd * __ldg(g + idx + i) + (bta ? __ldg(bta + idx + i) : 0.f);
    if (q8) {
      // Q8_0 round trip over the 32-element block held by 8 consecutive lanes
      // (ggml quantize_row_q8_0_ref semantics, as in the GEMM epilogue).
      float amax = fmaxf(fmaxf(fabsf(r[0]), fabsf(r[1])), fmaxf(fabsf(r[2]), fabsf(r[3])));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 4));
      const float d = amax / 127.0f;
      const float id = d != 0.f ? 1.0f / d : 0.0f;
      const float dh = __half2float(__float2half_rn(d));
#pragma unroll
      for (int i = 0; i < 4; ++i) r[i] = dh * roundf(r[i] * id);
    }
    uint2 u;
    *reinterpret_cast<__half2*>(&u.x) = __floats2half2_rn(r[0], r[1]);
    *reinterpret_cast<__half2*>(&u.y) = __floats2half2_rn(r[2], r[3]);
    *reinterpret_cast<uint2*>(dst + idx) = u;
  }
}

// Same LayerNorm with 8 consecutive elements per lane (element e -> lane (e / 8) % 32,
// slot (e / 256) * 8 + e % 8): 32-byte f32 / 16-byte f16 loads, gamma and beta as
// float4 pairs, one 16-byte store per 8 outputs. For D a multiple of 256.
template <typename Tin, int VPL>
__device__ __forceinline__ void ln8_row(int warp, const Tin* __restrict__ in, int ld_in, int rows, int D,
                                        const float* __restrict__ g, const float* __restrict__ bta, float eps,
                                        __half* __restrict__ out, int ld_out, int col_off, int rm_div, int rm_mul,
                                        int rm_add, int q8) {
  const int lane = threadIdx.x & 31;
  if (warp >= rows) return;
  const int in_row = rm_div > 0 ? (warp / rm_div) * rm_mul + rm_add + warp % rm_div : warp;
  const Tin* src = in + static_cast<size_t>(in_row) * ld_in;
  float v[VPL];
#pragma unroll
  for (int j = 0; j < VPL; j += 8) {
    const int idx = (j / 8) * 256 + lane * 8;
    if (sizeof(Tin) == 4) {
      const float4 f0 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + idx);
      const float4 f1 = *reinterpret_cast<const float4*>(reinterpret_cast<const float*>(src) + idx + 4);
      v[j] = f0.x; v[j + 1] = f0.y; v[j + 2] = f0.z; v[j + 3] = f0.w;
      v[j + 4] = f1.x; v[j + 5] = f1.y; v[j + 6] = f1.z; v[j + 7] = f1.w;
    } else {
      const uint4 u = *reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(src) + idx);
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const float2 f = __half22float2(h[k]);
        v[j + 2 * k] = f.x;
        v[j + 2 * k + 1] = f.y;
      }
    }
  }
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) s += v[j];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / D;
  float q = 0.f;
#pragma unroll
  for (int j = 0; j < VPL; ++j) {
    const float d = v[j] - mean;
    q += d * d;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
  const float rstd = rsqrtf(q / D + eps);
  __half* dst = out + static_cast<size_t>(warp) * ld_out + col_off;
#pragma unroll
  for (int j = 0; j < VPL; j += 8) {
    const int idx = (j / 8) * 256 + lane * 8;
    const float4 g0 = __ldg(reinterpret_cast<const float4*>(g + idx));
    const float4 g1 = __ldg(reinterpret_cast<const float4*>(g + idx + 4));
    float4 b0 = make_float4(0.f, 0.f, 0.f, 0.f), b1 = b0;
    if (bta) {
      b0 = __ldg(reinterpret_cast<const float4*>(bta + idx));
      b1 = __ldg(reinterpret_cast<const float4*>(bta + idx + 4));
    }
    const float gg[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
    const float bb[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
    float r[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) r[i] = (v[j + i] - mean) * rstd * gg[i] + bb[i];
    if (q8) {
      // Q8_0 round trip over the 32-element block held by 4 consecutive lanes
      float amax = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) amax = fmaxf(amax, fabsf(r[i]));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
      amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
      const float d = amax / 127.0f;
      const float id = d != 0.f ? 1.0f / d : 0.0f;
      const float dh = __half2float(__float2half_rn(d));
#pragma unroll
      for (int i = 0; i < 8; ++i) r[i] = dh * roundf(r[i] * id);
    }
    uint4 u;
    __half2* hu = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int k = 0; k < 4; ++k) hu[k] = __floats2half2_rn(r[2 * k], r[2 * k + 1]);
    *reinterpret_cast<uint4*>(dst + idx) = u;
  }
}

template <typename Tin, int VPL>
__global__ void k_layernorm8(const Tin* __restrict__ in, int ld_in, int rows, int D, const float* __restrict__ g,
                             const float* __restrict__ bta, float eps, __half* __restrict__ out, int ld_out,
                             int col_off, int rm_div, int rm_mul, int rm_add, int q8) {
  ln8_row<Tin, VPL>((blockIdx.x * blockDim.x + threadIdx.x) >> 5, in, ld_in, rows, D, g, bta, eps, out, ld_out,
                    col_off, rm_div, rm_mul, rm_add, q8);
}

// The same LayerNorm in blocks [0, ln_blocks) and the staging dequantisation of a ViT
// block's planar Q8_0 linears in the blocks after: two independent memory-bound passes
// that each take a few microseconds at one image, in one launch.
template <int VPL>
__global__ void k_layernorm8_dq(const float* __restrict__ in, int ld_in, int rows, int D, const float* __restrict__ g,
                                const float* __restrict__ bta, float eps, __half* __restrict__ out, int ld_out,
                                int col_off, int rm_div, int rm_mul, int rm_add, int q8, const Q8Segs dq,
                                unsigned ln_blocks) {
  if (blockIdx.x < ln_blocks) {
    ln8_row<float, VPL>((blockIdx.x * blockDim.x + threadIdx.x) >> 5, in, ld_in, rows, D, g, bta, eps, out, ld_out,
                        col_off, rm_div, rm_mul, rm_add, q8);
  } else {
    q8p_segs_dequant(dq, static_cast<long>(blockIdx.x - ln_blocks) * blockDim.x + threadIdx.x,
                     static_cast<long>(gridDim.x - ln_blocks) * blockDim.x);
  }
}

template <typename Tin>
static int ln_dispatch(const Tin* in, int ld_in, int rows, int D, const float* g, const float* b, float eps,
                       __half* out, int ld_out, int col_off, int rm_div, int rm_mul, int rm_add, int q8,
                       cudaStream_t s, const Q8Segs* dq = nullptr) {
  if (rows <= 0) return dq ? dequant_q8p_segs(*dq, s) : 0;
  const unsigned blocks = static_cast<unsigned>((static_cast<long>(rows) * 32 + 255) / 256);
  const bool wide = D % 256 == 0 && D <= 2048 && ld_in % 8 == 0 && ld_out % 8 == 0 && col_off % 8 == 0 &&
                    (reinterpret_cast<uintptr_t>(in) & 31) == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 &&
                    (reinterpret_cast<uintptr_t>(g) & 15) == 0 && (reinterpret_cast<uintptr_t>(b) & 15) == 0;
  if (wide && dq && sizeof(Tin) == 4) {
    for (int k = 0; k < dq->n; ++k)
      if (reinterpret_cast<uintptr_t>(dq->s[k].q8) & 15 || reinterpret_cast<uintptr_t>(dq->s[k].out) & 15) return -3;
    const unsigned total = blocks + static_cast<unsigned>(q8p_segs_blocks(*dq));
    const float* fin = reinterpret_cast<const float*>(in);
#define DA3B_LN8DQ(VPL)                                                                                           \
  k_layernorm8_dq<VPL><<<total, 256, 0, s>>>(fin, ld_in, rows, D, g, b, eps, out, ld_out, col_off, rm_div, rm_mul, \
                                            rm_add, q8, *dq, blocks)
    switch (D) {
      case 256: DA3B_LN8DQ(8); break;
      case 512: DA3B_LN8DQ(16); break;
      case 768: DA3B_LN8DQ(24); break;
      case 1024: DA3B_LN8DQ(32); break;
      case 1536: DA3B_LN8DQ(48); break;
      case 2048: DA3B_LN8DQ(64); break;
      default: return -1;
    }
#undef DA3B_LN8DQ
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
  }
  if (dq) {
    if (int rc = dequant_q8p_segs(*dq, s)) return rc;
  }
  if (wide) {
#define DA3B_LN8(VPL)                                                                                          \
  k_layernorm8<Tin, VPL><<<blocks, 256, 0, s>>>(in, ld_in, rows, D, g, b, eps, out, ld_out, col_off, rm_div, rm_mul, \
                                                rm_add, q8)
    switch (D) {
      case 256: DA3B_LN8(8); break;
      case 512: DA3B_LN8(16); break;
      case 768: DA3B_LN8(24); break;
      case 1024: DA3B_LN8(32); break;
      case 1536: DA3B_LN8(48); break;
      case 2048: DA3B_LN8(64); break;
      default: return -1;
    }
#undef DA3B_LN8
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
  }
#define DA3B_LN(VPL)                                                                                           \
  k_layernorm<Tin, VPL><<<blocks, 256, 0, s>>>(in, ld_in, rows, D, g, b, eps, out, ld_out, col_off, rm_div, rm_mul, \
                                               rm_add, q8)
  switch (D) {
    case 128: DA3B_LN(4); break;
    case 256: DA3B_LN(8); break;
    case 384: DA3B_LN(12); break;
    case 512: DA3B_LN(16); break;
    case 768: DA3B_LN(24); break;
    case 1024: DA3B_LN(32); break;
    case 1536: DA3B_LN(48); break;
    case 2048: DA3B_LN(64); break;
    default: return -1;
  }
#undef DA3B_LN
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int layernorm_f32(const float* in, int ld_in, int rows, int D, const float* g, const float* b, float eps, __half* out,
                  int ld_out, int col_off, int rm_div, int rm_mul, int rm_add, cudaStream_t s, int q8,
                  const Q8Segs* dq) {
  return ln_dispatch<float>(in, ld_in, rows, D, g, b, eps, out, ld_out, col_off, rm_div, rm_mul, rm_add, q8, s, dq);
}
int layernorm_f16(const __half* in, int ld_in, int rows, int D, const float* g, const float* b, float eps,
                  __half* out, int ld_out, int col_off, int rm_div, int rm_mul, int rm_add, cudaStream_t s) {
  return ln_dispatch<__half>(in, ld_in, rows, D, g, b, eps, out, ld_out, col_off, rm_div, rm_mul, rm_add, 0, s);
}

// f32 rows -> f16 rows with the same row remap as the LayerNorm (DA3 local_x half of feats).
__global__ void k_cast_rows(const float* __restrict__ in, int ld_in, int rows, int D, __half* __restrict__ out,
                            int ld_out, int col_off, int rm_div, int rm_mul, int rm_add) {
  const long total = static_cast<long>(rows) * (D / 4);
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / (D / 4)), c = static_cast<int>(i % (D / 4)) * 4;
    const int ir = rm_div > 0 ? (r / rm_div) * rm_mul + rm_add + r % rm_div : r;
    const float4 f = *reinterpret_cast<const float4*>(in + static_cast<size_t>(ir) * ld_in + c);
    uint2 u;
    *reinterpret_cast<__half2*>(&u.x) = __floats2half2_rn(f.x, f.y);
    *reinterpret_cast<__half2*>(&u.y) = __floats2half2_rn(f.z, f.w);
    *reinterpret_cast<uint2*>(out + static_cast<size_t>(r) * ld_out + col_off + c) = u;
  }
}
int cast_rows(const float* in, int ld_in, int rows, int D, __half* out, int ld_out, int col_off, int rm_div, int rm_mul,
              int rm_add, cudaStream_t s) {
  if (D % 4) return -1;
  k_cast_rows<<<grid_for(static_cast<long>(rows) * (D / 4), 256), 256, 0, s>>>(in, ld_in, rows, D, out, ld_out,
                                                                               col_off, rm_div, rm_mul, rm_add);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// ---------------------------------------------------------------- QK-norm + 2-D RoPE
// In place on qkv [M][3D] (head_dim 64): one warp per (token, head), lane owns dims
// 2l, 2l+1. q/k LayerNorm over 64 (eps 1e-5, src/vit_block.cpp:5-11) then
// rotate-half RoPE per 32-dim half (src/rope2d.cpp:36-52; partner lane = l ^ 8).
// Table row = token % ntok (pos_local or the tiled pos_nodiff of global layers).
__global__ void k_qk_norm_rope(__half* __restrict__ qkv, int M, int H, int D, int ntok, const float* __restrict__ qg,
                               const float* __restrict__ qb, const float* __restrict__ kg,
                               const float* __restrict__ kb, const float* __restrict__ cs,
                               const float* __restrict__ sn) {
  const long warp = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= static_cast<long>(M) * H * 2) return;
  const int which = static_cast<int>(warp & 1);          // 0 = q, 1 = k
  const long th = warp >> 1;
  const int m = static_cast<int>(th / H), h = static_cast<int>(th % H);
  __half2* p = reinterpret_cast<__half2*>(qkv + static_cast<size_t>(m) * 3 * D + which * D + h * 64) + lane;
  float2 v = __half22float2(*p);
  const float* g = which ? kg : qg;
  const float* b = which ? kb : qb;
  if (g) {
    float s = v.x + v.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s * (1.0f / 64.0f);
    const float dx = v.x - mean, dy = v.y - mean;
    float q = dx * dx + dy * dy;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) q += __shfl_xor_sync(0xffffffffu, q, o);
    const float rstd = rsqrtf(q * (1.0f / 64.0f) + 1e-5f);
    v.x = dx * rstd * g[2 * lane] + (b ? b[2 * lane] : 0.f);
    v.y = dy * rstd * g[2 * lane + 1] + (b ? b[2 * lane + 1] : 0.f);
  }
  if (cs) {
    const float px = __shfl_xor_sync(0xffffffffu, v.x, 8);
    const float py = __shfl_xor_sync(0xffffffffu, v.y, 8);
    const bool lo = (lane & 8) == 0;  // first quarter of its half: rot = -partner
    const float rx = lo ? -px : px, ry = lo ? -py : py;
    const int t = m % ntok;
    const float c0 = cs[t * 64 + 2 * lane], c1 = cs[t * 64 + 2 * lane + 1];
    const float s0 = sn[t * 64 + 2 * lane], s1 = sn[t * 64 + 2 * lane + 1];
    v.x = v.x * c0 + rx * s0;
    v.y = v.y * c1 + ry * s1;
  }
  *p = __floats2half2_rn(v.x, v.y);
}
int qk_norm_rope(__half* qkv, int M, int H, int D, int ntok, const float* qg, const float* qb, const float* kg,
                 const float* kb, const float* cs, const float* sn, cudaStream_t s) {
  if (!qg && !cs) return 0;
  const long warps = static_cast<long>(M) * H * 2;
  k_qk_norm_rope<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, s>>>(qkv, M, H, D, ntok, qg, qb, kg, kb,
                                                                                 cs, sn);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ---------------------------------------------------------------- bilinear upsample
// Align-corners bilinear resize of NHWC f16, ggml CPU formula: sf = (dst-1)/(src-1),
// src = i / sf, lerp between floor and floor+1 with clamps (src/dpt_blocks.cpp:87-90).
// Optional f16 addend pe[(y*W + x)][c] (the 0.1 * UV embedding, src/dpt_head.cpp:204-209).
template <int CPT>
__global__ void k_upsample_ac(const __half* __restrict__ in, int B, int hs, int ws, int C, __half* __restrict__ out,
                              int H, int W, const __half* __restrict__ pe) {
  // one output row per blockIdx.y step (its source rows and vertical weight computed
  // once); a thread owns one output pixel x and CPT 8-channel chunks of it, with the
  // channel groups of a pixel on consecutive lanes so that stores stay contiguous
  const int G = C / (8 * CPT);  // channel groups per pixel
  const int per_row = W * G;
  const float sf0 = (W > 1 && ws > 1) ? static_cast<float>(W - 1) / (ws - 1) : static_cast<float>(W) / ws;
  const float sf1 = (H > 1 && hs > 1) ? static_cast<float>(H - 1) / (hs - 1) : static_cast<float>(H) / hs;
  const long rows = static_cast<long>(B) * H;
  for (long orow = blockIdx.y; orow < rows; orow += gridDim.y) {
    const int y = static_cast<int>(orow % H);
    const int b = static_cast<int>(orow / H);
    const float fy = static_cast<float>(y) / sf1;
    int y0 = static_cast<int>(floorf(fy));
    int y1 = y0 + 1;
    const float dy = fminf(fmaxf(fy - floorf(fy), 0.f), 1.f);
    y0 = max(0, min(y0, hs - 1));
    y1 = max(0, min(y1, hs - 1));
    const __half* src0 = in + (static_cast<size_t>(b) * hs + y0) * ws * C;
    const __half* src1 = in + (static_cast<size_t>(b) * hs + y1) * ws * C;
    __half* dst = out + static_cast<size_t>(orow) * W * C;
    const __half* prow = pe ? pe + static_cast<size_t>(y) * W * C : nullptr;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < per_row; i += gridDim.x * blockDim.x) {
      const int x = i / G;
      const int c0 = (i - x * G) * (8 * CPT);
      const float fx = static_cast<float>(x) / sf0;
      int x0 = static_cast<int>(floorf(fx));
      int x1 = x0 + 1;
      const float dx = fminf(fmaxf(fx - floorf(fx), 0.f), 1.f);
      x0 = max(0, min(x0, ws - 1));
      x1 = max(0, min(x1, ws - 1));
      const float wa = (1 - dx) * (1 - dy), wb = dx * (1 - dy), wc = (1 - dx) * dy, wd = dx * dy;
      const float2 wa2 = make_float2(wa, wa), wb2 = make_float2(wb, wb), wc2 = make_float2(wc, wc),
                   wd2 = make_float2(wd, wd);
#pragma unroll
      for (int q = 0; q < CPT; ++q) {
        const int c = c0 + 8 * q;
        const uint4 ua = *reinterpret_cast<const uint4*>(src0 + x0 * C + c);
        const uint4 ub = *reinterpret_cast<const uint4*>(src0 + x1 * C + c);
        const uint4 uc = *reinterpret_cast<const uint4*>(src1 + x0 * C + c);
        const uint4 ud = *reinterpret_cast<const uint4*>(src1 + x1 * C + c);
        const __half2* ha = reinterpret_cast<const __half2*>(&ua);
        const __half2* hb = reinterpret_cast<const __half2*>(&ub);
        const __half2* hc = reinterpret_cast<const __half2*>(&uc);
        const __half2* hd = reinterpret_cast<const __half2*>(&ud);
        uint4 up = make_uint4(0, 0, 0, 0);
        if (prow) up = *reinterpret_cast<const uint4*>(prow + x * C + c);
        const __half2* hp = reinterpret_cast<const __half2*>(&up);
        uint4 uo;
        __half2* ho = reinterpret_cast<__half2*>(&uo);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          float2 r = __fmul2_rn(__half22float2(ha[k]), wa2);
          r = __ffma2_rn(__half22float2(hb[k]), wb2, r);
          r = __ffma2_rn(__half22float2(hc[k]), wc2, r);
          r = __ffma2_rn(__half22float2(hd[k]), wd2, r);
          if (prow) r = __fadd2_rn(r, __half22float2(hp[k]));
          ho[k] = __floats2half2_rn(r.x, r.y);
        }
        *reinterpret_cast<uint4*>(dst + x * C + c) = uo;
      }
    }
  }
}
// Slice-staged variant: one block per (output row, 64-channel slice). The two source
// rows of the slice are read once, coalesced, into shared memory; every output pixel of
// the row is then blended from there (the per-thread form above re-reads each source
// value from L1/L2 about eight times). Same f32 expressions, so the same f16 results.
constexpr int kUpCS = 64;
__global__ void __launch_bounds__(256) k_upsample_staged(const __half* __restrict__ in, int hs, int ws, int C,
                                                         __half* __restrict__ out, int H, int W,
                                                         const __half* __restrict__ pe) {
  extern __shared__ uint4 srow[];  // [2][ws][kUpCS / 8], then the column table
  constexpr int nch = kUpCS / 8;
  const int orow = blockIdx.x, cs0 = blockIdx.y * kUpCS;
  const int y = orow % H, b = orow / H;
  const float sf0 = (W > 1 && ws > 1) ? static_cast<float>(W - 1) / (ws - 1) : static_cast<float>(W) / ws;
  const float sf1 = (H > 1 && hs > 1) ? static_cast<float>(H - 1) / (hs - 1) : static_cast<float>(H) / hs;
  const float fy = static_cast<float>(y) / sf1;
  int y0 = static_cast<int>(floorf(fy));
  int y1 = y0 + 1;
  const float dy = fminf(fmaxf(fy - floorf(fy), 0.f), 1.f);
  y0 = max(0, min(y0, hs - 1));
  y1 = max(0, min(y1, hs - 1));
  const __half* s0 = in + (static_cast<size_t>(b) * hs + y0) * ws * C + cs0;
  const __half* s1 = in + (static_cast<size_t>(b) * hs + y1) * ws * C + cs0;
  // per output column: source columns (x0 | x1 << 16) and weight, computed once per
  // block instead of once per channel chunk
  int2* xtab = reinterpret_cast<int2*>(srow + 2 * ws * nch);
  for (int x = threadIdx.x; x < W; x += blockDim.x) {
    const float fx = static_cast<float>(x) / sf0;
    int x0 = static_cast<int>(floorf(fx));
    int x1 = x0 + 1;
    const float dx = fminf(fmaxf(fx - floorf(fx), 0.f), 1.f);
    x0 = max(0, min(x0, ws - 1));
    x1 = max(0, min(x1, ws - 1));
    xtab[x] = make_int2(x0 | (x1 << 16), __float_as_int(dx));
  }
  const int row_items = ws * nch;
  for (int k = threadIdx.x; k < row_items; k += blockDim.x) {
    const int x = k / nch, c = k % nch;  // nch is a power of two: shifts
    srow[k] = *reinterpret_cast<const uint4*>(s0 + static_cast<size_t>(x) * C + c * 8);
    srow[row_items + k] = *reinterpret_cast<const uint4*>(s1 + static_cast<size_t>(x) * C + c * 8);
  }
  __syncthreads();
  __half* dst = out + static_cast<size_t>(orow) * W * C + cs0;
  const __half* prow = pe ? pe + static_cast<size_t>(y) * W * C + cs0 : nullptr;
  const float dy1 = 1 - dy;
  for (int i = threadIdx.x; i < W * nch; i += blockDim.x) {
    const int x = i / nch, c = i % nch;
    const int2 t = xtab[x];
    const int x0 = t.x & 0xffff, x1 = t.x >> 16;
    const float dx = __int_as_float(t.y);
    const float wa = (1 - dx) * dy1, wb = dx * dy1, wc = (1 - dx) * dy, wd = dx * dy;
    const uint4 ua = srow[x0 * nch + c], ub = srow[x1 * nch + c];
    const uint4 uc = srow[row_items + x0 * nch + c], ud = srow[row_items + x1 * nch + c];
    uint4 up = make_uint4(0, 0, 0, 0);
    if (prow) up = *reinterpret_cast<const uint4*>(prow + static_cast<size_t>(x) * C + c * 8);
    const __half2* ha = reinterpret_cast<const __half2*>(&ua);
    const __half2* hb = reinterpret_cast<const __half2*>(&ub);
    const __half2* hc = reinterpret_cast<const __half2*>(&uc);
    const __half2* hd = reinterpret_cast<const __half2*>(&ud);
    const __half2* hp = reinterpret_cast<const __half2*>(&up);
    uint4 uo;
    __half2* ho = reinterpret_cast<__half2*>(&uo);
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      float2 r = __fmul2_rn(__half22float2(ha[k]), make_float2(wa, wa));
      r = __ffma2_rn(__half22float2(hb[k]), make_float2(wb, wb), r);
      r = __ffma2_rn(__half22float2(hc[k]), make_float2(wc, wc), r);
      r = __ffma2_rn(__half22float2(hd[k]), make_float2(wd, wd), r);
      if (prow) r = __fadd2_rn(r, __half22float2(hp[k]));
      ho[k] = __floats2half2_rn(r.x, r.y);
    }
    *reinterpret_cast<uint4*>(dst + static_cast<size_t>(x) * C + c * 8) = uo;
  }
}

int upsample_ac(const __half* in, int B, int hs, int ws, int C, __half* out, int H, int W, const __half* pe,
                cudaStream_t s) {
  if (C % 8) return -1;
  const long rows = static_cast<long>(B) * H;
  if (rows <= 0 || W <= 0) return 0;
  const int staged_smem = 2 * ws * kUpCS * 2 + 8 * W;  // two source rows + the column table
  if (C % kUpCS == 0 && staged_smem <= 96 * 1024 && ws <= 0xffff && rows <= 0x7fffffffL) {
    static std::atomic<uint64_t> attr_set{0};  // one bit per device; first calls may race
    int dev = 0;
    cudaGetDevice(&dev);
    if (!((attr_set.load() >> (dev & 63)) & 1)) {
      if (cudaFuncSetAttribute(k_upsample_staged, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024) !=
          cudaSuccess)
        return -3;
      attr_set.fetch_or(uint64_t(1) << (dev & 63));
    }
    k_upsample_staged<<<dim3(static_cast<unsigned>(rows), C / kUpCS), 256, staged_smem, s>>>(in, hs, ws, C, out, H, W,
                                                                                               pe);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
  }
  const unsigned gy = static_cast<unsigned>(rows < 65535 ? rows : 65535);
  if (C % 32 == 0) {
    const int per_row = W * (C / 32);
    k_upsample_ac<4><<<dim3((per_row + 127) / 128, gy), 128, 0, s>>>(in, B, hs, ws, C, out, H, W, pe);
  } else {
    const int per_row = W * (C / 8);
    k_upsample_ac<1><<<dim3((per_row + 127) / 128, gy), 128, 0, s>>>(in, B, hs, ws, C, out, H, W, pe);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// ---------------------------------------------------------------- im2col (3x3, stride 2, pad 1)
// NHWC [B][h][w][C] -> [B*ho*wo][9*icp], column = tap*icp + c (the packed conv weight
// layout [OC][9][icp]); columns c >= C are left untouched (zeroed once by the caller).
__global__ void k_im2col_s2(const __half* __restrict__ in, int B, int h, int w, int C, int icp, int ho, int wo,
                            __half* __restrict__ out) {
  const int c8 = C / 8;
  const long total = static_cast<long>(B) * ho * wo * 9 * c8;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % c8) * 8;
    const int tap = static_cast<int>((i / c8) % 9);
    const long pix = i / (static_cast<long>(c8) * 9);
    const int ox = static_cast<int>(pix % wo), oy = static_cast<int>((pix / wo) % ho);
    const int b = static_cast<int>(pix / (static_cast<long>(wo) * ho));
    const int iy = oy * 2 + tap / 3 - 1, ix = ox * 2 + tap % 3 - 1;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (iy >= 0 && iy < h && ix >= 0 && ix < w)
      v = *reinterpret_cast<const uint4*>(in + ((static_cast<size_t>(b) * h + iy) * w + ix) * C + c);
    *reinterpret_cast<uint4*>(out + pix * 9 * icp + tap * icp + c) = v;
  }
}
int im2col_s2(const __half* in, int B, int h, int w, int C, int icp, __half* out, cudaStream_t s) {
  if (C % 8 || icp < C) return -1;
  const int ho = (h + 2 - 3) / 2 + 1, wo = (w + 2 - 3) / 2 + 1;
  const long total = static_cast<long>(B) * ho * wo * 9 * (C / 8);
  k_im2col_s2<<<grid_for(total, 256), 256, 0, s>>>(in, B, h, w, C, icp, ho, wo, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// ---------------------------------------------------------------- V transpose
// v third of qkv [nseq*seqlen][3D] -> vt [nseq][H][64][ld] (per head, token-contiguous).
// 32 x 32 tiles through shared memory: coalesced reads along d, writes along tokens.
__global__ void k_transpose_v(const __half* __restrict__ qkv, int nseq, int seqlen, int H, int D,
                              __half* __restrict__ vt, int ld) {
  __shared__ __half tile[32][33];
  const int tok0 = blockIdx.x * 32, c0 = blockIdx.y * 32, sq = blockIdx.z;  // c0: column within v (0..D)
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;                       // 32 x 8 threads
  for (int i = ty; i < 32; i += 8) {
    const int tok = tok0 + i;
    tile[i][tx] = tok < seqlen ? qkv[(static_cast<size_t>(sq) * seqlen + tok) * 3 * D + 2 * D + c0 + tx]
                               : __float2half(0.f);
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int c = c0 + i, tok = tok0 + tx;
    if (tok < seqlen) vt[(static_cast<size_t>(sq) * D + c) * ld + tok] = tile[tx][i];
  }
}
int transpose_v(const __half* qkv, int nseq, int seqlen, int H, int D, __half* vt, int ld, cudaStream_t s) {
  if (D != H * 64 || ld < seqlen) return -1;
  dim3 grid((seqlen + 31) / 32, D / 32, nseq);
  k_transpose_v<<<grid, 256, 0, s>>>(qkv, nseq, seqlen, H, D, vt, ld);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// ---------------------------------------------------------------- reference-view selection
// One block per scene: saddle-balanced choice over the views' token-0 features after
// the local blocks [0, alt_start-1) (src/dino_backbone.cpp:372-412), in double.
__global__ void k_select_ref_view(const float* __restrict__ x, int S, int ntok, int D, int* __restrict__ b_idx) {
  extern __shared__ double sh[];
  const int scene = blockIdx.x;
  double* nrm = sh;              // [S]
  double* sim = sh + S;          // [S]
  double* var = sh + 2 * S;      // [S]
  double* red = sh + 3 * S;      // [blockDim.x]
  const float* base = x + static_cast<size_t>(scene) * S * ntok * D;
  auto reduce = [&](double v) -> double {
    red[threadIdx.x] = v;
    __syncthreads();
    for (int o = blockDim.x / 2; o > 0; o >>= 1) {
      if (threadIdx.x < o) red[threadIdx.x] += red[threadIdx.x + o];
      __syncthreads();
    }
    const double r = red[0];
    __syncthreads();
    return r;
  };
  for (int v = 0; v < S; ++v) {
    const float* cv = base + static_cast<size_t>(v) * ntok * D;
    double a = 0;
    for (int e = threadIdx.x; e < D; e += blockDim.x) a += static_cast<double>(cv[e]) * cv[e];
    const double n = sqrt(reduce(a));
    if (threadIdx.x == 0) nrm[v] = n;
    __syncthreads();
  }
  for (int v = 0; v < S; ++v) {
    const float* cv = base + static_cast<size_t>(v) * ntok * D;
    const double iv = nrm[v] > 0 ? 1.0 / nrm[v] : 0.0;
    double s = 0;
    for (int w = 0; w < S; ++w) {
      if (w == v) continue;
      const float* cw = base + static_cast<size_t>(w) * ntok * D;
      const double iw = nrm[w] > 0 ? 1.0 / nrm[w] : 0.0;
      double a = 0;
      for (int e = threadIdx.x; e < D; e += blockDim.x) a += (cv[e] * iv) * (cw[e] * iw);
      s += reduce(a);
    }
    double m = 0;
    for (int e = threadIdx.x; e < D; e += blockDim.x) m += cv[e] * iv;
    const double mean = reduce(m) / D;
    double q = 0;
    for (int e = threadIdx.x; e < D; e += blockDim.x) {
      const double d = cv[e] * iv - mean;
      q += d * d;
    }
    const double vv = reduce(q) / (D - 1);
    if (threadIdx.x == 0) {
      sim[v] = s / (S - 1);
      var[v] = vv;
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    double* arrs[3] = {sim, nrm, var};
    for (int k = 0; k < 3; ++k) {
      double mn = arrs[k][0], mx = arrs[k][0];
      for (int v = 0; v < S; ++v) { mn = fmin(mn, arrs[k][v]); mx = fmax(mx, arrs[k][v]); }
      for (int v = 0; v < S; ++v) arrs[k][v] = (arrs[k][v] - mn) / (mx - mn + 1e-8);
    }
    int best = 0;
    double bb = 1e300;
    for (int v = 0; v < S; ++v) {
      const double bal = fabs(sim[v] - 0.5) + fabs(nrm[v] - 0.5) + fabs(var[v] - 0.5);
      if (bal < bb) { bb = bal; best = v; }
    }
    b_idx[scene] = best;
  }
}
int select_ref_view(const float* x, int scenes, int S, int ntok, int D, int* b_idx, cudaStream_t s) {
  const int threads = 256;
  const size_t shm = (3 * S + threads) * sizeof(double);
  k_select_ref_view<<<scenes, threads, shm, s>>>(x, S, ntok, D, b_idx);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Processing position q of a scene holds original view order[q]: order[0] = b,
// order[q] = q-1 for 1 <= q <= b, q otherwise (src/dino_backbone.cpp:435-441).
__device__ __forceinline__ int view_at(int q, int b) { return q == 0 ? b : (q <= b ? q - 1 : q); }

// dst[scene][q] = src[scene][order[q]] for rows of `row_elems` floats per view.
__global__ void k_permute_views(const float* __restrict__ src, float* __restrict__ dst, int scenes, int S,
                                long view_elems, const int* __restrict__ b_idx) {
  const long per_scene = static_cast<long>(S) * view_elems;
  const long total4 = static_cast<long>(scenes) * per_scene / 4;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total4;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long e = i * 4;
    const int scene = static_cast<int>(e / per_scene);
    const long r = e % per_scene;
    const int q = static_cast<int>(r / view_elems);
    const long off = r % view_elems;
    const int v = view_at(q, b_idx[scene]);
    *reinterpret_cast<float4*>(dst + e) =
        *reinterpret_cast<const float4*>(src + static_cast<size_t>(scene) * per_scene + v * view_elems + off);
  }
}
int permute_views(const float* src, float* dst, int scenes, int S, long view_elems, const int* b_idx, cudaStream_t s) {
  if (view_elems % 4) return -1;
  const long total4 = static_cast<long>(scenes) * S * view_elems / 4;
  k_permute_views<<<grid_for(total4, 256), 256, 0, s>>>(src, dst, scenes, S, view_elems, b_idx);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// Inverse for f16 feature rows: dst[scene][t] = src[scene][q] with view_at(q) == t.
__global__ void k_unpermute_views_h(const __half* __restrict__ src, __half* __restrict__ dst, int scenes, int S,
                                    long view_elems, const int* __restrict__ b_idx) {
  const long per_scene = static_cast<long>(S) * view_elems;
  const long total8 = static_cast<long>(scenes) * per_scene / 8;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total8;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long e = i * 8;
    const int scene = static_cast<int>(e / per_scene);
    const long r = e % per_scene;
    const int t = static_cast<int>(r / view_elems);
    const long off = r % view_elems;
    const int b = b_idx[scene];
    const int q = t < b ? t + 1 : (t == b ? 0 : t);
    *reinterpret_cast<uint4*>(dst + e) =
        *reinterpret_cast<const uint4*>(src + static_cast<size_t>(scene) * per_scene + q * view_elems + off);
  }
}
int unpermute_views_h(const __half* src, __half* dst, int scenes, int S, long view_elems, const int* b_idx,
                      cudaStream_t s) {
  if (view_elems % 8) return -1;
  const long total8 = static_cast<long>(scenes) * S * view_elems / 8;
  k_unpermute_views_h<<<grid_for(total8, 256), 256, 0, s>>>(src, dst, scenes, S, view_elems, b_idx);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace da3b

namespace da3b {

// ---------------------------------------------------------------- camera token / pose MLP
// dst[v][col_off + e] = x[v*Nt + 0][e]: token 0 of every view (f32), the camera token
// halves (src/dino_backbone.cpp:197-201).
__global__ void k_copy_token0(const float* __restrict__ x, int V, int Nt, int D, float* __restrict__ dst, int ld_dst,
                              int col_off) {
  const int total = V * D;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const int v = i / D, e = i - v * D;
    dst[static_cast<size_t>(v) * ld_dst + col_off + e] = x[static_cast<size_t>(v) * Nt * D + e];
  }
}
int copy_token0(const float* x, int V, int Nt, int D, float* dst, int ld_dst, int col_off, cudaStream_t s) {
  if (V <= 0 || D <= 0) return 0;
  k_copy_token0<<<grid_for(static_cast<long>(V) * D, 256), 256, 0, s>>>(x, V, Nt, D, dst, ld_dst, col_off);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// y[m][y_off + n] = act(sum_k x[m][k] W[n][k] + b[n]) for a handful of rows m (the
// camera decoder's M = views): one warp per output column n, f32 activations, f16
// weights, f32 accumulation.
__global__ void k_gemv_rows(const float* __restrict__ x, int M, int K, const __half* __restrict__ W, int ldw,
                            const float* __restrict__ b, int N, int act, float* __restrict__ y, int ldy, int y_off) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= N) return;
  const __half* w = W + static_cast<size_t>(warp) * ldw;
  for (int m = 0; m < M; ++m) {
    const float* xr = x + static_cast<size_t>(m) * K;
    float acc = 0.f;
    for (int k = lane; k < K; k += 32) acc = fmaf(__half2float(w[k]), xr[k], acc);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      float v = acc + (b ? b[warp] : 0.f);
      if (act == 1) v = fmaxf(v, 0.f);
      y[static_cast<size_t>(m) * ldy + y_off + warp] = v;
    }
  }
}
int gemv_rows(const float* x, int M, int K, const __half* W, int ldw, const float* b, int N, int act, float* y,
              int ldy, int y_off, cudaStream_t s) {
  if (M <= 0 || N <= 0) return 0;
  const int threads = 256, warps = threads / 32;
  k_gemv_rows<<<(N + warps - 1) / warps, threads, 0, s>>>(x, M, K, W, ldw, b, N, act, y, ldy, y_off);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace da3b
