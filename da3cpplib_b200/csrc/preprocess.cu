// Preprocessing on the GPU: the uint8 resizers of preprocess_real and the normalise +
// patchify kernel that builds the patch-embed GEMM operand.
//
// Resizes follow DA3cpplib's own cv2-style uint8 resizers (src/preprocess.cpp:45-148)
// to the bit: the per-axis taps and weights are built on the host with the reference's
// double/float arithmetic (cubic: Catmull-Rom a = -0.75 on src = (dst + 0.5) * scale
// - 0.5 with clamped indices; area: cv2's INTER_AREA decimation table), and the device
// passes accumulate in the reference's order with explicitly rounded multiplies and
// adds (no fused multiply-add), through a float intermediate, and saturate to uint8
// with round-half-to-even.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "da3b.h"
#include "kernels.h"
#include "preprocess.h"

namespace da3b {

// ------------------------------------------------------------------ host tables
namespace {

float cubic_weight(float x) {  // Catmull-Rom, a = -0.75 (src/preprocess.cpp:51-56)
  const float a = -0.75f;
  x = std::fabs(x);
  if (x < 1) return ((a + 2) * x - (a + 3)) * x * x + 1;
  if (x < 2) return (((x - 5) * x + 8) * x - 4) * a;
  return 0.f;
}

}  // namespace

AxisTaps cubic_taps(int ssize, int dsize) {
  AxisTaps t;
  t.off.push_back(0);
  const double scale = static_cast<double>(ssize) / dsize;
  for (int d = 0; d < dsize; ++d) {
    const double f = (d + 0.5) * scale - 0.5;
    const int i = static_cast<int>(std::floor(f));
    const float u = static_cast<float>(f - i);
    const float w[4] = {cubic_weight(u + 1), cubic_weight(u), cubic_weight(u - 1), cubic_weight(u - 2)};
    for (int k = 0; k < 4; ++k) {
      t.idx.push_back(std::min(std::max(i - 1 + k, 0), ssize - 1));
      t.w.push_back(w[k]);
    }
    t.off.push_back(static_cast<int>(t.idx.size()));
  }
  return t;
}

// cv2 INTER_AREA decimation (computeResizeAreaTab): per destination index, the
// partially covered first source cell, the fully covered ones, the partial last one.
AxisTaps area_taps(int ssize, int dsize) {
  AxisTaps t;
  t.off.push_back(0);
  const double scale = static_cast<double>(ssize) / dsize;
  for (int d = 0; d < dsize; ++d) {
    const double f1 = d * scale, f2 = f1 + scale;
    const double cell = std::min(scale, static_cast<double>(ssize) - f1);
    int s1 = static_cast<int>(std::ceil(f1)), s2 = static_cast<int>(std::floor(f2));
    s2 = std::min(s2, ssize - 1);
    s1 = std::min(s1, s2);
    if (s1 - f1 > 1e-3) {
      t.idx.push_back(s1 - 1);
      t.w.push_back(static_cast<float>((s1 - f1) / cell));
    }
    for (int s = s1; s < s2; ++s) {
      t.idx.push_back(s);
      t.w.push_back(static_cast<float>(1.0 / cell));
    }
    if (f2 - s2 > 1e-3) {
      t.idx.push_back(s2);
      t.w.push_back(static_cast<float>(std::min(std::min(f2 - s2, 1.0), cell) / cell));
    }
    t.off.push_back(static_cast<int>(t.idx.size()));
  }
  return t;
}

// ------------------------------------------------------------------ device passes
namespace {

__device__ __forceinline__ uint8_t sat_u8(float v) {  // round half to even, clamp [0, 255]
  const int r = __float2int_rn(v);
  return static_cast<uint8_t>(r < 0 ? 0 : (r > 255 ? 255 : r));
}

// horizontal pass: tmp[b][y][dx][c] = sum_t w[t] * src[b][y][idx[t]][c], taps in table order
__global__ void k_resize_h(const uint8_t* __restrict__ src, int rows, int sw, int dw, const int* __restrict__ off,
                           const int* __restrict__ idx, const float* __restrict__ w, float* __restrict__ tmp) {
  const long total = static_cast<long>(rows) * dw * 3;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % 3);
    const long rest = i / 3;
    const int dx = static_cast<int>(rest % dw);
    const long row = rest / dw;
    const uint8_t* s = src + static_cast<size_t>(row) * sw * 3 + c;
    float acc = 0.f;
    for (int t = off[dx]; t < off[dx + 1]; ++t)
      acc = __fadd_rn(acc, __fmul_rn(w[t], static_cast<float>(s[idx[t] * 3])));
    tmp[i] = acc;
  }
}

// vertical pass + saturation: dst[b][dy][x][c] = u8(sum_t w[t] * tmp[b][idx[t]][x][c])
__global__ void k_resize_v(const float* __restrict__ tmp, int B, int sh, int dh, int dw, const int* __restrict__ off,
                           const int* __restrict__ idx, const float* __restrict__ w, uint8_t* __restrict__ dst) {
  const long total = static_cast<long>(B) * dh * dw * 3;
  const long plane = static_cast<long>(dw) * 3;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const long col = i % plane;  // x * 3 + c
    const long r2 = i / plane;
    const int dy = static_cast<int>(r2 % dh);
    const long b = r2 / dh;
    const float* t0 = tmp + static_cast<size_t>(b) * sh * plane + col;
    float acc = 0.f;
    for (int t = off[dy]; t < off[dy + 1]; ++t)
      acc = __fadd_rn(acc, __fmul_rn(w[t], t0[static_cast<size_t>(idx[t]) * plane]));
    dst[i] = sat_u8(acc);
  }
}

// INTER_AREA asked to enlarge both axes: the reference falls back to its float
// bilinear (src/preprocess.cpp:8-24, :122-130) and saturates.
__global__ void k_resize_bilinear_u8(const uint8_t* __restrict__ src, int B, int sw, int sh, int dw, int dh, float sx,
                                     float sy, uint8_t* __restrict__ dst) {
  const long total = static_cast<long>(B) * dh * dw * 3;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int c = static_cast<int>(i % 3);
    const long p = i / 3;
    const int x = static_cast<int>(p % dw);
    const long r = p / dw;
    const int y = static_cast<int>(r % dh);
    const long b = r / dh;
    const float fy = __fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(y), 0.5f), sy), 0.5f);
    const int y0 = static_cast<int>(floorf(fy));
    const float wy = __fsub_rn(fy, static_cast<float>(y0));
    const int y0c = min(max(y0, 0), sh - 1), y1c = min(max(y0 + 1, 0), sh - 1);
    const float fx = __fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(x), 0.5f), sx), 0.5f);
    const int x0 = static_cast<int>(floorf(fx));
    const float wx = __fsub_rn(fx, static_cast<float>(x0));
    const int x0c = min(max(x0, 0), sw - 1), x1c = min(max(x0 + 1, 0), sw - 1);
    const uint8_t* s = src + static_cast<size_t>(b) * sh * sw * 3 + c;
    auto P = [&](int yy, int xx) { return static_cast<float>(s[(static_cast<size_t>(yy) * sw + xx) * 3]); };
    const float iwx = __fsub_rn(1.f, wx), iwy = __fsub_rn(1.f, wy);
    const float top = __fadd_rn(__fmul_rn(P(y0c, x0c), iwx), __fmul_rn(P(y0c, x1c), wx));
    const float bot = __fadd_rn(__fmul_rn(P(y1c, x0c), iwx), __fmul_rn(P(y1c, x1c), wx));
    dst[i] = sat_u8(__fadd_rn(__fmul_rn(top, iwy), __fmul_rn(bot, wy)));
  }
}

unsigned blocks_for(long n) {
  long b = (n + 255) / 256;
  if (b > (1L << 20)) b = 1L << 20;
  return static_cast<unsigned>(b < 1 ? 1 : b);
}

}  // namespace

// ------------------------------------------------------------------ Resizer
Resizer::~Resizer() {
  if (tmp_) cudaFree(tmp_);
  for (auto& kv : tables_) cudaFree(kv.second.dev);
  if (mid_) cudaFree(mid_);
}

const Resizer::DevTaps* Resizer::taps(int ssize, int dsize, int mode) {
  const auto key = std::make_tuple(ssize, dsize, mode);
  auto it = tables_.find(key);
  if (it != tables_.end()) return &it->second;
  const AxisTaps t = mode == 0 ? cubic_taps(ssize, dsize) : area_taps(ssize, dsize);
  const size_t n_off = t.off.size(), n = t.idx.size();
  const size_t bytes = (n_off + n) * sizeof(int) + n * sizeof(float);
  DevTaps d;
  if (cudaMalloc(&d.dev, bytes) != cudaSuccess) return nullptr;
  d.off = static_cast<int*>(d.dev);
  d.idx = d.off + n_off;
  d.w = reinterpret_cast<float*>(d.idx + n);
  if (cudaMemcpy(d.off, t.off.data(), n_off * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(d.idx, t.idx.data(), n * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemcpy(d.w, t.w.data(), n * sizeof(float), cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(d.dev);
    return nullptr;
  }
  return &tables_.emplace(key, d).first->second;
}

int Resizer::resize(const uint8_t* src, int B, int sw, int sh, uint8_t* dst, int dw, int dh, int mode,
                    cudaStream_t s) {
  if (B <= 0 || sw <= 0 || sh <= 0 || dw <= 0 || dh <= 0 || (mode != 0 && mode != 1)) return -1;
  if (mode == 1 && dw >= sw && dh >= sh) {
    const float sx = static_cast<float>(sw) / dw, sy = static_cast<float>(sh) / dh;
    const long total = static_cast<long>(B) * dh * dw * 3;
    k_resize_bilinear_u8<<<blocks_for(total), 256, 0, s>>>(src, B, sw, sh, dw, dh, sx, sy, dst);
    return cudaGetLastError() == cudaSuccess ? 0 : -2;
  }
  const DevTaps* tx = taps(sw, dw, mode);
  const DevTaps* ty = taps(sh, dh, mode);
  if (!tx || !ty) return -3;
  const size_t need = static_cast<size_t>(B) * sh * dw * 3 * sizeof(float);
  if (need > tmp_cap_) {
    if (tmp_) {
      cudaStreamSynchronize(s);
      cudaFree(tmp_);
    }
    tmp_ = nullptr;
    tmp_cap_ = 0;
    if (cudaMalloc(&tmp_, need) != cudaSuccess) return -4;
    tmp_cap_ = need;
  }
  const long th = static_cast<long>(B) * sh * dw * 3;
  k_resize_h<<<blocks_for(th), 256, 0, s>>>(src, B * sh, sw, dw, tx->off, tx->idx, tx->w, tmp_);
  const long tv = static_cast<long>(B) * dh * dw * 3;
  k_resize_v<<<blocks_for(tv), 256, 0, s>>>(tmp_, B, sh, dh, dw, ty->off, ty->idx, ty->w, dst);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// preprocess_real's two resizes (src/preprocess.cpp:157-190): bound side to target
// (cubic when enlarging, area otherwise), then each side to its nearest multiple of the
// patch size. The sizes are computed exactly as the reference does.
int Resizer::preprocess_real(const uint8_t* src, int B, int w, int h, int patch, int target, bool upper, uint8_t* dst,
                             int* out_w, int* out_h, cudaStream_t s) {
  int w1 = w, h1 = h;
  bool step1 = false;
  const int bound = upper ? std::max(w, h) : std::min(w, h);
  const double scale = static_cast<double>(target) / bound;
  if (bound != target) {
    w1 = std::max(1, static_cast<int>(std::nearbyint(w * scale)));
    h1 = std::max(1, static_cast<int>(std::nearbyint(h * scale)));
    step1 = true;
  }
  auto nearest = [](int x, int p) {
    const int down = (x / p) * p, up = down + p;
    return (std::abs(up - x) <= std::abs(x - down)) ? up : down;
  };
  const int w2 = std::max(1, nearest(w1, patch)), h2 = std::max(1, nearest(h1, patch));
  const bool step2 = w2 != w1 || h2 != h1;
  *out_w = w2;
  *out_h = h2;
  if (!dst) return 0;  // size query only
  const int mode1 = scale > 1.0 ? 0 : 1;
  const int mode2 = (w2 > w1 || h2 > h1) ? 0 : 1;
  if (!step1 && !step2)
    return cudaMemcpyAsync(dst, src, static_cast<size_t>(B) * w * h * 3, cudaMemcpyDefault, s) == cudaSuccess ? 0 : -5;
  if (step1 && !step2) return resize(src, B, w, h, dst, w1, h1, mode1, s);
  if (!step1) return resize(src, B, w, h, dst, w2, h2, mode2, s);
  const size_t need = static_cast<size_t>(B) * w1 * h1 * 3;
  if (need > mid_cap_) {
    if (mid_) {
      cudaStreamSynchronize(s);
      cudaFree(mid_);
    }
    mid_ = nullptr;
    mid_cap_ = 0;
    if (cudaMalloc(&mid_, need) != cudaSuccess) return -4;
    mid_cap_ = need;
  }
  int rc = resize(src, B, w, h, mid_, w1, h1, mode1, s);
  if (rc) return rc;
  return resize(mid_, B, w1, h1, dst, w2, h2, mode2, s);
}

// ------------------------------------------------------------------ patchify
// RGB8 [B][H][W][3] -> normalised, patch-major A matrix of the patch-embed GEMM:
// row = b*Np + (py*gw + px), column k = c*P*P + ky*P + kx (the flattening of the
// conv weight [D][3][P][P]), zero for k >= 3*P*P. Normalisation is the reference's
// (v/255 - mean[c]) / std[c] in f32 (src/preprocess.cpp:192-196), stored as f16.
namespace {

// Patch size 14 (DINOv2): one CTA per (image, patch row, strip of up to kStrip patches).
// The 14 image rows of the strip are staged in shared memory with aligned 4-byte loads
// (the words that straddle the ends of the image buffer are read byte by byte), then
// every thread writes 8 consecutive f16 of one patch's operand row.
constexpr int kP = 14;
constexpr int kStrip = 16;  // patches per CTA
constexpr int kRowBytes = kStrip * kP * 3;

__global__ void __launch_bounds__(256) k_patchify14(const uint8_t* __restrict__ rgb, int B, int H, int W, int gh,
                                                    int gw, float m0, float m1, float m2, float s0, float s1, float s2,
                                                    __half* __restrict__ out, int ldk) {
  __shared__ __align__(16) uint8_t tile[kP * kRowBytes];
  // Per-channel value table: lut[c][v] = f16((v / 255 - mean_c) / sd_c), built with the
  // same f32 operations as the per-element formula, so the output bits are unchanged;
  // and per operand column k < 3 * 14 * 14 the staged-tile byte offset of patch 0
  // (ky * kRowBytes + kx * 3 + c) with the channel in bits 16+.
  __shared__ unsigned short lut[3 * 256];
  __shared__ int ktab[3 * kP * kP];
  for (int i = threadIdx.x; i < 3 * 256; i += blockDim.x) {
    const int c = i >> 8;
    const float u = static_cast<float>(i & 255) / 255.f;
    const float mean = c == 0 ? m0 : (c == 1 ? m1 : m2);
    const float sd = c == 0 ? s0 : (c == 1 ? s1 : s2);
    lut[i] = __half_as_ushort(__float2half_rn((u - mean) / sd));
  }
  for (int k = threadIdx.x; k < 3 * kP * kP; k += blockDim.x) {
    const int c = k / (kP * kP), r = k - c * (kP * kP), ky = r / kP, kx = r - ky * kP;
    ktab[k] = (ky * kRowBytes + kx * 3 + c) | (c << 16);
  }
  const uintptr_t lo = reinterpret_cast<uintptr_t>(rgb);
  const uintptr_t hi = lo + static_cast<size_t>(B) * H * W * 3;
  const int px0 = blockIdx.x * kStrip, py = blockIdx.y, b = blockIdx.z;
  const int np = min(kStrip, gw - px0);
  const int row_bytes = np * kP * 3;
  for (int ky = 0; ky < kP; ++ky) {
    const uint8_t* base = rgb + ((static_cast<size_t>(b) * H + py * kP + ky) * W + px0 * kP) * 3;
    const uintptr_t a0 = reinterpret_cast<uintptr_t>(base) & ~uintptr_t(3);
    const int lead = static_cast<int>(reinterpret_cast<uintptr_t>(base) - a0);
    const int nwords = (lead + row_bytes + 3) / 4;
    uint8_t* dst = tile + ky * kRowBytes;
    for (int wi = threadIdx.x; wi < nwords; wi += blockDim.x) {
      const uintptr_t wa = a0 + 4 * static_cast<uintptr_t>(wi);
      if (wa >= lo && wa + 4 <= hi) {
        const uint32_t v = *reinterpret_cast<const uint32_t*>(wa);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int o = wi * 4 + j - lead;  // byte offset within the staged row
          if (o >= 0 && o < row_bytes) dst[o] = static_cast<uint8_t>(v >> (8 * j));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int o = wi * 4 + j - lead;
          if (o >= 0 && o < row_bytes) dst[o] = base[o];
        }
      }
    }
  }
  __syncthreads();
  const int k8 = ldk / 8;  // 8-column groups per operand row
  const int kk = 3 * kP * kP;
  for (int item = threadIdx.x; item < np * k8; item += blockDim.x) {
    const int pl = item / k8, k0 = (item - pl * k8) * 8;
    const int poff = pl * kP * 3;
    uint32_t w[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      uint32_t h[2];
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        const int k = k0 + 2 * j + q;
        h[q] = 0u;  // operand columns past 3 * 14 * 14: zero padding
        if (k < kk) {
          const int e = ktab[k];
          h[q] = lut[(e >> 16) * 256 + tile[(e & 0xffff) + poff]];
        }
      }
      w[j] = h[0] | (h[1] << 16);
    }
    const size_t row = (static_cast<size_t>(b) * gh + py) * gw + px0 + pl;
    *reinterpret_cast<uint4*>(out + row * ldk + k0) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// Any patch size: one thread per pair of operand columns.
__global__ void k_patchify_any(const uint8_t* __restrict__ rgb, int B, int H, int W, int P, int gh, int gw, float m0,
                               float m1, float m2, float s0, float s1, float s2, __half* __restrict__ out, int ldk) {
  const long total = static_cast<long>(B) * gh * gw * (ldk / 2);
  const int kk = 3 * P * P;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int k2 = static_cast<int>(i % (ldk / 2)) * 2;
    const long row = i / (ldk / 2);
    const int p = static_cast<int>(row % (gh * gw));
    const int b = static_cast<int>(row / (gh * gw));
    const int py = p / gw, px = p % gw;
    float v[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int k = k2 + j;
      if (k < kk) {
        const int c = k / (P * P), r = k % (P * P), ky = r / P, kx = r % P;
        const int y = py * P + ky, x = px * P + kx;
        const float u = static_cast<float>(rgb[((static_cast<size_t>(b) * H + y) * W + x) * 3 + c]) / 255.f;
        const float mean = c == 0 ? m0 : (c == 1 ? m1 : m2);
        const float sd = c == 0 ? s0 : (c == 1 ? s1 : s2);
        v[j] = (u - mean) / sd;
      } else {
        v[j] = 0.f;
      }
    }
    *reinterpret_cast<__half2*>(out + row * ldk + k2) = __floats2half2_rn(v[0], v[1]);
  }
}

}  // namespace

int patchify(const uint8_t* rgb, int B, int H, int W, int P, const float* mean, const float* sd, __half* out, int ldk,
             cudaStream_t s) {
  if (H % P || W % P || ldk % 2 || ldk < 3 * P * P) return -1;
  const int gh = H / P, gw = W / P;
  if (B <= 0 || gh <= 0 || gw <= 0) return 0;
  if (P == kP && ldk % 8 == 0 && (reinterpret_cast<uintptr_t>(out) & 15) == 0 && gh <= 65535 && B <= 65535) {
    const dim3 grid((gw + kStrip - 1) / kStrip, gh, B);
    k_patchify14<<<grid, 256, 0, s>>>(rgb, B, H, W, gh, gw, mean[0], mean[1], mean[2], sd[0], sd[1], sd[2], out,
                                      ldk);
  } else {
    const long total = static_cast<long>(B) * gh * gw * (ldk / 2);
    k_patchify_any<<<blocks_for(total), 256, 0, s>>>(rgb, B, H, W, P, gh, gw, mean[0], mean[1], mean[2], sd[0], sd[1],
                                                     sd[2], out, ldk);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

namespace {

// planar f32 [B][3][H][W] -> operand rows (8 consecutive columns per thread)
__global__ void k_patchify_chw(const float* __restrict__ chw, int B, int H, int W, int P, int gh, int gw,
                               __half* __restrict__ out, int ldk) {
  const int k8 = ldk / 8, kk = 3 * P * P;
  const long total = static_cast<long>(B) * gh * gw * k8;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int k0 = static_cast<int>(i % k8) * 8;
    const long row = i / k8;
    const int p = static_cast<int>(row % (gh * gw));
    const int b = static_cast<int>(row / (gh * gw));
    const int py = p / gw, px = p % gw;
    float v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int k = k0 + j;
      if (k < kk) {
        const int c = k / (P * P), r = k % (P * P), ky = r / P, kx = r % P;
        v[j] = chw[((static_cast<size_t>(b) * 3 + c) * H + py * P + ky) * W + px * P + kx];
      } else {
        v[j] = 0.f;
      }
    }
    uint4 o;
    __half2* h2 = reinterpret_cast<__half2*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) h2[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
    *reinterpret_cast<uint4*>(out + row * ldk + k0) = o;
  }
}

}  // namespace

// Legacy preprocess (src/preprocess.cpp:8-41): float bilinear resize of RGB8 to the
// floor-to-patch size, then (v / 255 - mean[c]) / std[c] into planar f32 [B][3][dh][dw],
// with the reference's f32 operations in its order (explicit rounding, no FMA).
__global__ void k_legacy_pre(const uint8_t* __restrict__ src, int B, int sw, int sh, int dw, int dh, float sx, float sy,
                             float m0, float m1, float m2, float s0, float s1, float s2, float* __restrict__ out) {
  const long total = static_cast<long>(B) * 3 * dh * dw;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int x = static_cast<int>(i % dw);
    const long r = i / dw;
    const int y = static_cast<int>(r % dh);
    const long r2 = r / dh;
    const int c = static_cast<int>(r2 % 3);
    const long b = r2 / 3;
    const float fy = __fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(y), 0.5f), sy), 0.5f);
    const int y0 = static_cast<int>(floorf(fy));
    const float wy = __fsub_rn(fy, static_cast<float>(y0));
    const int y0c = min(max(y0, 0), sh - 1), y1c = min(max(y0 + 1, 0), sh - 1);
    const float fx = __fsub_rn(__fmul_rn(__fadd_rn(static_cast<float>(x), 0.5f), sx), 0.5f);
    const int x0 = static_cast<int>(floorf(fx));
    const float wx = __fsub_rn(fx, static_cast<float>(x0));
    const int x0c = min(max(x0, 0), sw - 1), x1c = min(max(x0 + 1, 0), sw - 1);
    const uint8_t* sp = src + static_cast<size_t>(b) * sh * sw * 3 + c;
    auto P = [&](int yy, int xx) { return static_cast<float>(sp[(static_cast<size_t>(yy) * sw + xx) * 3]); };
    const float iwx = __fsub_rn(1.f, wx), iwy = __fsub_rn(1.f, wy);
    const float top = __fadd_rn(__fmul_rn(P(y0c, x0c), iwx), __fmul_rn(P(y0c, x1c), wx));
    const float bot = __fadd_rn(__fmul_rn(P(y1c, x0c), iwx), __fmul_rn(P(y1c, x1c), wx));
    const float v = __fdiv_rn(__fadd_rn(__fmul_rn(top, iwy), __fmul_rn(bot, wy)), 255.f);
    const float mean = c == 0 ? m0 : (c == 1 ? m1 : m2);
    const float sd = c == 0 ? s0 : (c == 1 ? s1 : s2);
    out[i] = __fdiv_rn(__fsub_rn(v, mean), sd);
  }
}

int legacy_preprocess(const uint8_t* src, int B, int w, int h, int patch, const float* mean, const float* sd,
                      float* out, int* out_w, int* out_h, cudaStream_t s) {
  if (B <= 0 || w <= 0 || h <= 0 || patch <= 0) return -1;
  int dw = (w / patch) * patch, dh = (h / patch) * patch;
  if (dw == 0) dw = patch;
  if (dh == 0) dh = patch;
  *out_w = dw;
  *out_h = dh;
  if (!out) return 0;
  const float sx = static_cast<float>(w) / dw, sy = static_cast<float>(h) / dh;
  const long total = static_cast<long>(B) * 3 * dh * dw;
  k_legacy_pre<<<blocks_for(total), 256, 0, s>>>(src, B, w, h, dw, dh, sx, sy, mean[0], mean[1], mean[2], sd[0], sd[1],
                                                 sd[2], out);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int patchify_chw(const float* chw, int B, int H, int W, int P, __half* out, int ldk, cudaStream_t s) {
  if (H % P || W % P || ldk % 8 || ldk < 3 * P * P || (reinterpret_cast<uintptr_t>(out) & 15)) return -1;
  const int gh = H / P, gw = W / P;
  if (B <= 0 || gh <= 0 || gw <= 0) return 0;
  const long total = static_cast<long>(B) * gh * gw * (ldk / 8);
  k_patchify_chw<<<blocks_for(total), 256, 0, s>>>(chw, B, H, W, P, gh, gw, out, ldk);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace da3b

// ------------------------------------------------------------------ C ABI
namespace {
std::mutex g_rs_mu;
da3b::Resizer* g_rs[64] = {nullptr};
}  // namespace

extern "C" {

DA3B_API int da3b_resize_u8(const void* src, int B, int sw, int sh, void* dst, int dw, int dh, int mode,
                            void* stream) {
  if (!src || !dst || B <= 0 || sw <= 0 || sh <= 0 || dw <= 0 || dh <= 0 || (mode != 0 && mode != 1)) return -100;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -101;
  std::lock_guard<std::mutex> lk(g_rs_mu);
  if (!g_rs[dev]) g_rs[dev] = new da3b::Resizer();
  return g_rs[dev]->resize(static_cast<const uint8_t*>(src), B, sw, sh, static_cast<uint8_t*>(dst), dw, dh, mode,
                           static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_preprocess_legacy(const void* rgb, int B, int w, int h, int patch, const float* mean,
                                    const float* std_, void* chw_out, int* out_h, int* out_w, void* stream) {
  if (!rgb || !mean || !std_ || !out_h || !out_w) return -100;
  return da3b::legacy_preprocess(static_cast<const uint8_t*>(rgb), B, w, h, patch, mean, std_,
                                 static_cast<float*>(chw_out), out_w, out_h, static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_patchify(const void* rgb, int B, int H, int W, int patch, const float* mean, const float* std_,
                           void* out, int ldk, void* stream) {
  if (!rgb || !out || !mean || !std_ || B < 0 || H <= 0 || W <= 0 || patch <= 0) return -100;
  return da3b::patchify(static_cast<const uint8_t*>(rgb), B, H, W, patch, mean, std_, static_cast<__half*>(out), ldk,
                        static_cast<cudaStream_t>(stream));
}

}  // extern "C"
