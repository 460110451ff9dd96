// Fused DPT output stage: align-corners upsample of out1 to the image size (+ the
// 0.1 UV pos-embed), output_conv2's 3x3 conv to 32 channels, relu, the 1x1 conv to
// output_dim and the output activation (src/dpt_head.cpp:199-222 and :327-338; the
// feature map `feat_map` of the reference is never written to memory).
//
// One CTA = a strip of 120 output pixels of a band of consecutive output rows of one
// image (kRows rows, fewer when the batch would otherwise leave SMs idle). The
// upsampled rows the 3x3 taps need are built once each in shared memory, in a ring of
// four row slots laid out K-major without swizzle ([16-byte channel
// chunk][row][8 halves]); slot row r = 32 w + l holds strip pixel 30 w + l, so each
// 32-row block (one epilogue warp's TMEM lanes) carries its 30 pixels plus the 2 halo
// pixels on its right. The three horizontal taps go into N: per row and vertical tap
// dy, one tcgen05.mma (M = 128 rows, N = 96 = 3 taps x 32 channels, K = 16) per 16
// input channels gives Z_dx[r] = sum_c A[r][c] W[dy][dx][c] for all three dx at once,
// and lane l < 30 of an epilogue warp forms out = Z_0[l] + Z_1[l + 1] + Z_2[l + 2] with
// shuffles inside the warp (a small-N MMA costs about as much per instruction as
// N = 96, so one wide MMA replaces three narrow ones; no warp needs another's data).
//   warps 0-7  build row j+2 while the tensor core works on row j (bilinear from the
//              NHWC out1 map, the f32 weights of k_upsample_ac, PE added, f16), after
//              a bulk L2 prefetch of the source rows three steps ahead; warps 0-3 (even
//              rows) and 4-7 (odd rows) also run the epilogue: TMEM -> tap sum,
//              bias, relu, 1x1 conv, activation;
//   warp 8     one thread issues the 3 x C/16 MMAs of a row into one of two TMEM
//              accumulators of 96 columns.
#include <algorithm>
#include <atomic>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "gemm.h"
#include "ops.h"
#include "ptx.cuh"

namespace da3b {
namespace {

constexpr int kPx = 128;               // slot rows per strip (MMA M)
constexpr int kTile = 120;             // output pixels per strip: 4 warps x 30
constexpr int kPitch = kPx + 1;        // rows per channel-chunk plane: the extra 16 B spread the
                                       // builders' 16-byte stores over all banks (2048 B would not)
constexpr int kSlots = 4;              // upsampled-row ring
constexpr int kRows = 74;              // output rows per CTA (at most)
constexpr int kBuildWarps = 8;
constexpr int kThreads = (kBuildWarps + 1) * 32;
constexpr int kOC = 32;                // output_conv2 hidden channels
constexpr int kN = 3 * kOC;            // MMA N: three horizontal taps x 32 channels
constexpr int kConsts = 360;           // bias 32 | LN gamma 32 | LN beta 32 | out2b 8x32 | out2b bias 8

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// Bulk prefetch of [p, p + bytes) into L2 (16-byte aligned address, bytes % 16 == 0).
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// K-major operand without swizzle: 8-row core matrices of 16-byte rows, 8-row groups
// `sbo` apart, 16-byte channel chunks `lbo` apart.
__device__ __forceinline__ uint64_t desc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100; swizzle field 0 = none
  return d;
}

struct Layout {
  uint32_t slot_bytes, w_bytes, total;
};

__host__ __device__ inline Layout layout_for(int C) {
  Layout l;
  l.slot_bytes = static_cast<uint32_t>(C / 8) * kPitch * 16;
  l.w_bytes = 9u * static_cast<uint32_t>(C / 8) * kOC * 16;
  l.total = 1024 + kSlots * l.slot_bytes + l.w_bytes + kConsts * 4 + kPx * 12 + 16 * 8 + 16;
  return l;
}

// C (the out1 channel count) is a template parameter: 16, 32, 64 or 128.
template <int C>
__global__ void __launch_bounds__(kThreads, 1)
    k_up_out2(const __half* __restrict__ src, int hs, int ws, const __half* __restrict__ pe, int H, int W,
              const __half* __restrict__ wp, int icp, int rows, const EpiArgs e, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const Layout L = layout_for(C);
  constexpr int nkc = C >> 3;
  uint8_t* sRows = smem;
  uint8_t* sW = sRows + kSlots * L.slot_bytes;
  float* sC = reinterpret_cast<float*>(sW + L.w_bytes);
  int* sX0 = reinterpret_cast<int*>(sC + kConsts);
  int* sX1 = sX0 + kPx;
  float* sDX = reinterpret_cast<float*>(sX1 + kPx);
  uint64_t* bars = reinterpret_cast<uint64_t*>((reinterpret_cast<uintptr_t>(sDX + kPx) + 7) & ~uintptr_t(7));
  uint64_t* row_full = bars;       // [4] a row slot built (8 builder warps)
  uint64_t* slot_free = bars + 4;  // [4] the last MMA reading a row slot completed
  uint64_t* acc_full = bars + 8;   // [2] a row's accumulator complete
  uint64_t* acc_empty = bars + 10; // [2] its epilogue drained it (4 warps)
  uint64_t* drain = bars + 12;     // every issued MMA completed (teardown)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.z, xs0 = blockIdx.x * kTile, ya = blockIdx.y * rows;
  const int R = min(rows, H - ya);
  // align-corners source scale, as k_upsample_ac
  const float sf0 = (W > 1 && ws > 1) ? static_cast<float>(W - 1) / (ws - 1) : static_cast<float>(W) / ws;
  const float sf1 = (H > 1 && hs > 1) ? static_cast<float>(H - 1) / (hs - 1) : static_cast<float>(H) / hs;

  // per-CTA tables: source columns of the slot rows, epilogue constants, weights
  for (int p = threadIdx.x; p < kPx; p += blockDim.x) {
    const int xo = xs0 - 1 + 30 * (p >> 5) + (p & 31);  // slot row -> image column
    if (xo < 0 || xo >= W) {
      sX0[p] = -1;
      sX1[p] = -1;
      sDX[p] = 0.f;
    } else {
      const float fx = static_cast<float>(xo) / sf0;
      int x0 = static_cast<int>(floorf(fx));
      int x1 = x0 + 1;
      sDX[p] = fminf(fmaxf(fx - floorf(fx), 0.f), 1.f);
      sX0[p] = max(0, min(x0, ws - 1));
      sX1[p] = max(0, min(x1, ws - 1));
    }
  }
  for (int i = threadIdx.x; i < kConsts; i += blockDim.x) {
    float v = 0.f;
    if (i < 32) v = e.bias ? e.bias[i] : 0.f;
    else if (i < 64) v = e.o2_ln_g ? e.o2_ln_g[i - 32] : 1.f;
    else if (i < 96) v = e.o2_ln_b ? e.o2_ln_b[i - 64] : 0.f;
    else if (i < 352) v = (i - 96) < e.o2_dim * 32 ? e.o2_w[i - 96] : 0.f;
    else v = (i - 352) < e.o2_dim ? e.o2_b[i - 352] : 0.f;
    sC[i] = v;
  }
  // packed weights [32][9][icp] (tap = 3 dy + dx) -> [dy][chunk][dx * 32 + oc][8 halves],
  // four loads in flight per thread
  constexpr int kWItems = kOC * 9 * nkc;
  for (int i0 = threadIdx.x; i0 < kWItems; i0 += 4 * kThreads) {
    uint4 wv[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = i0 + q * kThreads;
      const int c8 = i % nkc, t = (i / nkc) % 9, oc = i / (nkc * 9);
      wv[q] = i < kWItems ? *reinterpret_cast<const uint4*>(wp + (static_cast<size_t>(oc) * 9 + t) * icp + c8 * 8)
                          : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = i0 + q * kThreads;
      if (i >= kWItems) break;
      const int c8 = i % nkc, t = (i / nkc) % 9, oc = i / (nkc * 9);
      const int dy = t / 3, dx = t % 3;
      *reinterpret_cast<uint4*>(sW + ((dy * nkc + c8) * kN + dx * kOC + oc) * 16) = wv[q];
    }
  }
  fence_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      mbar_init(&row_full[s], kBuildWarps);
      mbar_init(&slot_free[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
  }
  if (warp == kBuildWarps) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kBuildWarps) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA
      // output row i reads row slots (i, i+1, i+2) & 3 = upsampled rows y-1, y, y+1
      constexpr uint32_t idesc = umma_idesc_f16(128, kN);
      const uint32_t lbo_a = kPitch * 16, lbo_b = kN * 16;
      const uint32_t rows0 = smem_u32(sRows), w0 = smem_u32(sW);
      bool ok = true;
      int issued = 0;
      for (int i = 0; i < R && ok; ++i) {
        for (int j = (i == 0 ? 0 : i + 2); j <= i + 2 && ok; ++j)
          ok = mbar_wait(&row_full[j & 3], (j >> 2) & 1, status, kStatusTimeoutFull);
        if (ok && i >= 2) ok = mbar_wait(&acc_empty[i & 1], ((i >> 1) - 1) & 1, status, kStatusTimeoutAccumFree);
        if (!ok) break;
        tc_fence_after();
        const uint32_t tAcc = tmem + (i & 1) * 128;
        uint32_t acc = 0;
#pragma unroll 1
        for (int dy = 0; dy < 3; ++dy) {
          const uint32_t rb = rows0 + ((i + dy) & 3) * L.slot_bytes;
          for (int k = 0; k < nkc / 2; ++k) {
            const uint64_t a = desc_noswz(rb + (2 * k * kPitch) * 16, lbo_a, 128);
            const uint64_t bw = desc_noswz(w0 + ((dy * nkc + 2 * k) * kN) * 16, lbo_b, 128);
            umma_f16(tAcc, a, bw, idesc, acc);
            acc = 1;
          }
        }
        umma_commit(&acc_full[i & 1]);
        umma_commit(&slot_free[i & 3]);
        ++issued;
      }
      // every issued MMA has landed before the accumulator is freed (also on a timeout)
      if (issued > 0) {
        umma_commit(drain);
        mbar_wait(drain, 0, status, kStatusTimeoutAccum);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ builders
    const int tb = threadIdx.x;  // 0 .. 255
    const size_t img = static_cast<size_t>(b) * hs;
    // first / last slot row inside the image (source column range of the strip)
    const int xlo_row = xs0 == 0 ? 1 : 0;
    int xhi_row = kPx - 1;
    while (xhi_row > xlo_row && sX0[xhi_row] < 0) --xhi_row;
    auto build = [&](int j) {
      const int u = ya - 1 + j;  // upsampled row
      uint8_t* dst = sRows + (j & 3) * L.slot_bytes;
      const bool row_ok = u >= 0 && u < H;
      float dy = 0.f;
      const __half* s0 = src;
      const __half* s1 = src;
      const __half* prow = nullptr;
      // L2 prefetch, by one thread with bulk (TMA-unit) prefetches of whole row
      // segments, of the source rows (and PE row) of upsampled row u + 3, built three
      // steps later; the first build also covers rows u .. u + 2. A per-line
      // prefetch.global.L2 left a third of the builders' loads missing L2.
      if (tb == 0) {
        for (int uu = (j == 0 ? u : u + 3); uu <= u + 3; ++uu) {
          if (uu < 0 || uu >= H) continue;
          const float f2 = static_cast<float>(uu) / sf1;
          const int r0 = max(0, min(static_cast<int>(floorf(f2)), hs - 1));
          const int r1 = max(0, min(static_cast<int>(floorf(f2)) + 1, hs - 1));
          const int xlo = sX0[xlo_row], xhi = sX1[xhi_row];
          const uint32_t bytes = static_cast<uint32_t>(xhi - xlo + 1) * C * 2;
          bulk_prefetch_l2(src + ((img + r0) * ws + xlo) * C, bytes);
          if (r1 != r0) bulk_prefetch_l2(src + ((img + r1) * ws + xlo) * C, bytes);
          if (pe) {
            const int plo = max(0, xs0 - 1), phi = min(W, xs0 + kTile + 2);
            bulk_prefetch_l2(pe + (static_cast<size_t>(uu) * W + plo) * C, static_cast<uint32_t>(phi - plo) * C * 2);
          }
        }
      }
      if (row_ok) {
        const float fy = static_cast<float>(u) / sf1;
        int y0 = static_cast<int>(floorf(fy));
        int y1 = y0 + 1;
        dy = fminf(fmaxf(fy - floorf(fy), 0.f), 1.f);
        y0 = max(0, min(y0, hs - 1));
        y1 = max(0, min(y1, hs - 1));
        s0 = src + (img + y0) * ws * C;
        s1 = src + (img + y1) * ws * C;
        if (pe) prow = pe + static_cast<size_t>(u) * W * C;
      }
      constexpr int kBatch = 4;
      {
        // C / 8 = nkc is a power of two (the launcher checks): thread tb owns one
        // 16-byte channel chunk of every pstep-th slot row
        constexpr int pstep = (kBuildWarps * 32) / nkc;  // slot rows covered per pass
        constexpr int nit = kPx / pstep;                 // items per thread: nkc / 2
        const int kc_own = tb & (nkc - 1);
        const int p0 = tb / nkc;  // its slot rows: p0 + t * pstep, t < nit
        // kBatch items' corner loads are in flight before any is used (zero-filled
        // first, which also keeps the compiler from spilling)
        uint8_t* dcol = dst + (kc_own * kPitch) * 16;
        if (!row_ok) {
          for (int t = 0; t < nit; ++t) *reinterpret_cast<uint4*>(dcol + (p0 + t * pstep) * 16) = make_uint4(0, 0, 0, 0);
        } else {
          const __half* s0c = s0 + kc_own * 8;
          const __half* s1c = s1 + kc_own * 8;
#pragma unroll 1
          for (int t0 = 0; t0 < nit; t0 += kBatch) {
            uint4 ua[kBatch], ub[kBatch], uc[kBatch], ud[kBatch], up[kBatch];
#pragma unroll
            for (int q = 0; q < kBatch; ++q) ua[q] = ub[q] = uc[q] = ud[q] = up[q] = make_uint4(0, 0, 0, 0);
#pragma unroll
            for (int q = 0; q < kBatch; ++q) {
              const int p = p0 + (t0 + q) * pstep;
              const int x0 = (t0 + q < nit) ? sX0[p] : -1;
              if (x0 >= 0) {
                const int x1 = sX1[p];
                ua[q] = *reinterpret_cast<const uint4*>(s0c + x0 * C);
                ub[q] = *reinterpret_cast<const uint4*>(s0c + x1 * C);
                uc[q] = *reinterpret_cast<const uint4*>(s1c + x0 * C);
                ud[q] = *reinterpret_cast<const uint4*>(s1c + x1 * C);
                if (prow) up[q] = *reinterpret_cast<const uint4*>(prow + (xs0 - 1 + 30 * (p >> 5) + (p & 31)) * C + kc_own * 8);
              }
            }
#pragma unroll
            for (int q = 0; q < kBatch; ++q) {
              if (t0 + q >= nit) break;
              const int p = p0 + (t0 + q) * pstep;
              uint4 uo = make_uint4(0, 0, 0, 0);
              if (sX0[p] >= 0) {
                const float dx = sDX[p];
                const float wa = (1 - dx) * (1 - dy), wb = dx * (1 - dy), wc = (1 - dx) * dy, wd = dx * dy;
                const float2 wa2 = make_float2(wa, wa), wb2 = make_float2(wb, wb), wc2 = make_float2(wc, wc),
                             wd2 = make_float2(wd, wd);
                const __half2* ha = reinterpret_cast<const __half2*>(&ua[q]);
                const __half2* hb = reinterpret_cast<const __half2*>(&ub[q]);
                const __half2* hc = reinterpret_cast<const __half2*>(&uc[q]);
                const __half2* hd = reinterpret_cast<const __half2*>(&ud[q]);
                const __half2* hp = reinterpret_cast<const __half2*>(&up[q]);
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
              }
              *reinterpret_cast<uint4*>(dcol + p * 16) = uo;
            }
          }
        }
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&row_full[j & 3]);
    };
    const float* cb = sC;
    auto epilogue = [&](int i) -> bool {
      if (!mbar_wait_warp(&acc_full[i & 1], (i >> 1) & 1, status, kStatusTimeoutAccum)) return false;
      tc_fence_after();
      // lane l of warp w: slot row 32 (w mod 4) + l, Z_dx for dx = 0, 1, 2
      const uint32_t ta = tmem + (i & 1) * 128 + (static_cast<uint32_t>((warp & 3) * 32) << 16);
      uint32_t z0[32], z1[32], z2[32];
      tmem_ld32(ta, z0);
      tmem_ld32(ta + kOC, z1);
      tmem_ld32(ta + 2 * kOC, z2);
      tmem_wait_ld();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[i & 1]);
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float a1 = __shfl_down_sync(0xffffffffu, __uint_as_float(z1[j]), 1);
        const float a2 = __shfl_down_sync(0xffffffffu, __uint_as_float(z2[j]), 2);
        v[j] = ((__uint_as_float(z0[j]) + a1) + a2) + cb[j];
      }
      const int xo = xs0 + (warp & 3) * 30 + lane;
      if (lane < 30 && xo < W) {
        if (e.o2_ln_g) {
          float mean = 0.f;
#pragma unroll
          for (int j = 0; j < 32; ++j) mean += v[j];
          mean *= (1.0f / 32.0f);
          float var = 0.f;
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float d = v[j] - mean;
            var += d * d;
          }
          var *= (1.0f / 32.0f);
          const float rstd = rsqrtf(var + e.o2_ln_eps);
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = (v[j] - mean) * rstd * cb[32 + j] + cb[64 + j];
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.0f);
        const size_t pix = (static_cast<size_t>(b) * H + ya + i) * W + xo;
        for (int od = 0; od < e.o2_dim; ++od) {
          float l = cb[352 + od];
          const float* w = cb + 96 + od * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j) l = fmaf(v[j], w[j], l);
          e.o2_out[od][pix] = out_act(l, e.o2_act[od], e.o2_scale);
        }
      }
      return true;
    };
    bool ok = true;
    for (int j = 0; j <= R + 1 && ok; ++j) {
      // slot j & 3 last held row j - 4, last read by MMA(j - 4)
      if (j >= 4) ok = mbar_wait_warp(&slot_free[j & 3], ((j - 4) >> 2) & 1, status, kStatusTimeoutEmpty);
      if (!ok) break;
      build(j);
      // even rows' epilogues on warps 0-3, odd rows' on warps 4-7 (same TMEM lane
      // quarters), so both halves of the builders carry the same load
      if (j >= 3 && ((j - 3) & 1) == (warp >> 2)) ok = epilogue(j - 3);
    }
    if (ok && R >= 1 && ((R - 1) & 1) == (warp >> 2)) epilogue(R - 1);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kBuildWarps) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

}  // namespace

int up_out2(const __half* src, int B, int hs, int ws, int C, const __half* pe, int H, int W, const __half* wp,
            int icp, const EpiArgs& e, int* status, cudaStream_t s) {
  if (B <= 0 || hs <= 0 || ws <= 0 || H <= 0 || W <= 0) return 0;
  // C = 16, 32, 64 or 128: the builders give each thread one 16-byte chunk of C / 8
  if (C < 16 || C > 128 || (C & (C - 1)) || icp < C || icp % 8 || e.kind != kEpiOut2 || e.o2_dim < 1 ||
      e.o2_dim > 8)
    return -1;
  for (int i = 0; i < e.o2_dim; ++i)
    if (!e.o2_out[i]) return -1;
  if ((reinterpret_cast<uintptr_t>(src) & 15) || (pe && (reinterpret_cast<uintptr_t>(pe) & 15)) ||
      (reinterpret_cast<uintptr_t>(wp) & 15))
    return -2;
  const Layout L = layout_for(C);
  static std::atomic<uint64_t> attr_set{0};  // one bit per device; first calls may race
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((attr_set.load() >> (dev & 63)) & 1)) {
    if (cudaFuncSetAttribute(k_up_out2<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, layout_for(16).total) !=
            cudaSuccess ||
        cudaFuncSetAttribute(k_up_out2<32>, cudaFuncAttributeMaxDynamicSharedMemorySize, layout_for(32).total) !=
            cudaSuccess ||
        cudaFuncSetAttribute(k_up_out2<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, layout_for(64).total) !=
            cudaSuccess ||
        cudaFuncSetAttribute(k_up_out2<128>, cudaFuncAttributeMaxDynamicSharedMemorySize, layout_for(128).total) !=
            cudaSuccess)
      return -3;
    attr_set.fetch_or(uint64_t(1) << (dev & 63));
  }
  // Row bands of kRows, or shorter ones when that would give fewer CTAs than SMs (a
  // band costs its two halo rows extra; one 518 x 518 image: 5 x 7 CTAs of 74 rows
  // against 5 x 29 of 18). The rows per CTA do not change any output value.
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int gx = (W + kTile - 1) / kTile;
  const long long per_band = static_cast<long long>(gx) * B;
  const int bands = static_cast<int>(std::min<long long>(H, (sms + per_band - 1) / per_band));
  const int rows = std::max(std::min(kRows, (H + bands - 1) / bands), 1);
  dim3 grid(gx, (H + rows - 1) / rows, B);
  switch (C) {
    case 16: k_up_out2<16><<<grid, kThreads, L.total, s>>>(src, hs, ws, pe, H, W, wp, icp, rows, e, status); break;
    case 32: k_up_out2<32><<<grid, kThreads, L.total, s>>>(src, hs, ws, pe, H, W, wp, icp, rows, e, status); break;
    case 64: k_up_out2<64><<<grid, kThreads, L.total, s>>>(src, hs, ws, pe, H, W, wp, icp, rows, e, status); break;
    default: k_up_out2<128><<<grid, kThreads, L.total, s>>>(src, hs, ws, pe, H, W, wp, icp, rows, e, status); break;
  }
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace da3b
