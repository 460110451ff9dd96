// 3x3 NHWC convolution (stride 1, zero padding 1), output channels in groups of 128,
// with one input tile read per channel chunk. Replaces the implicit-GEMM conv for the DPT
// head's output_conv1 (src/dpt_head.cpp:199-203; ggml_conv_2d of the features map,
// 256 -> 128 channels at 8 x the patch grid).
//
// The implicit GEMM fetches the input once per tap (nine times per pixel). Here a CTA
// owns a 16 x 16 output-pixel tile as two 8-wide halves, one TMEM accumulator
// (M = 128 pixels, N = 128 channels) each. Per 64-channel chunk one TMA box of the
// 18 x 18 input pixels around the tile lands in shared memory channel-chunk-major
// ([chunk][y][x][8 halves], the K-major no-swizzle operand layout with a 16-byte
// core-matrix row per pixel), and each of the nine taps is the same box read with a
// descriptor whose start is shifted by (dy * 18 + dx) pixels: rows of one 8-pixel
// output row are 16 bytes apart, output rows 18 pixels (288 bytes) apart. Each
// 128 x 64 weight tile (SW128, TMA) feeds both accumulators.
//   warp 0     TMA: per chunk, the nine weight tiles, after the next chunk's input
//              box (three box stages)
//   warp 1     one thread issues 2 halves x 9 taps x 4 K-steps of M = 128, N = 128,
//              K = 16 per chunk into one of two double-buffered accumulator pairs
//   warps 2-5  epilogue: TMEM -> + bias (+ res1 + res2, relu copy, activation) ->
//              f16 NHWC; the accumulator pair is released after it is read
// A tile is (128-channel output group, 16 x 16 pixels), the group index fastest so the
// groups of one pixel tile run side by side and share its input boxes in L2.
// A CTA-pair form (k_conv3_halo2, below) serves output counts in groups of 256.
// Persistent: grid = number of SMs, tiles assigned round-robin. Every wait is bounded
// (ptx.cuh); on a timeout the kernel records a status, drains its MMAs and exits.
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

namespace da3b {
namespace {

constexpr int kOCh = 128;                 // output channels (MMA N)
constexpr int kTw = 16, kTh = 16;         // output tile: two 8-wide halves
constexpr int kBoxW = kTw + 2, kBoxH = kTh + 2;
constexpr int kBoxPx = kBoxW * kBoxH;     // 324
constexpr uint32_t kABytes = kBoxPx * 128;          // 64 channels x 324 pixels x 2 B = 41 472
constexpr uint32_t kBBytes = kOCh * 128;            // 128 rows x 64 channels x 2 B = 16 384
constexpr int kAStages = 3, kBStages = 6;
constexpr uint32_t kLbo = kBoxPx * 16;    // channel-chunk plane stride
constexpr uint32_t kSbo = kBoxW * 16;     // next output row (8-row group)
constexpr int kThreads = 192;
constexpr uint32_t kSmem = 1024 + kBStages * kBBytes + kAStages * kABytes + 256;

__device__ __forceinline__ uint64_t desc_noswz(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100; swizzle field 0 = none
  return d;
}

__device__ __forceinline__ void add_h8(const uint4& u, float (&v)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const float2 f = __half22float2(h[k]);
    v[2 * k] += f.x;
    v[2 * k + 1] += f.y;
  }
}

__device__ __forceinline__ void st_h8(__half* p, const float (&v)[8]) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int k = 0; k < 4; ++k) h[k] = __floats2half2_rn(v[2 * k], v[2 * k + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// Epilogue of one accumulator buffer, this thread's pixel in each 8-wide half (pix,
// valid): TMEM -> + bias (+ res1 + res2, relu copy, activation) -> f16 NHWC, 32
// channels (one tcgen05.ld) per chunk. The residual reads of chunk k + kDist are issued
// before chunk k's stores, and those of the first kDist chunks before the accumulator
// is waited on: a load cannot be moved above an earlier store through a pointer of the
// same type, so read one chunk at a time they each paid a full memory latency in turn
// (about 2 us of a 25 us batch-1 conv). Returns false when the accumulator wait timed out.
template <int kHalves, int kN, int kDist>
__device__ __forceinline__ bool halo_epilogue(uint32_t tacc, uint64_t* full, uint32_t parity, int* status,
                                              const EpiArgs& e, const size_t (&pix)[kHalves],
                                              const bool (&valid)[kHalves], int n0) {
  constexpr int kNc = kN / 32, kChunks = kHalves * kNc, kRing = kDist + 1;
  uint4 ra[kRing][4], rb[kRing][4];
  auto fetch = [&](int k) {
    const int h = k / kNc, c = k % kNc;
    if (!valid[h]) return;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int n = n0 + c * 32 + g * 8;
      if (e.res1) ra[k % kRing][g] = *reinterpret_cast<const uint4*>(e.res1 + pix[h] * e.ld_res1 + n);
      if (e.res2) rb[k % kRing][g] = *reinterpret_cast<const uint4*>(e.res2 + pix[h] * e.ld_res2 + n);
    }
  };
#pragma unroll
  for (int k = 0; k < kDist && k < kChunks; ++k) fetch(k);
  if (!mbar_wait_warp(full, parity, status, kStatusTimeoutAccum)) return false;
  tc_fence_after();
#pragma unroll
  for (int k = 0; k < kChunks; ++k) {
    if (k + kDist < kChunks) fetch(k + kDist);
    const int h = k / kNc, c = k % kNc;
    uint32_t r[32];
    tmem_ld32(tacc + h * kN + c * 32, r);
    tmem_wait_ld();
    if (!valid[h]) continue;
#pragma unroll
    for (int g = 0; g < 4; ++g) {
      const int n = n0 + c * 32 + g * 8;
      float v[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) v[q] = __uint_as_float(r[g * 8 + q]);
      if (e.bias) {
        const float4 b0 = __ldg(reinterpret_cast<const float4*>(e.bias + n));
        const float4 b1 = __ldg(reinterpret_cast<const float4*>(e.bias + n + 4));
        v[0] += b0.x; v[1] += b0.y; v[2] += b0.z; v[3] += b0.w;
        v[4] += b1.x; v[5] += b1.y; v[6] += b1.z; v[7] += b1.w;
      }
      if (e.res1) add_h8(ra[k % kRing][g], v);
      if (e.res2) add_h8(rb[k % kRing][g], v);
      if (e.out_relu) {
        float rl[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) rl[q] = fmaxf(v[q], 0.0f);
        st_h8(e.out_relu + pix[h] * e.ld_out + n, rl);
      }
      if (e.act == kActRelu) {
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = fmaxf(v[q], 0.0f);
      }
      st_h8(e.out + pix[h] * e.ld_out + n, v);
    }
  }
  return true;
}

__global__ void __launch_bounds__(kThreads, 1)
    k_conv3_halo(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int B, int H, int W,
                 int nck, int icp, int n_oc, const EpiArgs e, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem;                              // [kBStages][128][64] SW128
  uint8_t* sA = sB + kBStages * kBBytes;           // [kAStages][8][18][18][8]
  uint64_t* bars = reinterpret_cast<uint64_t*>(sA + kAStages * kABytes);
  uint64_t* a_full = bars;                         // [kAStages]
  uint64_t* a_empty = bars + kAStages;             // [kAStages]
  uint64_t* b_full = a_empty + kAStages;           // [kBStages]
  uint64_t* b_empty = b_full + kBStages;           // [kBStages]
  uint64_t* acc_full = b_empty + kBStages;         // [2]
  uint64_t* acc_empty = acc_full + 2;              // [2] (4 epilogue warps)
  uint64_t* drain = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tiles_x = (W + kTw - 1) / kTw, tiles_y = (H + kTh - 1) / kTh;
  const int n_tiles = B * tiles_x * tiles_y * n_oc;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < kBStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 4);
    }
    mbar_init(drain, 1);
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------------------ TMA
      // chunks g = tile-step * nck + c in order; the input box of chunk g + 1 is
      // requested before the nine weight tiles of chunk g, a chunk ahead of its use
      const int my_tiles = blockIdx.x < n_tiles ? (n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
      const int n_chunks = my_tiles * nck;
      auto load_box = [&](int g) -> bool {
        const int t = blockIdx.x + (g / nck) * gridDim.x, c = g % nck;
        const int tp = t / n_oc;
        const int tx = tp % tiles_x, ty = (tp / tiles_x) % tiles_y, b = tp / (tiles_x * tiles_y);
        const uint32_t sa = static_cast<uint32_t>(g) % kAStages;
        if (!mbar_wait(&a_empty[sa], ((static_cast<uint32_t>(g) / kAStages) & 1) ^ 1u, status, kStatusTimeoutEmpty))
          return false;
        mbar_arrive_expect_tx(&a_full[sa], kABytes);
        tma_load_5d(sA + sa * kABytes, &tmA, &a_full[sa], 0, tx * kTw - 1, ty * kTh - 1, c * 8, b);
        return true;
      };
      uint32_t ib = 0;
      bool ok = n_chunks == 0 || load_box(0);
      for (int g = 0; g < n_chunks && ok; ++g) {
        if (g + 1 < n_chunks && !load_box(g + 1)) break;
        const int og = (blockIdx.x + (g / nck) * gridDim.x) % n_oc, c = g % nck;
        for (int tap = 0; tap < 9; ++tap) {
          const uint32_t sb = ib % kBStages;
          if (!mbar_wait(&b_empty[sb], ((ib / kBStages) & 1) ^ 1u, status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&b_full[sb], kBBytes);
          tma_load_2d(sB + sb * kBBytes, &tmB, &b_full[sb], tap * icp + c * 64, og * kOCh);
          ++ib;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------------------ MMA
      constexpr uint32_t idesc = umma_idesc_f16(128, kOCh);
      const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
      uint32_t ia = 0, ib = 0, tc = 0;
      bool ok = true;
      int issued = 0;
      for (int t = blockIdx.x; t < n_tiles && ok; t += gridDim.x, ++tc) {
        const uint32_t ab = tc & 1;
        if (tc >= 2 && !mbar_wait(&acc_empty[ab], ((tc >> 1) - 1) & 1, status, kStatusTimeoutAccumFree)) break;
        tc_fence_after();
        const uint32_t tAcc = tmem + ab * 256;
        for (int c = 0; c < nck && ok; ++c) {
          const uint32_t sa = ia % kAStages;
          if (!mbar_wait(&a_full[sa], (ia / kAStages) & 1, status, kStatusTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t abox = a0 + sa * kABytes;
          for (int tap = 0; tap < 9; ++tap) {
            const uint32_t sb = ib % kBStages;
            if (!mbar_wait(&b_full[sb], (ib / kBStages) & 1, status, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const int dy = tap / 3, dx = tap - 3 * dy;
            const uint64_t bd = umma_desc_sw128(b0 + sb * kBBytes);
#pragma unroll
            for (int half = 0; half < 2; ++half) {
              const uint32_t start = abox + static_cast<uint32_t>((dy * kBoxW + 8 * half + dx) * 16);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_f16(tAcc + half * 128, desc_noswz(start + 2 * k * kLbo, kLbo, kSbo), bd + 2 * k, idesc,
                         (c | tap | k) ? 1u : 0u);
            }
            umma_commit(&b_empty[sb]);
            ++ib;
            ++issued;
          }
          umma_commit(&a_empty[sa]);
          ++ia;
        }
        if (!ok) break;
        umma_commit(&acc_full[ab]);
      }
      // every issued MMA has landed before TMEM is freed (also on a timeout)
      if (issued > 0) {
        umma_commit(drain);
        mbar_wait(drain, 0, status, kStatusTimeoutAccum);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quarter of this warp
    const int m = q * 32 + lane;            // accumulator row: output pixel (m / 8, m % 8)
    const int i = m >> 3, j = m & 7;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    uint32_t tc = 0;
    for (int t = blockIdx.x; t < n_tiles; t += gridDim.x, ++tc) {
      const uint32_t ab = tc & 1;
      const int og = t % n_oc, tp = t / n_oc;
      const int tx = tp % tiles_x, ty = (tp / tiles_x) % tiles_y, b = tp / (tiles_x * tiles_y);
      const int y = ty * kTh + i;
      size_t pix[2];
      bool valid[2];
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        const int x = tx * kTw + 8 * half + j;
        valid[half] = y < H && x < W;
        pix[half] = valid[half] ? (static_cast<size_t>(b) * H + y) * W + x : 0;
      }
      if (!halo_epilogue<2, kOCh, 2>(tmem + ab * 256 + lane_off, &acc_full[ab], (tc >> 1) & 1, status, e, pix,
                                     valid, og * kOCh))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---------------------------------------------------------------- CTA-pair form
// The same scheme over a cluster of two CTAs (cta_group::2). Each CTA owns its own
// 16-row pixel tile of kHalves 8-wide halves and loads its own input box, plus half of
// the N weight rows of every tap; the leader's single thread issues M = 256 MMAs
// whose rows 0-127 come from the leader's box and 128-255 from the peer's, leaving
// each CTA's accumulators in its own TMEM. Per CTA this halves the weight bytes
// written to and read from shared memory, which the 1-CTA form spends as much
// shared-memory bandwidth on as the MMA itself. All loads complete on the leader's
// barriers; MMA completions are multicast to both CTAs (tcgen05.commit), the peer's
// epilogue releases an accumulator with a remote arrive on the leader's barrier.
template <int N, int kHalves>
struct Halo2Cfg {
  static constexpr int kTw = 8 * kHalves, kTh = 16;
  static constexpr int kBoxW = kTw + 2, kBoxH = kTh + 2, kBoxPx = kBoxW * kBoxH;
  static constexpr uint32_t kABytes = kBoxPx * 128;
  static constexpr uint32_t kBBytes = (N / 2) * 128;      // this CTA's N/2 weight rows x 64 channels
  static constexpr int kAStages = 3, kBStages = 6;
  static constexpr uint32_t kLbo = kBoxPx * 16, kSbo = kBoxW * 16;
  static constexpr uint32_t kAccCols = kHalves * N;      // per accumulator buffer
  static constexpr uint32_t kSmem = 1024 + kBStages * kBBytes + kAStages * kABytes + 256;
  static_assert(2 * kAccCols <= 512, "two accumulator buffers must fit in TMEM");
};

template <int N, int kHalves>
__global__ void __launch_bounds__(kThreads, 1)
    k_conv3_halo2(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int B, int H,
                  int W, int nck, int icp, int n_oc, const EpiArgs e, int* status) {
  using Cfg = Halo2Cfg<N, kHalves>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sB = smem;
  uint8_t* sA = sB + Cfg::kBStages * Cfg::kBBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sA + Cfg::kAStages * Cfg::kABytes);
  uint64_t* a_full = bars;                            // [kAStages] (leader's used)
  uint64_t* a_empty = a_full + Cfg::kAStages;         // [kAStages]
  uint64_t* b_full = a_empty + Cfg::kAStages;         // [kBStages] (leader's used)
  uint64_t* b_empty = b_full + Cfg::kBStages;         // [kBStages]
  uint64_t* acc_full = b_empty + Cfg::kBStages;       // [2]
  uint64_t* acc_empty = acc_full + 2;                 // [2] (leader's: 2 x 4 epilogue warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles_x = (W + Cfg::kTw - 1) / Cfg::kTw, tiles_y = (H + Cfg::kTh - 1) / Cfg::kTh;
  const int n_px = B * tiles_x * tiles_y;             // pixel tiles; a pair takes two
  const int n_tiles = ((n_px + 1) / 2) * n_oc;        // pair tiles, output group fastest
  const int my_tiles = pair < n_tiles ? (n_tiles - 1 - pair) / npairs + 1 : 0;

  if (threadIdx.x == 0) {
    for (int s = 0; s < Cfg::kAStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    for (int s = 0; s < Cfg::kBStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 2 * 4);
    }
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
  }
  if (warp == 1) tmem_alloc2(tmem_slot, 512);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  // this CTA's pixel tile of pair tile t: (b, ty, tx); b == B past the last tile
  auto px_tile = [&](int t, int& b, int& ty, int& tx) {
    const int p = 2 * (t / n_oc) + static_cast<int>(rank);
    b = p / (tiles_x * tiles_y);
    const int rem = p - b * tiles_x * tiles_y;
    ty = rem / tiles_x;
    tx = rem - ty * tiles_x;
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- TMA (both CTAs)
      const int n_chunks = my_tiles * nck;
      auto load_box = [&](int g) -> bool {
        const int t = pair + (g / nck) * npairs, c = g % nck;
        int b, ty, tx;
        px_tile(t, b, ty, tx);
        const uint32_t sa = static_cast<uint32_t>(g) % Cfg::kAStages;
        if (!mbar_wait(&a_empty[sa], ((static_cast<uint32_t>(g) / Cfg::kAStages) & 1) ^ 1u, status,
                       kStatusTimeoutEmpty))
          return false;
        if (rank == 0) mbar_arrive_expect_tx(&a_full[sa], 2 * Cfg::kABytes);
        tma2_load_5d(sA + sa * Cfg::kABytes, &tmA, mapa_shared(smem_u32(&a_full[sa]), 0), 0, tx * Cfg::kTw - 1,
                     ty * Cfg::kTh - 1, c * 8, b);
        return true;
      };
      uint32_t ib = 0;
      bool ok = n_chunks == 0 || load_box(0);
      for (int g = 0; g < n_chunks && ok; ++g) {
        if (g + 1 < n_chunks && !load_box(g + 1)) break;
        const int og = (pair + (g / nck) * npairs) % n_oc, c = g % nck;
        for (int tap = 0; tap < 9; ++tap) {
          const uint32_t sb = ib % Cfg::kBStages;
          if (!mbar_wait(&b_empty[sb], ((ib / Cfg::kBStages) & 1) ^ 1u, status, kStatusTimeoutEmpty)) {
            ok = false;
            break;
          }
          if (rank == 0) mbar_arrive_expect_tx(&b_full[sb], 2 * Cfg::kBBytes);
          tma2_load_2d(sB + sb * Cfg::kBBytes, &tmB, mapa_shared(smem_u32(&b_full[sb]), 0), tap * icp + c * 64,
                       og * N + static_cast<int>(rank) * (N / 2));
          ++ib;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // ---------------------------------------------------------- MMA (leader only)
      constexpr uint32_t idesc = umma_idesc_f16(256, N);
      const uint32_t a0 = smem_u32(sA), b0 = smem_u32(sB);
      uint32_t ia = 0, ib = 0;
      bool ok = true;
      for (int it = 0; it < my_tiles && ok; ++it) {
        const uint32_t ab = it & 1;
        if (!mbar_wait(&acc_empty[ab], ((it >> 1) & 1) ^ 1u, status, kStatusTimeoutAccumFree)) break;
        tc_fence_after();
        const uint32_t tAcc = tmem + ab * Cfg::kAccCols;
        for (int c = 0; c < nck && ok; ++c) {
          const uint32_t sa = ia % Cfg::kAStages;
          if (!mbar_wait(&a_full[sa], (ia / Cfg::kAStages) & 1, status, kStatusTimeoutFull)) { ok = false; break; }
          tc_fence_after();
          const uint32_t abox = a0 + sa * Cfg::kABytes;
          for (int tap = 0; tap < 9; ++tap) {
            const uint32_t sb = ib % Cfg::kBStages;
            if (!mbar_wait(&b_full[sb], (ib / Cfg::kBStages) & 1, status, kStatusTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            const int dy = tap / 3, dx = tap - 3 * dy;
            const uint64_t bd = umma_desc_sw128(b0 + sb * Cfg::kBBytes);
#pragma unroll
            for (int half = 0; half < kHalves; ++half) {
              const uint32_t start = abox + static_cast<uint32_t>((dy * Cfg::kBoxW + 8 * half + dx) * 16);
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma2_f16(tAcc + half * N, desc_noswz(start + 2 * k * Cfg::kLbo, Cfg::kLbo, Cfg::kSbo), bd + 2 * k,
                          idesc, (c | tap | k) ? 1u : 0u);
            }
            umma2_commit_mc(&b_empty[sb], 0x3);
            ++ib;
          }
          umma2_commit_mc(&a_empty[sa], 0x3);
          ++ia;
        }
        if (ok) umma2_commit_mc(&acc_full[ab], 0x3);
      }
    }
    __syncwarp();
  } else {
    // ---------------------------------------------------------- epilogue (both CTAs)
    const int q = warp & 3;
    const int m = q * 32 + lane;
    const int i = m >> 3, j = m & 7;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    const uint32_t acc_empty_leader[2] = {mapa_shared(smem_u32(&acc_empty[0]), 0),
                                          mapa_shared(smem_u32(&acc_empty[1]), 0)};
    for (int it = 0; it < my_tiles; ++it) {
      const uint32_t ab = it & 1;
      const int t = pair + it * npairs;
      int b, ty, tx;
      px_tile(t, b, ty, tx);
      const int og = t % n_oc;
      const int y = ty * Cfg::kTh + i;
      size_t pix[kHalves];
      bool valid[kHalves];
#pragma unroll
      for (int half = 0; half < kHalves; ++half) {
        const int x = tx * Cfg::kTw + 8 * half + j;
        valid[half] = b < B && y < H && x < W;
        pix[half] = valid[half] ? (static_cast<size_t>(b) * H + y) * W + x : 0;
      }
      if (!halo_epilogue<kHalves, N, 2>(tmem + ab * Cfg::kAccCols + lane_off, &acc_full[ab], (it >> 1) & 1,
                                        status, e, pix, valid, og * N))
        break;
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote_relaxed(acc_empty_leader[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // no CTA leaves while its peer may still signal its barriers
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc2(tmem, 512);
  }
}

template <int N, int kHalves>
int launch_halo2(const __half* X, int B, int H, int W, int IC, const __half* Wp, int OC, const EpiArgs& e,
                 int* status, cudaStream_t s, int sms) {
  using Cfg = Halo2Cfg<N, kHalves>;
  const int icp = conv_icp(IC);
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_tmap_nhwc_planes(&ta, X, B, H, W, IC, Cfg::kBoxW, Cfg::kBoxH))) return rc - 100;
  if ((rc = make_tmap_2d(&tb, Wp, OC, 9 * icp, 9 * icp, N / 2))) return rc - 200;
  static std::atomic<uint64_t> attr_set{0};  // one bit per device; first calls may race
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((attr_set.load() >> (dev & 63)) & 1)) {
    if (cudaFuncSetAttribute(k_conv3_halo2<N, kHalves>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::kSmem) !=
        cudaSuccess)
      return -3;
    attr_set.fetch_or(uint64_t(1) << (dev & 63));
  }
  const long n_px = static_cast<long>(B) * ((W + Cfg::kTw - 1) / Cfg::kTw) * ((H + Cfg::kTh - 1) / Cfg::kTh);
  const long tiles = ((n_px + 1) / 2) * (OC / N);
  if (tiles > 0x7fffffffL) return 1;
  int pairs = sms / 2;
  if (tiles < pairs) pairs = static_cast<int>(tiles);
  if (pairs <= 0) return 0;
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(2 * pairs, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = Cfg::kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, k_conv3_halo2<N, kHalves>, ta, tb, B, H, W, IC / 64, icp, OC / N, e, status) !=
      cudaSuccess)
    return -11;
  return cudaGetLastError() == cudaSuccess ? 0 : -11;
}

}  // namespace

// Returns 1 (nothing launched) when the shape or epilogue is not one this kernel
// covers, so the caller can take the implicit-GEMM path; 0 on launch; < 0 on error.
int conv3_halo(const __half* X, int B, int H, int W, int IC, const __half* Wp, int OC, const EpiArgs& e, int* status,
               cudaStream_t s) {
  if ((OC % kOCh && OC != 64) || OC <= 0 || IC % 64 || IC <= 0 || B <= 0 || H <= 0 || W <= 0) return 1;
  if (e.kind != kEpiF16 || e.q8 || e.rm_div || (e.res1 && e.res1_mod) || e.ld_out != OC ||
      (e.act != kActNone && e.act != kActRelu))
    return 1;
  if ((e.res1 && e.ld_res1 % 8) || (e.res2 && e.ld_res2 % 8)) return 1;
  if ((reinterpret_cast<uintptr_t>(X) & 15) || (reinterpret_cast<uintptr_t>(e.out) & 15) ||
      (e.out_relu && (reinterpret_cast<uintptr_t>(e.out_relu) & 15)) ||
      (e.bias && (reinterpret_cast<uintptr_t>(e.bias) & 15)) || (e.res1 && (reinterpret_cast<uintptr_t>(e.res1) & 15)) ||
      (e.res2 && (reinterpret_cast<uintptr_t>(e.res2) & 15)))
    return 1;
  int dev0 = 0, sms = 0;
  cudaGetDevice(&dev0);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev0);
  // Form: the CTA pair for output counts in groups of 256 (one 8-wide half of N = 256
  // per CTA; measured 6-10% faster than the 2-SM implicit GEMM on the DPT head's
  // shapes). For 128 outputs, by the number of 16 x 16 tiles (one image, batch 1):
  //   at most half the SMs (maps up to about 128 x 128): none; the implicit GEMM on
  //     one-CTA tiles, whose K split spreads the few tiles over more SMs, is faster
  //     (13.1-14.6 against 15.3-15.8 us with a residual at 37-112 px; 19.0 against 42.4
  //     us for 768 inputs at 19 x 19);
  //   up to the SMs (148 x 148): CTA pairs of one 8-wide half each, twice the CTAs of
  //     the one-CTA form, each with half the MMAs and half the epilogue (21.8 against
  //     22.9 us for the implicit GEMM);
  //   more: one CTA (the pair form with two halves of N = 128 per CTA was measured 4%
  //     slower on the batched maps).
  // $DA3B_CONV_HALO_PAIR=1 / =0 force the pair form with two halves / the one-CTA form.
  const char* pe = getenv("DA3B_CONV_HALO_PAIR");
  const int pmode = pe && pe[0] == '1' ? 1 : (pe && pe[0] == '0' ? 0 : -1);
  if (sms >= 2 && pmode != 0) {
    if (OC % 256 == 0) return launch_halo2<256, 1>(X, B, H, W, IC, Wp, OC, e, status, s, sms);
    if (OC == 128 && pmode == 1) return launch_halo2<128, 2>(X, B, H, W, IC, Wp, OC, e, status, s, sms);
    // 64 outputs (one image's out1, 128 -> 64 at 296 x 296): CTA pairs with two halves
    // of N = 64 per CTA on maps of more 16 x 16 tiles than SMs
    if (OC == 64) {
      const long t16 = static_cast<long>(B) * ((W + 15) / 16) * ((H + 15) / 16);
      return (t16 > sms || pmode == 1) ? launch_halo2<64, 2>(X, B, H, W, IC, Wp, OC, e, status, s, sms) : 1;
    }
    const long tiles16 = static_cast<long>(B) * ((W + 15) / 16) * ((H + 15) / 16);
    if (OC == 128 && 2 * tiles16 <= sms) return 1;
    if (OC == 128 && tiles16 <= sms) return launch_halo2<128, 1>(X, B, H, W, IC, Wp, OC, e, status, s, sms);
  }
  if (OC % kOCh) return 1;  // the one-CTA form serves groups of 128 outputs only
  const int icp = conv_icp(IC);
  CUtensorMap ta, tb;
  int rc;
  if ((rc = make_tmap_nhwc_planes(&ta, X, B, H, W, IC, kBoxW, kBoxH))) return rc - 100;
  if ((rc = make_tmap_2d(&tb, Wp, OC, 9 * icp, 9 * icp, kOCh))) return rc - 200;
  static std::atomic<uint64_t> attr_set{0};  // one bit per device; first calls may race
  int dev = 0;
  cudaGetDevice(&dev);
  if (!((attr_set.load() >> (dev & 63)) & 1)) {
    if (cudaFuncSetAttribute(k_conv3_halo, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess)
      return -3;
    attr_set.fetch_or(uint64_t(1) << (dev & 63));
  }
  const long n_tiles = static_cast<long>(B) * ((W + kTw - 1) / kTw) * ((H + kTh - 1) / kTh) * (OC / kOCh);
  if (n_tiles > 0x7fffffffL) return 1;
  const int grid = static_cast<int>(n_tiles < sms ? n_tiles : sms);
  k_conv3_halo<<<grid, kThreads, kSmem, s>>>(ta, tb, B, H, W, IC / 64, icp, OC / kOCh, e, status);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace da3b
