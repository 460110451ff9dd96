// Q8_0 x Q8_0 linear on the int8 tensor cores (tcgen05.mma kind::i8), bit-exact with
// ggml's CPU dot product.
//
// The reference's linear() is ggml_mul_mat(W_q8_0, x_f32) (src/ggml_extend.hpp:6-10).
// On the CPU ggml quantises every 32-element block of x to Q8_0 (d = amax / 127, q =
// round(x / d), d kept as f16) and computes, per output, sum over blocks b in order of
// float(isum_b) * (d_w,b * d_x,b), where isum_b is the exact int32 dot product of the
// block's 32 int8 pairs (vec_dot_q8_0_q8_0, generic form).
//
// Here one kind::i8 MMA (K = 32 int8 = one Q8_0 block) writes the int32 block dots of a
// 128-row x 128-column tile into its own TMEM buffer (four buffers, ping-pong); the
// epilogue warps read each block's int32 results and accumulate
//   acc = acc + float(isum) * (d_w * d_x)
// with explicitly rounded f32 multiplies and adds in block order, so every output equals
// the scalar ggml result bit for bit. The per-block rescale is the cost of this route:
// three f32 operations and one conversion per (row, column, block) on the CUDA cores
// against 32 multiply-adds of tensor-core work, so the epilogue, not the int8 MMA, bounds
// the kernel (see the microbench part A8). The product path uses f16 weights and the
// kind::f16 GEMM instead; this kernel measures the int8 route and serves as the
// reference-exact linear.
//
// Roles (192 threads, one CTA per 128 x 128 output tile):
//   warp 0     TMA: per stage of 4 blocks (128 K bytes) the x tile [128][128 B], the
//              weight tile [128][128 B] (128B swizzle) and the weights' block scales
//              [4][128] f32, into a 4-deep ring;
//   warp 1     allocates 512 TMEM columns; one thread issues one MMA per block into
//              buffer b % 4 once the epilogue released it;
//   warps 2-5  epilogue: thread = output row (its TMEM lane); 128 f32 accumulators in
//              registers; per block four 32-column TMEM loads, the rescale-accumulate,
//              then release of the buffer (and of the stage after its fourth block).
// Every wait is bounded (ptx.cuh); on a timeout the kernel records a status and exits.
#include <atomic>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "da3b.h"
#include "ops.h"
#include "ptx.cuh"

namespace da3b {

namespace {

constexpr int kTileM = 128, kTileN = 128;
constexpr int kKB = 128;                         // K bytes (int8 elements) per stage: 4 blocks
constexpr int kStages = 4;
constexpr int kABytes = kTileM * kKB;            // 16 KB
constexpr int kBBytes = kTileN * kKB;            // 16 KB
constexpr int kSBytes = 4 * kTileN * 4;          // weight scales of the stage's 4 blocks
constexpr int kStageBytes = kABytes + kBBytes + kSBytes;
constexpr int kNBuf = 4;                         // TMEM int32 block-dot buffers
constexpr uint32_t kTmemCols = kNBuf * kTileN;   // 512
constexpr int kSmem = 1024 + kStages * kStageBytes + 256;

// Instruction descriptor for kind::i8: signed 8-bit A and B, s32 accumulator, both
// K-major, M = 128, N = 128.
__host__ __device__ constexpr uint32_t umma_idesc_i8(int M, int N) {
  return (2u << 4)                                  // D format: s32
         | (1u << 7) | (1u << 10)                   // A, B format: signed 8-bit
         | (static_cast<uint32_t>(N >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

__device__ __forceinline__ void umma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, 0, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc)
      : "memory");
}

__global__ void __launch_bounds__(192, 1)
    k_q8q8_i8(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const __grid_constant__ CUtensorMap tmS, const float* __restrict__ dx, int M, int N, int K,
              const float* __restrict__ bias, float* __restrict__ y, int ldy, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* full = bars;                      // [kStages] TMA bytes landed
  uint64_t* empty = full + kStages;           // [kStages] MMA done (1) + scales read (4 warps)
  uint64_t* buf_full = empty + kStages;       // [kNBuf] block dots in TMEM
  uint64_t* buf_empty = buf_full + kNBuf;     // [kNBuf] epilogue read them (4 warps)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(buf_empty + kNBuf);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kTileM, n0 = blockIdx.y * kTileN;
  const int nks = K / kKB, nb = K / 32;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1 + 4);
    }
    for (int b = 0; b < kNBuf; ++b) {
      mbar_init(&buf_full[b], 1);
      mbar_init(&buf_empty[b], 4);
    }
    fence_mbar_init();
    prefetch_tmap(&tmA);
    prefetch_tmap(&tmB);
    prefetch_tmap(&tmS);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int j = 0; j < nks; ++j) {
        const int s = j % kStages;
        if (!mbar_wait(&empty[s], ((j / kStages) & 1) ^ 1u, status, kStatusTimeoutEmpty)) break;
        uint8_t* st = smem + s * kStageBytes;
        mbar_arrive_expect_tx(&full[s], kStageBytes);
        tma_load_2d(st, &tmA, &full[s], j * kKB, m0);
        tma_load_2d(st + kABytes, &tmB, &full[s], j * kKB, n0);
        tma_load_2d(st + kABytes + kBBytes, &tmS, &full[s], n0, 4 * j);
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_i8(kTileM, kTileN);
      bool ok = true;
      for (int j = 0; j < nks && ok; ++j) {
        const int s = j % kStages;
        if (!mbar_wait(&full[s], (j / kStages) & 1, status, kStatusTimeoutFull)) break;
        tc_fence_after();
        const uint8_t* st = smem + s * kStageBytes;
        const uint64_t adesc = umma_desc_sw128(smem_u32(st));
        const uint64_t bdesc = umma_desc_sw128(smem_u32(st + kABytes));
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          const int b = 4 * j + kb, bb = b % kNBuf;
          if (!mbar_wait(&buf_empty[bb], ((b / kNBuf) & 1) ^ 1u, status, kStatusTimeoutAccumFree)) {
            ok = false;
            break;
          }
          tc_fence_after();
          umma_i8(tmem + bb * kTileN, adesc + 2 * kb, bdesc + 2 * kb, idesc);
          umma_commit(&buf_full[bb]);
        }
        umma_commit(&empty[s]);
      }
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int r = q * 32 + lane;                  // output row within the tile == TMEM lane
    const int m = m0 + r;
    const uint32_t lane_off = static_cast<uint32_t>(q * 32) << 16;
    float acc[kTileN];
#pragma unroll
    for (int i = 0; i < kTileN; ++i) acc[i] = 0.f;
    bool ok = true;
    for (int j = 0; j < nks && ok; ++j) {
      const int s = j % kStages;
      const float* sc = reinterpret_cast<const float*>(smem + s * kStageBytes + kABytes + kBBytes);
      float4 dxv = make_float4(0.f, 0.f, 0.f, 0.f);
      if (m < M) dxv = *reinterpret_cast<const float4*>(dx + static_cast<size_t>(m) * nb + 4 * j);
      const float dxs[4] = {dxv.x, dxv.y, dxv.z, dxv.w};
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        const int b = 4 * j + kb, bb = b % kNBuf;
        if (!mbar_wait_warp(&buf_full[bb], (b / kNBuf) & 1, status, kStatusTimeoutAccum)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float* scb = sc + kb * kTileN;
#pragma unroll
        for (int c = 0; c < kTileN / 32; ++c) {
          uint32_t v[32];
          tmem_ld32(tmem + bb * kTileN + c * 32 + lane_off, v);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float prod = __fmul_rn(scb[c * 32 + i], dxs[kb]);
            acc[c * 32 + i] = __fadd_rn(acc[c * 32 + i], __fmul_rn(__int2float_rn(static_cast<int>(v[i])), prod));
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&buf_empty[bb]);
        if (kb == 3 && lane == 0) mbar_arrive(&empty[s]);
      }
    }
    if (__all_sync(0xffffffffu, ok) && m < M) {
      float* yr = y + static_cast<size_t>(m) * ldy + n0;
#pragma unroll
      for (int i = 0; i < kTileN; i += 4) {
        if (n0 + i >= N) break;
        float4 o;
        o.x = __fadd_rn(acc[i], bias ? bias[n0 + i] : 0.f);
        o.y = __fadd_rn(acc[i + 1], bias ? bias[n0 + i + 1] : 0.f);
        o.z = __fadd_rn(acc[i + 2], bias ? bias[n0 + i + 2] : 0.f);
        o.w = __fadd_rn(acc[i + 3], bias ? bias[n0 + i + 3] : 0.f);
        *reinterpret_cast<float4*>(yr + i) = o;
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ggml's reference Q8_0 quantiser per 32-element block of f32 rows: d = amax / 127,
// id = 1 / d (0 when d == 0), q = round-half-away(x * id); the scale is kept as the f16
// value it is stored as, returned as f32. One warp per (row, block): lane = element.
__global__ void k_quantize_q8_0(const float* __restrict__ x, int M, int K, int8_t* __restrict__ q,
                                float* __restrict__ d) {
  const int nb = K / 32;
  const long blocks = static_cast<long>(M) * nb;
  const int lane = threadIdx.x & 31;
  for (long wb = (static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; wb < blocks;
       wb += (static_cast<long>(gridDim.x) * blockDim.x) >> 5) {
    const int m = static_cast<int>(wb / nb), b = static_cast<int>(wb % nb);
    const float v = x[static_cast<size_t>(m) * K + b * 32 + lane];
    float amax = fabsf(v);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    const float dd = __fdiv_rn(amax, 127.0f);
    const float id = dd != 0.f ? __fdiv_rn(1.0f, dd) : 0.0f;
    q[static_cast<size_t>(m) * K + b * 32 + lane] = static_cast<int8_t>(roundf(__fmul_rn(v, id)));
    if (lane == 0) d[static_cast<size_t>(m) * nb + b] = __half2float(__float2half_rn(dd));
  }
}

// GGUF Q8_0 rows [N][K/32][34 B] (f16 d, then 32 int8) -> int8 [N][K] and the scales
// as f32, transposed to [K/32][N] (the layout the kernel's scale tiles are read in).
__global__ void k_repack_q8_0(const uint8_t* __restrict__ raw, int N, int K, int8_t* __restrict__ qw,
                              float* __restrict__ dwT) {
  const int nb = K / 32;
  const long blocks = static_cast<long>(N) * nb;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < blocks;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(i / nb), b = static_cast<int>(i % nb);
    const uint8_t* blk = raw + static_cast<size_t>(i) * 34;
    const uint16_t dh = static_cast<uint16_t>(blk[0] | (blk[1] << 8));
    dwT[static_cast<size_t>(b) * N + n] = __half2float(__ushort_as_half(dh));
    int8_t* dst = qw + static_cast<size_t>(n) * K + b * 32;
#pragma unroll
    for (int k = 0; k < 32; ++k) dst[k] = static_cast<int8_t>(blk[2 + k]);
  }
}

}  // namespace

int quantize_q8_0_rows(const float* x, int M, int K, int8_t* q, float* d, cudaStream_t s) {
  if (M <= 0 || K <= 0 || K % 32) return -1;
  const long warps = static_cast<long>(M) * (K / 32);
  long blocks = (warps * 32 + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  k_quantize_q8_0<<<static_cast<unsigned>(blocks), 256, 0, s>>>(x, M, K, q, d);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int repack_q8_0(const void* raw, int N, int K, int8_t* qw, float* dwT, cudaStream_t s) {
  if (N <= 0 || K <= 0 || K % 32) return -1;
  const long n = static_cast<long>(N) * (K / 32);
  long blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  k_repack_q8_0<<<static_cast<unsigned>(blocks), 256, 0, s>>>(static_cast<const uint8_t*>(raw), N, K, qw, dwT);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

int linear_q8q8_i8(const int8_t* qx, const float* dx, int M, int K, const int8_t* qw, const float* dwT, int N,
                   const float* bias, float* y, int ldy, int* status, cudaStream_t s) {
  if (M <= 0 || N <= 0) return 0;
  if (K % kKB || N % kTileN || ldy < N || (ldy % 4) || (reinterpret_cast<uintptr_t>(y) & 15) ||
      (reinterpret_cast<uintptr_t>(dx) & 15))
    return -1;
  CUtensorMap ta, tb, ts;
  int rc;
  if ((rc = make_tmap_2d_typed(&ta, qx, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, M, K, K, kKB, kTileM,
                               CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc - 100;
  if ((rc = make_tmap_2d_typed(&tb, qw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, N, K, K, kKB, kTileN,
                               CU_TENSOR_MAP_SWIZZLE_128B)))
    return rc - 200;
  if ((rc = make_tmap_2d_typed(&ts, dwT, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, K / 32, N, N, kTileN, 4,
                               CU_TENSOR_MAP_SWIZZLE_NONE)))
    return rc - 300;
  static std::atomic<uint64_t> attr_set{0};  // one bit per device; first calls may race
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(attr_set.load() & bit)) {
    if (cudaFuncSetAttribute(k_q8q8_i8, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess) return -3;
    attr_set.fetch_or(bit);
  }
  dim3 grid((M + kTileM - 1) / kTileM, N / kTileN);
  k_q8q8_i8<<<grid, 192, kSmem, s>>>(ta, tb, ts, dx, M, N, K, bias, y, ldy, status);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace da3b

using namespace da3b;

extern "C" {

DA3B_API int da3b_quantize_q8_0(const float* x, int M, int K, void* q_int8, float* d, void* stream) {
  if (!x || !q_int8 || !d) return -100;
  return quantize_q8_0_rows(x, M, K, static_cast<int8_t*>(q_int8), d, static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_repack_q8_0(const void* q8, int N, int K, void* qw_int8, float* dw_t, void* stream) {
  if (!q8 || !qw_int8 || !dw_t) return -100;
  return repack_q8_0(q8, N, K, static_cast<int8_t*>(qw_int8), dw_t, static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_linear_q8q8_i8(const void* qx, const float* dx, int M, int K, const void* qw, const float* dw_t,
                                 int N, const float* bias, float* y, int ldy, void* stream) {
  if (!qx || !dx || !qw || !dw_t || !y || M < 0 || K <= 0 || N <= 0) return -100;
  int* st = device_status_word();
  if (!st) return -101;
  return linear_q8q8_i8(static_cast<const int8_t*>(qx), dx, M, K, static_cast<const int8_t*>(qw), dw_t, N, bias, y,
                        ldy, st, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
