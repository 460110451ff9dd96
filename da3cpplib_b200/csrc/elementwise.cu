// Memory-bound helper kernels: Q8_0 weight repacks and dequantisation, casts, and the
// per-device status word.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>
#include <mutex>

#include "ops.h"
#include "q8planar.cuh"

namespace da3b {

// GGUF Q8_0 row = K/32 blocks of {f16 d; int8 q[32]} (34 bytes, no padding).
// out[r][k] = f16(d * q) for k < K, zero for K <= k < ldo. One thread per (row, block).
__global__ void k_dequant_q8_0(const uint8_t* __restrict__ q8, int rows, int nblk, __half* __restrict__ out, int ldo) {
  const long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int nb_out = ldo / 32;
  if (idx >= static_cast<long>(rows) * nb_out) return;
  const int r = static_cast<int>(idx / nb_out), b = static_cast<int>(idx % nb_out);
  __half* o = out + static_cast<size_t>(r) * ldo + b * 32;
  uint4 packed[4];
  __half2* h = reinterpret_cast<__half2*>(packed);
  if (b < nblk) {
    const uint8_t* blk = q8 + (static_cast<size_t>(r) * nblk + b) * 34;
    const float d = __half2float(*reinterpret_cast<const __half*>(blk));
    const int8_t* q = reinterpret_cast<const int8_t*>(blk + 2);
#pragma unroll
    for (int i = 0; i < 16; ++i) h[i] = __floats2half2_rn(d * static_cast<float>(q[2 * i]), d * static_cast<float>(q[2 * i + 1]));
  } else {
#pragma unroll
    for (int i = 0; i < 16; ++i) h[i] = __floats2half2_rn(0.f, 0.f);
  }
  uint4* o4 = reinterpret_cast<uint4*>(o);
#pragma unroll
  for (int i = 0; i < 4; ++i) o4[i] = packed[i];
}

int dequant_q8_0(const void* q8, int rows, int K, __half* out, int ldo, cudaStream_t s) {
  if (K % 32 || ldo % 32 || ldo < K || rows <= 0) return -1;
  if (reinterpret_cast<uintptr_t>(out) & 15) return -2;
  const long n = static_cast<long>(rows) * (ldo / 32);
  const int threads = 256;
  k_dequant_q8_0<<<static_cast<unsigned>((n + threads - 1) / threads), threads, 0, s>>>(
      static_cast<const uint8_t*>(q8), rows, K / 32, out, ldo);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

// GGUF Q8_0 rows -> planar Q8_0 (q8planar.cuh), one thread per (row, block). Load time.
__global__ void k_repack_q8_0_planar(const uint8_t* __restrict__ raw, int N, int K, uint8_t* __restrict__ planar) {
  const int nb = K / 32;
  const long blocks = static_cast<long>(N) * nb;
  __half* dplane = reinterpret_cast<__half*>(planar + static_cast<size_t>(N) * K);
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < blocks;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int n = static_cast<int>(i / nb), b = static_cast<int>(i % nb);
    const uint16_t* blk = reinterpret_cast<const uint16_t*>(raw + static_cast<size_t>(i) * 34);  // 2-byte aligned
    dplane[static_cast<size_t>(b) * N + n] = __ushort_as_half(blk[0]);
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) w[k] = static_cast<uint32_t>(blk[1 + 2 * k]) | (static_cast<uint32_t>(blk[2 + 2 * k]) << 16);
    uint4* dst = reinterpret_cast<uint4*>(planar + static_cast<size_t>(n) * K + b * 32);
    dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
    dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
  }
}

int repack_q8_0_planar(const void* raw, int N, int K, void* planar, cudaStream_t s) {
  if (N <= 0 || K <= 0 || K % 32 || (reinterpret_cast<uintptr_t>(raw) & 1) || (reinterpret_cast<uintptr_t>(planar) & 15))
    return -1;
  const long n = static_cast<long>(N) * (K / 32);
  long blocks = (n + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  k_repack_q8_0_planar<<<static_cast<unsigned>(blocks), 256, 0, s>>>(static_cast<const uint8_t*>(raw), N, K,
                                                                      static_cast<uint8_t*>(planar));
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

// One launch dequantising up to four planar Q8_0 matrices (a ViT block's linears) into
// dense f16 [rows][K]: a thread takes 16 consecutive weights of a row (one 16-byte load
// of the q plane, its block's scale, two 16-byte stores), consecutive threads
// consecutive pieces, so every load and store of a warp is one contiguous run.
__global__ void __launch_bounds__(256) k_dequant_q8p_segs(Q8Segs g) {
  q8p_segs_dequant(g, static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x, static_cast<long>(gridDim.x) * blockDim.x);
}

int dequant_q8p_segs(const Q8Segs& g, cudaStream_t s) {
  if (g.n <= 0 || g.n > 4 || g.total <= 0) return -1;
  for (int k = 0; k < g.n; ++k)
    if (reinterpret_cast<uintptr_t>(g.s[k].q8) & 15 || reinterpret_cast<uintptr_t>(g.s[k].out) & 15) return -2;
  const long blocks = q8p_segs_blocks(g);
  k_dequant_q8p_segs<<<static_cast<unsigned>(blocks), 256, 0, s>>>(g);
  return cudaGetLastError() == cudaSuccess ? 0 : -3;
}

__global__ void k_f32_to_f16(const float* __restrict__ in, __half* __restrict__ out, size_t n) {
  for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<size_t>(gridDim.x) * blockDim.x)
    out[i] = __float2half_rn(in[i]);
}

int f32_to_f16(const float* in, __half* out, size_t n, cudaStream_t s) {
  if (n == 0) return 0;
  const int threads = 256;
  const unsigned blocks = static_cast<unsigned>((n + threads - 1) / threads < 65535 ? (n + threads - 1) / threads : 65535);
  k_f32_to_f16<<<blocks, threads, 0, s>>>(in, out, n);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ------------------------------------------------------------------ status word
static std::mutex g_status_mu;
static int* g_status_words[64] = {nullptr};

int* device_status_word() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_status_mu);
  if (!g_status_words[dev]) {
    int* p = nullptr;
    if (cudaMalloc(&p, sizeof(int)) != cudaSuccess) return nullptr;
    if (cudaMemset(p, 0, sizeof(int)) != cudaSuccess) return nullptr;
    g_status_words[dev] = p;
  }
  return g_status_words[dev];
}

int read_and_reset_status(int* word, int* out_status) {
  int v = 0;
  if (cudaMemcpy(&v, word, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (v != 0 && cudaMemset(word, 0, sizeof(int)) != cudaSuccess) return -1;
  *out_status = v;
  return 0;
}

}  // namespace da3b
