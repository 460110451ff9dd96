// Memory-bound helper kernels: Q8_0 weight repack, casts, and the per-device status word.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "ops.h"

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

// One launch dequantising up to four Q8_0 matrices (a ViT block's linears) into dense
// f16 [rows][K]: one thread per 32-element block, f16(d * q) like k_dequant_q8_0.
__global__ void k_dequant_q8_0_segs(Q8Segs g) {
  for (long idx = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; idx < g.total;
       idx += static_cast<long>(gridDim.x) * blockDim.x) {
    int k = 0;
    while (k + 1 < g.n && idx >= g.s[k + 1].first) ++k;
    const Q8Seg& sg = g.s[k];
    const long li = idx - sg.first;
    const int r = static_cast<int>(li / sg.nblk), b = static_cast<int>(li % sg.nblk);
    const uint8_t* blk = sg.q8 + static_cast<size_t>(li) * 34;
    const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
    uint4 packed[4];
    __half2* h = reinterpret_cast<__half2*>(packed);
#pragma unroll
    for (int i = 0; i < 16; ++i)
      h[i] = __floats2half2_rn(d * static_cast<float>(static_cast<int8_t>(blk[2 + 2 * i])),
                               d * static_cast<float>(static_cast<int8_t>(blk[3 + 2 * i])));
    uint4* o4 = reinterpret_cast<uint4*>(sg.out + static_cast<size_t>(r) * sg.nblk * 32 + b * 32);
#pragma unroll
    for (int i = 0; i < 4; ++i) o4[i] = packed[i];
  }
}

int dequant_q8_0_segs(const Q8Segs& g, cudaStream_t s) {
  if (g.n <= 0 || g.n > 4 || g.total <= 0) return -1;
  long blocks = (g.total + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  k_dequant_q8_0_segs<<<static_cast<unsigned>(blocks), 256, 0, s>>>(g);
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
