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
// f16 [rows][K], f16(d * q) like k_dequant_q8_0. A warp takes 32 consecutive blocks
// of one matrix: their 1088 source bytes come in as 16-byte coalesced loads into shared
// memory, then each lane converts one block and writes its 64 output bytes (the warp's
// stores are one contiguous 2 KB run). A matrix's last partial chunk reads per lane.
__device__ __forceinline__ void dequant_block32(const uint8_t* blk, __half* out) {
  const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(blk[0] | (blk[1] << 8))));
  uint4 packed[4];
  __half2* h = reinterpret_cast<__half2*>(packed);
#pragma unroll
  for (int i = 0; i < 16; ++i)
    h[i] = __floats2half2_rn(d * static_cast<float>(static_cast<int8_t>(blk[2 + 2 * i])),
                             d * static_cast<float>(static_cast<int8_t>(blk[3 + 2 * i])));
  uint4* o4 = reinterpret_cast<uint4*>(out);
#pragma unroll
  for (int i = 0; i < 4; ++i) o4[i] = packed[i];
}

__global__ void __launch_bounds__(256) k_dequant_q8_0_segs(Q8Segs g) {
  __shared__ __align__(16) uint8_t stage[8][1088];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const long gw = static_cast<long>(blockIdx.x) * 8 + warp, nw = static_cast<long>(gridDim.x) * 8;
  for (int k = 0; k < g.n; ++k) {
    const Q8Seg& sg = g.s[k];
    const long nblk = static_cast<long>(sg.rows) * sg.nblk;
    const long nch = (nblk + 31) / 32;
    for (long c = gw; c < nch; c += nw) {
      const long b0 = c * 32;
      const uint8_t* src = sg.q8 + static_cast<size_t>(b0) * 34;
      if (b0 + 32 <= nblk) {
        const uint4* s4 = reinterpret_cast<const uint4*>(src);
        uint4* d4 = reinterpret_cast<uint4*>(stage[warp]);
        for (int i = lane; i < 68; i += 32) d4[i] = s4[i];
        __syncwarp();
        dequant_block32(stage[warp] + lane * 34, sg.out + static_cast<size_t>(b0 + lane) * 32);
        __syncwarp();  // the stage is reused by this warp's next chunk
      } else if (b0 + lane < nblk) {
        dequant_block32(src + lane * 34, sg.out + static_cast<size_t>(b0 + lane) * 32);
      }
    }
  }
}

int dequant_q8_0_segs(const Q8Segs& g, cudaStream_t s) {
  if (g.n <= 0 || g.n > 4 || g.total <= 0) return -1;
  for (int k = 0; k < g.n; ++k)
    if (reinterpret_cast<uintptr_t>(g.s[k].q8) & 15 || reinterpret_cast<uintptr_t>(g.s[k].out) & 15) return -2;
  const long chunks = (g.total + 31) / 32;
  long blocks = (chunks + 7) / 8;
  if (blocks > 148 * 8) blocks = 148 * 8;
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
