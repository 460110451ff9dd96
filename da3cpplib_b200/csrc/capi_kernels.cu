// Kernel-level C ABI (include/da3b.h): thin validated wrappers over the launchers.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>
#include <string.h>

#include "da3b.h"
#include "kernels.h"
#include "ops.h"
#include "ptx.cuh"

namespace da3b {

// w_f32: torch conv layout [OC][IC][k][k]; out: [OC][k*k][icp] f16, zero padded.
__global__ void k_pack_conv(const float* __restrict__ w, int OC, int IC, int ks, int icp, __half* __restrict__ out) {
  const long total = static_cast<long>(OC) * ks * ks * icp;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int ic = static_cast<int>(i % icp);
    const int tap = static_cast<int>((i / icp) % (ks * ks));
    const int oc = static_cast<int>(i / (static_cast<long>(icp) * ks * ks));
    float v = 0.f;
    if (ic < IC) v = w[(static_cast<size_t>(oc) * IC + ic) * ks * ks + tap];
    out[i] = __float2half_rn(v);
  }
}

int pack_conv_weight(const float* w, int OC, int IC, int ks, __half* out, cudaStream_t s) {
  const int icp = conv_icp(IC);
  const long total = static_cast<long>(OC) * ks * ks * icp;
  const int threads = 256;
  long blocks = (total + threads - 1) / threads;
  if (blocks > 65535) blocks = 65535;
  k_pack_conv<<<static_cast<unsigned>(blocks), threads, 0, s>>>(w, OC, IC, ks, icp, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Wait-timeout probe: an mbarrier that nothing ever arrives on, waited on by both warps
// with the given limit through the same bounded wait every pipeline uses. When
// use_tmem is set, warp 0 first allocates 32 TMEM columns and frees them after the
// failed wait, as the pipelined kernels do on their timeout path. elapsed (optional)
// receives the nanoseconds thread 0 spent waiting.
__global__ void k_wait_probe(int* status, uint64_t limit_ns, int use_tmem, unsigned long long* elapsed) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ uint32_t slot;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_mbar_init();
  }
  if (use_tmem && warp == 0) tmem_alloc(&slot, 32);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint64_t t0 = globaltimer_ns();
  const bool ok = mbar_wait_warp(&bar, 0, status, kStatusTimeoutFull, limit_ns);
  const uint64_t t1 = globaltimer_ns();
  tc_fence_before();
  __syncthreads();
  if (use_tmem && warp == 0) {
    tc_fence_after();
    tmem_dealloc(slot, 32);
  }
  if (threadIdx.x == 0 && elapsed) *elapsed = ok ? 0ull : static_cast<unsigned long long>(t1 - t0);
}

// Tensor-pipe rate probe: one CTA per SM; thread 0 issues iters x 4 back-to-back
// M = 128, K = 16 f16 MMAs (N columns) into one TMEM accumulator, A from shared memory
// (A_TMEM = 0) or tensor memory (A_TMEM = 1), B from shared memory (zeros), and writes
// the cycles from the first issue to the completion of the last to cycles[blockIdx.x].
// The values in the A columns of tensor memory are whatever the allocation holds: the
// probe times the pipe, not the arithmetic.
template <int A_TMEM, int N>
__global__ void __launch_bounds__(128, 1) k_mma_rate(int iters, unsigned long long* cycles, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;          // [128][64] f16, 128B swizzle
  uint8_t* sB = smem + 16384;  // [256][64] f16
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + 16384 + 32768);
  uint32_t* slot = reinterpret_cast<uint32_t*>(bar + 1);
  for (int i = threadIdx.x; i < (16384 + 32768) / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(smem)[i] = make_uint4(0u, 0u, 0u, 0u);
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  if (threadIdx.x < 32) tmem_alloc(slot, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *slot;
  if (threadIdx.x == 0) {
    constexpr uint32_t id = umma_idesc_f16(128, N);
    const uint64_t ad = umma_desc_sw128(smem_u32(sA)), bd = umma_desc_sw128(smem_u32(sB));
    for (int k = 0; k < 4; ++k) {
      if (A_TMEM) umma_f16_tmem_a(tmem, tmem + 256 + 8 * k, bd + 2 * k, id, k > 0 ? 1u : 0u);
      else umma_f16(tmem, ad + 2 * k, bd + 2 * k, id, k > 0 ? 1u : 0u);
    }
    umma_commit(bar);
    bool ok = mbar_wait(bar, 0, status, kStatusTimeoutAccum);
    const unsigned long long t0 = clock64();
    for (int i = 0; i < iters && ok; ++i) {
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        if (A_TMEM) umma_f16_tmem_a(tmem, tmem + 256 + 8 * k, bd + 2 * k, id, 1u);
        else umma_f16(tmem, ad + 2 * k, bd + 2 * k, id, 1u);
      }
    }
    umma_commit(bar);
    if (ok) ok = mbar_wait(bar, 1, status, kStatusTimeoutAccum);
    cycles[blockIdx.x] = ok ? clock64() - t0 : 0ull;
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x < 32) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int A_TMEM, int N>
static int mma_rate(int ctas, int iters, unsigned long long* cycles, int* status, cudaStream_t s) {
  const int smem = 120 * 1024;  // one CTA per SM
  if (cudaFuncSetAttribute(k_mma_rate<A_TMEM, N>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return -3;
  k_mma_rate<A_TMEM, N><<<ctas, 128, smem, s>>>(iters, cycles, status);
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace da3b

using namespace da3b;

extern "C" {

DA3B_API int da3b_abi_version(void) { return 1; }

DA3B_API int da3b_device_status(void) {
  if (cudaDeviceSynchronize() != cudaSuccess) return -1;
  int* w = device_status_word();
  if (!w) return -2;
  int st = 0;
  if (read_and_reset_status(w, &st)) return -3;
  return st;
}

DA3B_API int da3b_dequant_q8_0(const void* q8, int rows, int K, void* w_f16, int ldw, void* stream) {
  if (!q8 || !w_f16) return -100;
  return dequant_q8_0(q8, rows, K, static_cast<__half*>(w_f16), ldw, static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_linear_f16(const void* x, int M, int K, int lda, const void* w, int N, int ldw, const float* bias,
                             int act, void* out, int ldo, void* stream) {
  if (!x || !w || !out || act < 0 || act > 3) return -100;
  int* st = device_status_word();
  if (!st) return -101;
  EpiArgs e = epi_default();
  e.kind = kEpiF16;
  e.act = act;
  e.bias = bias;
  e.out = static_cast<__half*>(out);
  e.ld_out = ldo;
  return gemm_linear(static_cast<const __half*>(x), M, K, lda, static_cast<const __half*>(w), N, ldw, 0, e, st,
                     static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_linear_resid_f32(const void* x, int M, int K, int lda, const void* w, int N, int ldw,
                                   const float* bias, const float* scale, float* resid, int ldr, void* stream) {
  if (!x || !w || !resid) return -100;
  int* st = device_status_word();
  if (!st) return -101;
  EpiArgs e = epi_default();
  e.kind = kEpiResid;
  e.bias = bias;
  e.scale = scale;
  e.resid = resid;
  e.ld_resid = ldr;
  return gemm_linear(static_cast<const __half*>(x), M, K, lda, static_cast<const __half*>(w), N, ldw, 0, e, st,
                     static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_repack_q8_0_planar(const void* q8, int N, int K, void* planar, void* stream) {
  if (!q8 || !planar) return -100;
  return repack_q8_0_planar(q8, N, K, planar, static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_dequant_q8p(const void* planar, int N, int K, void* w_f16, void* stream) {
  if (!planar || !w_f16 || N <= 0 || K <= 0 || K % 32) return -100;
  Q8Segs g;
  memset(&g, 0, sizeof(g));
  g.s[0] = Q8Seg{static_cast<const uint8_t*>(planar), static_cast<__half*>(w_f16), N, K / 32, 0};
  g.n = 1;
  g.total = static_cast<long>(N) * (K / 32);
  return dequant_q8p_segs(g, static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_linear_q8p_f16(const void* x, int M, int K, int lda, const void* planar, int N, const float* bias,
                                 int act, void* out, int ldo, void* stream) {
  if (!x || !planar || !out || act < 0 || act > 3) return -100;
  int* st = device_status_word();
  if (!st) return -101;
  EpiArgs e = epi_default();
  e.kind = kEpiF16;
  e.act = act;
  e.bias = bias;
  e.out = static_cast<__half*>(out);
  e.ld_out = ldo;
  return gemm_linear_q8p(static_cast<const __half*>(x), M, K, lda, static_cast<const uint8_t*>(planar), N, e, st,
                         static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_linear_q8p_resid_f32(const void* x, int M, int K, int lda, const void* planar, int N,
                                       const float* bias, const float* scale, float* resid, int ldr, void* stream) {
  if (!x || !planar || !resid) return -100;
  int* st = device_status_word();
  if (!st) return -101;
  EpiArgs e = epi_default();
  e.kind = kEpiResid;
  e.bias = bias;
  e.scale = scale;
  e.resid = resid;
  e.ld_resid = ldr;
  return gemm_linear_q8p(static_cast<const __half*>(x), M, K, lda, static_cast<const uint8_t*>(planar), N, e, st,
                         static_cast<cudaStream_t>(stream));
}

// Scratch for the transposed V of da3b_attention: one grow-only buffer per device,
// allocated by the library on first use (cudaMalloc) and reused by later calls.
static std::mutex g_vt_mu;
static void* g_vt_buf[64] = {nullptr};
static size_t g_vt_cap[64] = {0};

static __half* vt_scratch(size_t bytes) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_vt_mu);
  if (g_vt_cap[dev] < bytes) {
    if (g_vt_buf[dev]) {
      cudaDeviceSynchronize();
      cudaFree(g_vt_buf[dev]);
    }
    g_vt_buf[dev] = nullptr;
    g_vt_cap[dev] = 0;
    if (cudaMalloc(&g_vt_buf[dev], bytes) != cudaSuccess) return nullptr;
    g_vt_cap[dev] = bytes;
  }
  return static_cast<__half*>(g_vt_buf[dev]);
}

DA3B_API int da3b_attention(const void* qkv, int nseq, int seqlen, int heads, void* out, void* stream) {
  if (!qkv || !out || heads <= 0 || nseq < 0 || seqlen < 0) return -100;
  if (nseq == 0 || seqlen == 0) return 0;
  int* st = device_status_word();
  if (!st) return -101;
  const int D = heads * 64, ld = (seqlen + 7) / 8 * 8;
  __half* vt = vt_scratch(static_cast<size_t>(nseq) * D * ld * sizeof(__half));
  if (!vt) return -102;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = transpose_v(static_cast<const __half*>(qkv), nseq, seqlen, heads, D, vt, ld, s);
  if (rc) return rc;
  return attention_tc(static_cast<const __half*>(qkv), vt, ld, nseq, seqlen, heads, D, static_cast<__half*>(out), 0,
                      st, s);
}

DA3B_API int da3b_debug_wait_timeout(unsigned long long limit_ns, int use_tmem, int* status_dev,
                                     unsigned long long* elapsed_dev, void* stream) {
  if (limit_ns == 0 || limit_ns > 1000000000ull) return -100;  // at most 1 s
  int* st = status_dev ? status_dev : device_status_word();
  if (!st) return -101;
  k_wait_probe<<<1, 64, 0, static_cast<cudaStream_t>(stream)>>>(st, limit_ns, use_tmem ? 1 : 0, elapsed_dev);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

DA3B_API int da3b_debug_mma_cycles(int n, int a_tmem, int iters, int ctas, unsigned long long* cycles_dev, void* stream) {
  if (!cycles_dev || iters <= 0 || iters > 100000 || ctas <= 0 || ctas > 1024) return -100;
  int* st = device_status_word();
  if (!st) return -101;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
#define DA3B_MMA_RATE(NN) \
  if (n == NN) return a_tmem ? mma_rate<1, NN>(ctas, iters, cycles_dev, st, s) : mma_rate<0, NN>(ctas, iters, cycles_dev, st, s);
  DA3B_MMA_RATE(64)
  DA3B_MMA_RATE(80)
  DA3B_MMA_RATE(128)
  DA3B_MMA_RATE(256)
#undef DA3B_MMA_RATE
  return -100;
}

DA3B_API int da3b_linear_tiles(int M, int N, int K, int* bn, int* ksplit) {
  return gemm_linear_tiles(M, N, K, bn, ksplit);
}

DA3B_API int da3b_set_attention_split(int n) {
  set_attention_split(n);
  return 0;
}

DA3B_API int da3b_transpose_v(const void* qkv, int nseq, int seqlen, int heads, void* vt, int ld_vt, void* stream) {
  if (!qkv || !vt || heads <= 0 || nseq < 0 || seqlen < 0 || ld_vt < seqlen || ld_vt % 8) return -100;
  if (nseq == 0 || seqlen == 0) return 0;
  return transpose_v(static_cast<const __half*>(qkv), nseq, seqlen, heads, heads * 64, static_cast<__half*>(vt), ld_vt,
                     static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_attention_vt(const void* qkv, const void* vt, int ld_vt, int nseq, int seqlen, int heads, void* out,
                               void* stream) {
  if (!qkv || !vt || !out || heads <= 0 || nseq < 0 || seqlen < 0) return -100;
  if (nseq == 0 || seqlen == 0) return 0;
  int* st = device_status_word();
  if (!st) return -101;
  return attention_tc(static_cast<const __half*>(qkv), static_cast<const __half*>(vt), ld_vt, nseq, seqlen, heads,
                      heads * 64, static_cast<__half*>(out), 0, st, static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_upsample_nhwc(const void* in, int B, int hs, int ws, int C, void* out, int H, int W, void* stream) {
  if (!in || !out || B < 0 || hs <= 0 || ws <= 0 || H <= 0 || W <= 0 || C <= 0 || C % 8) return -100;
  return upsample_ac(static_cast<const __half*>(in), B, hs, ws, C, static_cast<__half*>(out), H, W, nullptr,
                     static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_pack_conv_weight(const float* w_f32, int OC, int IC, int ksize, void* w_packed, void* stream) {
  if (!w_f32 || !w_packed || OC <= 0 || IC <= 0 || ksize <= 0) return -100;
  return pack_conv_weight(w_f32, OC, IC, ksize, static_cast<__half*>(w_packed), static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_conv_nhwc(const void* x, int B, int H, int W, int IC, const void* w_packed, int OC, int ksize,
                            const float* bias, const void* res1, const void* res2, int act, void* out, void* out_relu,
                            void* stream) {
  if (!x || !w_packed || !out || act < 0 || act > 2) return -100;
  int* st = device_status_word();
  if (!st) return -101;
  EpiArgs e = epi_default();
  e.kind = kEpiF16;
  e.act = act;
  e.bias = bias;
  e.out = static_cast<__half*>(out);
  e.ld_out = OC;
  e.out_relu = static_cast<__half*>(out_relu);
  e.res1 = static_cast<const __half*>(res1);
  e.ld_res1 = OC;
  e.res2 = static_cast<const __half*>(res2);
  e.ld_res2 = OC;
  return conv_nhwc(static_cast<const __half*>(x), B, H, W, IC, static_cast<const __half*>(w_packed), OC, ksize, 0, e,
                   st, static_cast<cudaStream_t>(stream));
}

DA3B_API int da3b_output_conv2(const void* feat, int B, int hs, int ws, int C, const void* pe, int H, int W,
                               const void* w_packed, const float* out2a_bias, const float* out2b_w,
                               const float* out2b_b, int od, const int* act, float scale, float* const* out,
                               int fused, void* stream) {
  if (!feat || !w_packed || !out2b_w || !out2b_b || !act || !out || od < 1 || od > 8) return -100;
  int* st = device_status_word();
  if (!st) return -101;
  EpiArgs e = epi_default();
  e.kind = kEpiOut2;
  e.bias = out2a_bias;
  e.o2_w = out2b_w;
  e.o2_b = out2b_b;
  e.o2_dim = od;
  e.o2_scale = scale;
  for (int i = 0; i < od; ++i) {
    if (act[i] < 0 || act[i] > 4 || !out[i]) return -100;
    e.o2_act[i] = act[i];
    e.o2_out[i] = out[i];
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const __half* x = static_cast<const __half*>(feat);
  const __half* wp = static_cast<const __half*>(w_packed);
  if (fused) return up_out2(x, B, hs, ws, C, static_cast<const __half*>(pe), H, W, wp, conv_icp(C), e, st, s);
  __half* up = nullptr;
  if (cudaMallocAsync(reinterpret_cast<void**>(&up), static_cast<size_t>(B) * H * W * C * 2, s) != cudaSuccess)
    return -102;
  int rc = upsample_ac(x, B, hs, ws, C, up, H, W, static_cast<const __half*>(pe), s);
  if (!rc) rc = conv_nhwc(up, B, H, W, C, wp, 32, 3, 32, e, st, s);
  cudaFreeAsync(up, s);
  return rc;
}

}  // extern "C"
