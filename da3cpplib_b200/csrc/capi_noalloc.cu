// da3b_attention_noalloc: the attention entry point for callers that cannot let the
// library allocate device memory. Its only scratch, the transposed V, lives in a
// fixed file-scope device array; nothing here calls cudaMalloc, cudaFree or any other
// allocating routine, and the caller supplies the status word.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "da3b.h"
#include "kernels.h"

namespace {

// V^T scratch of DA3B_NOALLOC_VT_BYTES, allocated with the module (zero-initialised
// at load, but nothing relies on that: every element a call reads is written by the
// same call's transpose first).
__device__ __align__(256) unsigned char g_vt_static[DA3B_NOALLOC_VT_BYTES];

// Address of g_vt_static per device, resolved once (cudaGetSymbolAddress).
std::mutex g_mu;
void* g_addr[64] = {nullptr};

void* vt_static_address(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_addr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_vt_static) != cudaSuccess) return nullptr;
    g_addr[dev] = p;
  }
  return g_addr[dev];
}

}  // namespace

extern "C" {

DA3B_API int da3b_attention_noalloc(const void* qkv, int nseq, int seqlen, int heads, void* out, int* status_dev,
                                    void* stream) {
  if (!qkv || !out || !status_dev || heads <= 0 || nseq < 0 || seqlen < 0) return -100;
  if (nseq == 0 || seqlen == 0) return 0;
  const int D = heads * 64, ld = (seqlen + 7) / 8 * 8;
  const double need = static_cast<double>(nseq) * D * ld * sizeof(__half);
  if (need > static_cast<double>(DA3B_NOALLOC_VT_BYTES)) return DA3B_ERR_NOALLOC_TOO_LARGE;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -101;
  __half* vt = static_cast<__half*>(vt_static_address(dev));
  if (!vt) return -102;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int rc = da3b::transpose_v(static_cast<const __half*>(qkv), nseq, seqlen, heads, D, vt, ld, s);
  if (rc) return rc;
  return da3b::attention_tc(static_cast<const __half*>(qkv), vt, ld, nseq, seqlen, heads, D,
                            static_cast<__half*>(out), 0, status_dev, s);
}

}  // extern "C"
