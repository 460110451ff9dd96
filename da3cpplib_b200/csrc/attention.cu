// Fused bidirectional flash attention (head_dim 64, f16 in, f32 softmax/accumulate).
//
// Replaces the reference's ggml_flash_attn_ext with F32 precision
// (src/attention.cpp:63-77): per (query tile, head, sequence) one CTA of 8 warps,
// each warp owning 16 query rows; K/V tiles of 64 keys stream through a
// cp.async double buffer; S = Q K^T, the online softmax (base-2, scale folded)
// and O += P V never leave registers. Keys past the sequence end are masked;
// rows past it are not stored. Shared tiles use a 16-byte XOR swizzle so every
// ldmatrix phase is bank-conflict free.
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "kernels.h"

namespace da3b {

namespace {

constexpr int kQ = 128;   // query rows per CTA
constexpr int kKV = 64;   // keys per tile
constexpr int kHD = 64;   // head dim

__device__ __forceinline__ uint32_t s_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// row r, 16-byte chunk c of a [rows][64] f16 tile -> element offset
__device__ __forceinline__ int swz(int r, int c) { return r * kHD + ((c ^ (r & 7)) << 3); }

__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s_u32(p)));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(s_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Load a [rows][64] tile (row stride ld elements) whose first row is `row0` of a
// sequence of `seqlen` rows; rows past the end are zero-filled.
template <int ROWS>
__device__ __forceinline__ void load_tile(__half* dst, const __half* src, int ld, int row0, int seqlen) {
  for (int i = threadIdx.x; i < ROWS * 8; i += blockDim.x) {
    const int r = i >> 3, c = i & 7;
    const int row = row0 + r;
    const int valid = row < seqlen;
    const __half* g = src + static_cast<size_t>(valid ? row : 0) * ld + c * 8;
    cp_async16(dst + swz(r, c), g, valid ? 16 : 0);
  }
}

__global__ void __launch_bounds__(256, 2)
    k_flash_attn(const __half* __restrict__ qkv, int seqlen, int H, int D, __half* __restrict__ out, float sl2,
                 int q8) {
  __shared__ __align__(128) __half sQ[kQ * kHD];
  __shared__ __align__(128) __half sK[2][kKV * kHD];
  __shared__ __align__(128) __half sV[2][kKV * kHD];
  const int qt = blockIdx.x, h = blockIdx.y, sq = blockIdx.z;
  const int ld = 3 * D;
  const __half* Qg = qkv + static_cast<size_t>(sq) * seqlen * ld + h * kHD;
  const __half* Kg = Qg + D;
  const __half* Vg = Qg + 2 * D;
  const int q0 = qt * kQ;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;

  load_tile<kQ>(sQ, Qg, ld, q0, seqlen);
  load_tile<kKV>(sK[0], Kg, ld, 0, seqlen);
  load_tile<kKV>(sV[0], Vg, ld, 0, seqlen);
  cp_async_commit();

  const int nkt = (seqlen + kKV - 1) / kKV;
  uint32_t qf[4][4];
  float o[8][4];
#pragma unroll
  for (int i = 0; i < 8; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

  for (int kt = 0; kt < nkt; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < nkt) {
      load_tile<kKV>(sK[buf ^ 1], Kg, ld, (kt + 1) * kKV, seqlen);
      load_tile<kKV>(sV[buf ^ 1], Vg, ld, (kt + 1) * kKV, seqlen);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (kt == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) ldsm_x4(qf[kk], sQ + swz(warp * 16 + (lane & 15), kk * 2 + (lane >> 4)));
    }
    // ---- S = Q K^T (16 x 64 per warp)
    float s[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.f;
    const __half* K = sK[buf];
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t kf[4];
        const int key = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        ldsm_x4(kf, K + swz(key, kk * 2 + ((lane >> 3) & 1)));
        mma16816(s[2 * np], qf[kk], kf[0], kf[1]);
        mma16816(s[2 * np + 1], qf[kk], kf[2], kf[3]);
      }
    }
    // ---- mask keys past the end
    const int kbase = kt * kKV;
    if (kbase + kKV > seqlen) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = kbase + j * 8 + 2 * t;
        if (c >= seqlen) { s[j][0] = -INFINITY; s[j][2] = -INFINITY; }
        if (c + 1 >= seqlen) { s[j][1] = -INFINITY; s[j][3] = -INFINITY; }
      }
    }
    // ---- online softmax (rows g and g+8 of the warp's 16)
    float mx0 = m0, mx1 = m1;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx0 = fmaxf(mx0, fmaxf(s[j][0], s[j][1]));
      mx1 = fmaxf(mx1, fmaxf(s[j][2], s[j][3]));
    }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float a0 = (m0 == -INFINITY) ? 0.f : exp2f((m0 - mx0) * sl2);
    const float a1 = (m1 == -INFINITY) ? 0.f : exp2f((m1 - mx1) * sl2);
    m0 = mx0;
    m1 = mx1;
    const float b0 = mx0 * sl2, b1 = mx1 * sl2;
    float r0 = 0.f, r1 = 0.f;
    uint32_t pf[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p0 = exp2f(s[j][0] * sl2 - b0), p1 = exp2f(s[j][1] * sl2 - b0);
      const float p2 = exp2f(s[j][2] * sl2 - b1), p3 = exp2f(s[j][3] * sl2 - b1);
      r0 += p0 + p1;
      r1 += p2 + p3;
      // C-fragment pair (2 n-tiles) == A-fragment of the next MMA (k = 16 keys)
      pf[j >> 1][(j & 1) * 2 + 0] = pack_h2(p0, p1);
      pf[j >> 1][(j & 1) * 2 + 1] = pack_h2(p2, p3);
    }
    l0 = l0 * a0 + r0;
    l1 = l1 * a1 + r1;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      o[i][0] *= a0; o[i][1] *= a0;
      o[i][2] *= a1; o[i][3] *= a1;
    }
    // ---- O += P V
    const __half* V = sV[buf];
#pragma unroll
    for (int kc = 0; kc < 4; ++kc) {
      // A fragment order {a0,a1,a2,a3} = {(g, k0..), (g+8, k0..), (g, k8..), (g+8, k8..)}
      const uint32_t pa[4] = {pf[kc][0], pf[kc][1], pf[kc][2], pf[kc][3]};
#pragma unroll
      for (int dp = 0; dp < 4; ++dp) {
        uint32_t vf[4];
        const int key = kc * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        ldsm_x4_t(vf, V + swz(key, dp * 2 + (lane >> 4)));
        mma16816(o[2 * dp], pa, vf[0], vf[1]);
        mma16816(o[2 * dp + 1], pa, vf[2], vf[3]);
      }
    }
    __syncthreads();
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    o[j][0] *= i0; o[j][1] *= i0;
    o[j][2] *= i1; o[j][3] *= i1;
  }
  if (q8) {
    // Q8_0 round trip per (row, 32-dim block): block b = dim tiles 4b..4b+3, spread
    // over the 4 threads of a quad (ggml quantize_row_q8_0_ref semantics).
#pragma unroll
    for (int b = 0; b < 2; ++b) {
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        float amax = 0.f;
#pragma unroll
        for (int j = 4 * b; j < 4 * b + 4; ++j) amax = fmaxf(amax, fmaxf(fabsf(o[j][2 * half]), fabsf(o[j][2 * half + 1])));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
        const float d = amax / 127.0f;
        const float id = d != 0.f ? 1.0f / d : 0.0f;
        const float dh = __half2float(__float2half_rn(d));
#pragma unroll
        for (int j = 4 * b; j < 4 * b + 4; ++j) {
          o[j][2 * half] = dh * roundf(o[j][2 * half] * id);
          o[j][2 * half + 1] = dh * roundf(o[j][2 * half + 1] * id);
        }
      }
    }
  }
  const int row0 = q0 + warp * 16 + g, row1 = row0 + 8;
  __half* ob = out + static_cast<size_t>(sq) * seqlen * D + h * kHD;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int col = j * 8 + 2 * t;
    if (row0 < seqlen)
      *reinterpret_cast<__half2*>(ob + static_cast<size_t>(row0) * D + col) = __floats2half2_rn(o[j][0], o[j][1]);
    if (row1 < seqlen)
      *reinterpret_cast<__half2*>(ob + static_cast<size_t>(row1) * D + col) = __floats2half2_rn(o[j][2], o[j][3]);
  }
}

}  // namespace

int flash_attn(const __half* qkv, int nseq, int seqlen, int H, int D, __half* out, cudaStream_t s, int q8) {
  if (nseq <= 0 || seqlen <= 0) return 0;
  if (D != H * kHD || (reinterpret_cast<uintptr_t>(qkv) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return -1;
  dim3 grid((seqlen + kQ - 1) / kQ, H, nseq);
  const float sl2 = (1.0f / sqrtf(static_cast<float>(kHD))) * 1.4426950408889634f;
  k_flash_attn<<<grid, 256, 0, s>>>(qkv, seqlen, H, D, out, sl2, q8);
  return cudaGetLastError() == cudaSuccess ? 0 : -2;
}

}  // namespace da3b
