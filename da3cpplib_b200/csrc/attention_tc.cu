// tcgen05 flash attention for sm_100a (head_dim 64, bidirectional).
//
// Replaces ggml_flash_attn_ext (F32 precision) of attention() (src/attention.cpp:44-96)
// on the tensor cores. One CTA = 128 query rows of one (sequence, head); two CTAs per
// SM (~103 KB smem, 256 TMEM columns each) so one CTA's softmax overlaps the other's MMAs.
//   warp 0     TMA: Q tile once; per key tile of 64, the K tile [64 keys][64] and the
//              transposed V tile [64 dims][64 keys] (vt, written by the QKV GEMM
//              epilogue) into a 3-stage ring;
//   warp 1     one thread issues S_j = Q K_j^T (M=128, N=64, K=64) into one of two
//              TMEM S buffers, and once the softmax published P_j, O += P_j [V_j^T; 1]
//              (M=128, N=80, K=64) into one TMEM accumulator: column 64 (a row of ones
//              appended to V^T) accumulates the softmax row sums with the same f16 P;
//   warps 2-5  softmax: thread = query row (its TMEM lane); S_j read once into registers,
//              p = 2^(s*c - m*c) as f16 into one of two 128B-swizzled smem tiles. The
//              max m is only raised when a tile's max exceeds it by more than 2^8; then
//              O is rescaled in TMEM (once the previous P V landed). O / rowsum at the
//              end. P V completions alternate between two barriers by tile parity.
//              Keys past the sequence are masked; rows past it are not stored.
// Every wait is bounded (ptx.cuh); on a timeout the kernel records a status and exits.
#include <algorithm>
#include <atomic>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "kernels.h"
#include "ops.h"
#include "ptx.cuh"

namespace da3b {

namespace {

constexpr int kKT = 64;                  // keys per tile
constexpr int kStagesKV = 3;
constexpr int kQBytes = 128 * 64 * 2;    // Q tile [128][64]
constexpr int kKBytes = kKT * 64 * 2;    // K tile [64 keys][64]
constexpr int kVRows = 80;               // V^T rows: 64 dims, a row of ones (row sums), 15 zero rows
constexpr int kVBytes = kVRows * kKT * 2;
constexpr int kPBytes = 128 * kKT * 2;   // P tile [128][64 keys] (double buffered)
constexpr int kSmem = 1024 + kQBytes + kStagesKV * (kKBytes + kVBytes) + 2 * kPBytes + 256;
constexpr uint32_t kTmemCols = 256;      // S[0..1]: cols [0,128), O (80 cols): [128,208)
constexpr float kRescaleLog2 = 8.0f;     // rescale O only when the row max grows by > 2^8
constexpr int kShareBytes = 128 * 64 * 4 + 128 * 8;  // a split share: O [16][128] float4, (max, sum) [128]
static_assert(kShareBytes <= kStagesKV * (kKBytes + kVBytes), "a split share fits the K / V ring");

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }


// max(a, b, c) in one instruction (sm_100 three-input max.f32)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// 2^x of two values on the FMA/ALU pipes instead of the XU (MUFU) pipe, which one
// exponential per score otherwise saturates. Cody-Waite reduction x = j + f with
// j = round(x) (adding 1.5*2^23 leaves j in the low mantissa bits) and f in [-0.5, 0.5];
// 2^f by a degree-3 polynomial whose coefficients were fitted for this range by
// relative-error minimax (Lawson-weighted least squares; max relative error 7.5e-5,
// below the f16 rounding of P); 2^j is added to the exponent field. x is clamped at
// -125 so the exponent stays normal (the result then rounds to 0 in f16).
constexpr float kE2Shift = 12582912.0f;  // 1.5 * 2^23
constexpr float kE2C3 = 0.05517166853f, kE2C2 = 0.24261112511f, kE2C1 = 0.69326096773f, kE2C0 = 0.99992805719f;
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  x = make_float2(fmaxf(x.x, -125.0f), fmaxf(x.y, -125.0f));
  const float2 t = __fadd2_rn(x, make_float2(kE2Shift, kE2Shift));
  const float2 jf = __fadd2_rn(t, make_float2(-kE2Shift, -kE2Shift));
  const float2 f = __fadd2_rn(x, make_float2(-jf.x, -jf.y));
  float2 p = __ffma2_rn(make_float2(kE2C3, kE2C3), f, make_float2(kE2C2, kE2C2));
  p = __ffma2_rn(p, f, make_float2(kE2C1, kE2C1));
  p = __ffma2_rn(p, f, make_float2(kE2C0, kE2C0));
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

__global__ void __launch_bounds__(192, 2)
    k_attn_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
              const __grid_constant__ CUtensorMap tmV, int seqlen, int H, int D, __half* __restrict__ out, float sl2,
              int q8, int nsplit, int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + kQBytes;
  uint8_t* sV = sK + kStagesKV * kKBytes;
  uint8_t* sP = sV + kStagesKV * kVBytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + 2 * kPBytes);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kStagesKV;
  uint64_t* s_full = kv_empty + kStagesKV;  // [2]
  uint64_t* p_full = s_full + 2;            // [2] P_j written and S_j consumed
  uint64_t* o_full = p_full + 2;            // [2] P_j V_j done, j even / odd
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(o_full + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int split = static_cast<int>(blockIdx.x) % nsplit, qt = static_cast<int>(blockIdx.x) / nsplit;
  const int h = blockIdx.y, sq = blockIdx.z;
  const int q0 = qt * 128;
  const int row_base = sq * seqlen;               // first token row of this sequence
  // this CTA's key tiles [kt0, kt0 + nkt): all of them, or its share when the (query
  // tile, head) is split over a cluster of nsplit CTAs (nsplit <= key tiles)
  const int nkt_all = (seqlen + kKT - 1) / kKT;
  const int kt0 = split * nkt_all / nsplit;
  const int nkt = (split + 1) * nkt_all / nsplit - kt0;

  // rows 64..79 of every V^T stage: a row of ones (its product with P is the row sum
  // of P) and zeros; the TMA only ever writes rows 0..63. Swizzling permutes 16-byte
  // chunks within a row, so a constant row needs no swizzle.
  for (int i = threadIdx.x; i < kStagesKV * 16 * 8; i += blockDim.x) {
    const int st = i / 128, r = 64 + (i % 128) / 8, c = i % 8;
    const uint32_t v = (r == 64) ? 0x3C003C00u : 0u;  // f16 1.0 pairs
    *reinterpret_cast<uint4*>(sV + st * kVBytes + r * 128 + c * 16) = make_uint4(v, v, v, v);
  }
  fence_async_smem();
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStagesKV; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&p_full[b], 4);
      mbar_init(&o_full[b], 1);
    }
    fence_mbar_init();
    prefetch_tmap(&tmQ);
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tO = tmem + 128;
  float o[64];                           // softmax warps: this thread's output row,
  float lsum = 0.f, mrow = 0.f;          // its row sum and the max its exponentials used,
  bool have = false;                     // once the last P V product has landed
  const int r = (warp & 3) * 32 + lane;  // query row within the tile == TMEM lane
  // O / l as f16 into out (rows past the sequence are not stored); with q8 the Q8_0
  // round trip per 32-dim block (ggml quantize_row_q8_0_ref semantics). Warp-collective:
  // the warp's 32 rows go out through shared memory (the Q tile, idle once the last
  // product landed; 4 KB a warp, 16-byte chunks XOR-swizzled by row), four whole
  // 128-byte rows per store instruction instead of 32 pieces of 16 bytes.
  auto store_row = [&](float l) {
    const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
    for (int i = 0; i < 64; ++i) o[i] *= inv;
    if (q8) {
#pragma unroll
      for (int bb = 0; bb < 2; ++bb) {
        float amax = 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(o[32 * bb + i]));
        const float d = amax / 127.0f;
        const float id = d != 0.f ? 1.0f / d : 0.0f;
        const float dh = __half2float(__float2half_rn(d));
#pragma unroll
        for (int i = 0; i < 32; ++i) o[32 * bb + i] = dh * roundf(o[32 * bb + i] * id);
      }
    }
    uint8_t* stg = sQ + (warp & 3) * 4096;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      uint4 u;
      __half2* hh = reinterpret_cast<__half2*>(&u);
#pragma unroll
      for (int k = 0; k < 4; ++k) hh[k] = __floats2half2_rn(o[8 * c + 2 * k], o[8 * c + 2 * k + 1]);
      *reinterpret_cast<uint4*>(stg + lane * 128 + ((c ^ (lane & 7)) << 4)) = u;
    }
    __syncwarp();
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int row = 4 * k + (lane >> 3), c = lane & 7;
      const uint4 u = *reinterpret_cast<const uint4*>(stg + row * 128 + ((c ^ (row & 7)) << 4));
      const int qrow = q0 + (warp & 3) * 32 + row;
      if (qrow < seqlen) *reinterpret_cast<uint4*>(out + static_cast<size_t>(row_base + qrow) * D + h * 64 + c * 8) = u;
    }
  };

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------------- TMA
      mbar_arrive_expect_tx(q_full, kQBytes);
      tma_load_2d(sQ, &tmQ, q_full, h * 64, row_base + q0);
      int stage = 0;
      uint32_t phase = 0;
      const int vrow = (sq * H + h) * 64;
      for (int j = 0; j < nkt; ++j) {
        if (!mbar_wait(&kv_empty[stage], phase ^ 1u, status, kStatusTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&kv_full[stage], kKBytes + 64 * kKT * 2);
        tma_load_2d(sK + stage * kKBytes, &tmK, &kv_full[stage], D + h * 64, row_base + (kt0 + j) * kKT);
        tma_load_2d(sV + stage * kVBytes, &tmV, &kv_full[stage], (kt0 + j) * kKT, vrow);
        if (++stage == kStagesKV) { stage = 0; phase ^= 1u; }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------------- MMA
      // S_j -> S[j&1]; S_{j+2} is issued once the softmax consumed S_j. O (+ the row
      // sums in column 64) accumulates over all key tiles: O += P_j [V_j^T; 1; 0].
      constexpr uint32_t idS = umma_idesc_f16(128, kKT);
      constexpr uint32_t idO = umma_idesc_f16(128, kVRows);
      bool ok = mbar_wait(q_full, 0, status, kStatusTimeoutFull);
      const uint64_t qdesc = umma_desc_sw128(smem_u32(sQ));
      auto issue_s = [&](int j) -> bool {
        const int st = j % kStagesKV;
        if (!mbar_wait(&kv_full[st], (j / kStagesKV) & 1, status, kStatusTimeoutFull)) return false;
        tc_fence_after();
        const uint64_t kdesc = umma_desc_sw128(smem_u32(sK + st * kKBytes));
        const uint32_t tS = tmem + (j & 1) * 64;
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_f16(tS, qdesc + 2 * k, kdesc + 2 * k, idS, k > 0 ? 1u : 0u);
        umma_commit(&s_full[j & 1]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && nkt > 1) ok = issue_s(1);
      for (int j = 0; j < nkt && ok; ++j) {
        const int st = j % kStagesKV, b = j & 1;
        // P_j published (and, if the softmax rescaled O, that rescale is complete)
        if (!mbar_wait(&p_full[b], (j >> 1) & 1, status, kStatusTimeoutFull)) break;
        tc_fence_after();
        const uint64_t pdesc = umma_desc_sw128(smem_u32(sP + b * kPBytes));
        const uint64_t vdesc = umma_desc_sw128(smem_u32(sV + st * kVBytes));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tO, pdesc + 2 * kk, vdesc + 2 * kk, idO, (j > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&o_full[b]);
        umma_commit(&kv_empty[st]);
        if (j + 2 < nkt && !issue_s(j + 2)) break;
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------------ softmax
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    float m = -INFINITY;                             // max used for the exponentials so far
    bool ok = true;
    for (int j = 0; j < nkt; ++j) {
      const int b = j & 1;
      if (!mbar_wait_warp(&s_full[b], (j >> 1) & 1, status, kStatusTimeoutAccum)) { ok = false; break; }
      tc_fence_after();
      const uint32_t tS = tmem + b * 64 + lane_off;
      float sv[64];
      {
        uint32_t ra[32], rb[32];
        tmem_ld32(tS, ra);
        tmem_ld32(tS + 32, rb);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          sv[i] = __uint_as_float(ra[i]);
          sv[32 + i] = __uint_as_float(rb[i]);
        }
      }
      const int kvalid = seqlen - (kt0 + j) * kKT;  // keys of this tile inside the sequence (>= 1)
      if (kvalid < kKT) {
#pragma unroll
        for (int i = 0; i < kKT; ++i)
          if (i >= kvalid) sv[i] = -INFINITY;
      }
      // row max: 8 independent chains, each a two-input max of columns c and 56 + c and
      // three three-input maxima over columns 8..55 (32 instructions for 64 scores
      // instead of 63)
      float m8[8];
#pragma unroll
      for (int c = 0; c < 8; ++c) m8[c] = fmaxf(sv[c], sv[56 + c]);
#pragma unroll
      for (int i = 8; i < 56; i += 16) {
#pragma unroll
        for (int c = 0; c < 8; ++c) m8[c] = fmax3(m8[c], sv[i + c], sv[i + 8 + c]);
      }
      const float mt = fmaxf(fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), m8[6]), m8[7]);
      // The running max of a row is raised only when a tile's max exceeds it by more
      // than 2^8; the accumulated O (and its row-sum column) is then rescaled in TMEM
      // once P V_{j-1} has landed. The TMEM read-modify-write is warp-collective, so the
      // whole warp takes the branch if any of its rows needs it (alpha = 1 elsewhere).
      const bool need = (j > 0) && ((mt - m) * sl2 > kRescaleLog2);
      if (j == 0) m = mt;
      if (__any_sync(0xffffffffu, need)) {
        if (!mbar_wait_warp(&o_full[(j - 1) & 1], ((j - 1) >> 1) & 1, status, kStatusTimeoutAccum)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float alpha = need ? ex2_approx((m - mt) * sl2) : 1.0f;
        uint32_t ra[32], rb[32], rc;
        tmem_ld32(tO + lane_off, ra);
        tmem_ld32(tO + lane_off + 32, rb);
        tmem_ld1(tO + lane_off + 64, rc);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          ra[i] = __float_as_uint(__uint_as_float(ra[i]) * alpha);
          rb[i] = __float_as_uint(__uint_as_float(rb[i]) * alpha);
        }
        rc = __float_as_uint(__uint_as_float(rc) * alpha);
        tmem_st32(tO + lane_off, ra);
        tmem_st32(tO + lane_off + 32, rb);
        tmem_st1(tO + lane_off + 64, rc);
        tmem_wait_st();
        if (need) m = mt;
      }
      // p = 2^(s*c - m*c) (masked keys: 2^-inf = 0), f16 into the 128B-swizzled row r
      // of P[b], the A operand of O += P V
      const float mc = m * sl2;
      uint8_t* prow = sP + b * kPBytes + r * 128;
#pragma unroll
      for (int ch = 0; ch < 8; ++ch) {
        uint32_t pk[4];
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 a = __ffma2_rn(make_float2(sv[ch * 8 + 2 * k], sv[ch * 8 + 2 * k + 1]),
                                      make_float2(sl2, sl2), make_float2(-mc, -mc));
          float p0, p1;
          if (k == 0) {  // a quarter of the exponentials on the FMA pipe, the rest on MUFU
            const float2 e2 = exp2_poly2(a);
            p0 = e2.x;
            p1 = e2.y;
          } else {
            p0 = ex2_approx(a.x);
            p1 = ex2_approx(a.y);
          }
          __half2 hp = __floats2half2_rn(p0, p1);
          pk[k] = *reinterpret_cast<uint32_t*>(&hp);
        }
        *reinterpret_cast<uint4*>(prow + ((ch ^ (r & 7)) << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      // No wait on the P V products here: P_{j-2} V_{j-2} (the last reader of P[b])
      // completed before S_j could land, and the two o_full barriers stay within one
      // phase of every later wait (P_j V_j cannot be issued before P_j is published).
      tc_fence_before();
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[b]);
    }
    // final O and row sum after the last P V product
    ok = __all_sync(0xffffffffu, ok);
    if (ok) ok = mbar_wait_warp(&o_full[(nkt - 1) & 1], ((nkt - 1) >> 1) & 1, status, kStatusTimeoutAccum);
    if (ok) {
      tc_fence_after();
      uint32_t ra[32], rb[32], rc;
      tmem_ld32(tO + lane_off, ra);
      tmem_ld32(tO + lane_off + 32, rb);
      tmem_ld1(tO + lane_off + 64, rc);
      tmem_wait_ld();
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        o[i] = __uint_as_float(ra[i]);
        o[32 + i] = __uint_as_float(rb[i]);
      }
      lsum = __uint_as_float(rc);
      mrow = m;
      have = true;
    }
    if (nsplit == 1) {
      if (have) store_row(lsum);
    } else if (split != 0) {
      // this CTA's share: unnormalised O, its max and row sum, into its own (now idle)
      // K / V ring for the cluster's first CTA to read, column-chunk-major (float4 chunk
      // i of row r at [i][r], then (max, sum) pairs at [r]) so that each remote load of
      // a warp reads 512 contiguous bytes
      float4* dst = reinterpret_cast<float4*>(sK);
#pragma unroll
      for (int i = 0; i < 16; ++i) dst[i * 128 + r] = make_float4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
      reinterpret_cast<float2*>(dst + 16 * 128)[r] = make_float2(mrow, lsum);
    }
  }
  if (nsplit > 1) {
    // The cluster's first CTA merges the shares in rank order (so the result does not
    // depend on which CTA finished first): with M the largest share max,
    //   O = sum_s 2^((m_s - M) c) O_s / sum_s 2^((m_s - M) c) l_s.
    cluster_sync();  // every share is in its CTA's shared memory
    if (warp >= 2 && split == 0 && have) {
      const uint32_t share = smem_u32(sK);
      float pm[3], pl[3];
      float mx = mrow;
      float2 ml[3];
#pragma unroll
      for (int sp = 1; sp < 4; ++sp)
        if (sp < nsplit) ml[sp - 1] = ld_dsmem_f2(mapa_shared(share + 16 * 128 * 16 + r * 8, static_cast<uint32_t>(sp)));
#pragma unroll
      for (int sp = 1; sp < 4; ++sp) {
        if (sp >= nsplit) break;
        pm[sp - 1] = ml[sp - 1].x;
        pl[sp - 1] = ml[sp - 1].y;
        mx = fmaxf(mx, ml[sp - 1].x);
      }
      const float w0 = ex2_approx((mrow - mx) * sl2);
      float l = w0 * lsum;
#pragma unroll
      for (int i = 0; i < 64; ++i) o[i] *= w0;
#pragma unroll
      for (int sp = 1; sp < 4; ++sp) {
        if (sp >= nsplit) break;
        const float w = ex2_approx((pm[sp - 1] - mx) * sl2);
        l += w * pl[sp - 1];
        // all 16 loads of the share in flight before the first use: a remote load takes
        // a few hundred cycles, and the warp would wait out each one in turn
        const uint32_t peer = mapa_shared(share + r * 16, static_cast<uint32_t>(sp));
        float4 v[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = ld_dsmem_f4(peer + static_cast<uint32_t>(i * 128 * 16));
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          o[4 * i] += w * v[i].x;
          o[4 * i + 1] += w * v[i].y;
          o[4 * i + 2] += w * v[i].z;
          o[4 * i + 3] += w * v[i].w;
        }
      }
      store_row(l);
    }
    // no CTA leaves while the first one may still read its share; relaxed, so the
    // first CTA's output stores need not complete before the others may go
    asm volatile("barrier.cluster.arrive.relaxed.aligned;\n\tbarrier.cluster.wait.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ------------------------------------------------------- warp-specialised kernel
// Two 128-query tiles per CTA share every 128-key K / V^T tile, and the two softmax
// warpgroups alternate with the tensor core (one CTA per SM, 12 warps):
//   warp 0     TMA: per key tile of 128 the K tile [128 keys][64] (128B swizzle) and
//              V^T as two [64 dims][64 keys] halves, into a 4-stage ring;
//   warp 1     one thread issues, per key tile j and query tile t, once softmax t
//              published P_t(j): O_t += P_t(j) [V_j^T; 1; 0] (M=128, N=80, K=128; P_t
//              read from TMEM) and at once S_t(j+1) = Q_t K_{j+1}^T (M=128, N=128,
//              K=64; Q_t read from TMEM) into the same columns;
//   warps 4-7  softmax of query tile 0, warps 8-11 of query tile 1: thread = query row
//              (its TMEM lane); the whole 128-score row in registers (one pass), p =
//              2^(s*c - m*c) written back as f16 over S_t's first 64 columns: the A
//              operand of the P V product. Warps 2-3 are idle.
// TMEM (512 columns): S_0 | S_1 (128 each, P_t aliases S_t), O_0 | O_1 (80 each: 64
// dims, the row sums from the ones row of V^T, zeros), Q_0 | Q_1 (32 each: f16 pairs).
// The tcgen05.mma operations of one thread run in issue order, so S_t(j+1) overwrites
// P_t(j) only after P_t(j) V_j read it, and S_t(j+1) completing implies P_t(j) V_j
// completed: O_t is never being written while softmax t holds S_t, so the lazy rescale
// of O_t needs no extra wait.
// Measured on a B200 against k_attn_tc: 0.92 against 0.82 ms at the C3 shape, 1.19
// against 1.18 ms at the C4 global shape. Each softmax warpgroup computes a 128-key tile
// in about 1450 cycles and then waits about 1350 for its P V and next S products, whose
// tensor-pipe latency (issue to completion about 1130 cycles for 736 cycles of MMA
// work) this structure exposes once per tile; so it stays the alternative, not the
// default.
constexpr int kPKT = 128;                            // keys per tile
constexpr int kPStages = 4;
constexpr int kPKBytes = kPKT * 64 * 2;              // K tile [128 keys][64 dims]
constexpr int kPVRows = 80;                          // V^T rows: 64 dims, ones, 15 zeros
constexpr int kPVSub = kPVRows * 64 * 2;             // one 64-key half of the V^T tile
constexpr int kPStageBytes = kPKBytes + 2 * kPVSub;  // 36 KB
constexpr int kPSmem = 1024 + kPStages * kPStageBytes + 256;  // > 114 KB: one CTA per SM
constexpr uint32_t kPTmemCols = 512;
constexpr uint32_t kPColO = 256, kPColQ = 416;


// Register split of the warp-specialised kernel: launched with 384 threads at 168
// registers (64 512), warpgroup 0 (TMA, MMA, two idle warps) gives registers back down
// to 56 and the two softmax warpgroups grow to 224, enough to hold a whole 128-score row
// (one pass over S). setmaxnreg.inc waits until the registers are free, so the split
// must not exceed the launch's total; the host checks the kernel's register count.
constexpr int kWThreads = 384;
constexpr int kWRegsLaunch = 168, kWRegsCtl = 56, kWRegsSoft = 224;
static_assert(128 * kWRegsCtl + 256 * kWRegsSoft <= kWThreads * kWRegsLaunch, "register split exceeds the launch");

// 2^a of 64 arguments as 32 f16 pairs (pair c = arguments 2c, 2c+1, low half first): a
// quarter by exp2_poly2's polynomial (pairs 4i), staged across eight chains, the rest on
// MUFU.
__device__ __forceinline__ void exp2_pack64(const float* a, uint32_t (&pk)[32]) {
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    if ((i & 3) == 0) continue;
    __half2 hp = __floats2half2_rn(ex2_approx(a[2 * i]), ex2_approx(a[2 * i + 1]));
    pk[i] = *reinterpret_cast<uint32_t*>(&hp);
  }
  float2 x[8], t[8], q[8];
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    x[c] = make_float2(fmaxf(a[8 * c], -125.0f), fmaxf(a[8 * c + 1], -125.0f));
    t[c] = __fadd2_rn(x[c], make_float2(kE2Shift, kE2Shift));
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const float2 jf = __fadd2_rn(t[c], make_float2(-kE2Shift, -kE2Shift));
    x[c] = __fadd2_rn(x[c], make_float2(-jf.x, -jf.y));
  }
#pragma unroll
  for (int c = 0; c < 8; ++c) q[c] = __ffma2_rn(make_float2(kE2C3, kE2C3), x[c], make_float2(kE2C2, kE2C2));
#pragma unroll
  for (int c = 0; c < 8; ++c) q[c] = __ffma2_rn(q[c], x[c], make_float2(kE2C1, kE2C1));
#pragma unroll
  for (int c = 0; c < 8; ++c) q[c] = __ffma2_rn(q[c], x[c], make_float2(kE2C0, kE2C0));
#pragma unroll
  for (int c = 0; c < 8; ++c) {
    const float e0 = __uint_as_float(__float_as_uint(q[c].x) + (__float_as_uint(t[c].x) << 23));
    const float e1 = __uint_as_float(__float_as_uint(q[c].y) + (__float_as_uint(t[c].y) << 23));
    __half2 hp = __floats2half2_rn(e0, e1);
    pk[4 * c] = *reinterpret_cast<uint32_t*>(&hp);
  }
}

__global__ void __launch_bounds__(kWThreads, 1)
    k_attn_ws(const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
              const __half* __restrict__ qkv, int seqlen, int H, int D, __half* __restrict__ out, float sl2, int q8,
              int* status) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + kPStages * kPStageBytes);
  uint64_t* kv_full = bars;
  uint64_t* kv_empty = kv_full + kPStages;
  uint64_t* q_ready = kv_empty + kPStages;  // [2] Q_t in TMEM (4 warps)
  uint64_t* s_full = q_ready + 2;           // [2] S_t of the current key tile
  uint64_t* p_ready = s_full + 2;           // [2] P_t written, O_t rescaled (4 warps)
  uint64_t* pv_done = p_ready + 2;          // [2] P_t V_j complete
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pv_done + 2);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, sq = blockIdx.z;
  const int q0 = blockIdx.x * 256;
  const int nact = (seqlen - q0 > 128) ? 2 : 1;   // query tiles of this CTA inside the sequence
  const int row_base = sq * seqlen;
  const int nkt = (seqlen + kPKT - 1) / kPKT;

  // rows 64..79 of every V^T half: a row of ones (its product with P is the row sum of
  // P) and zeros; the TMA only writes rows 0..63. A constant row needs no swizzle.
  for (int i = threadIdx.x; i < kPStages * 2 * 16 * 8; i += blockDim.x) {
    const int st = i / 256, sub = (i / 128) & 1, r = 64 + (i % 128) / 8, c = i % 8;
    const uint32_t v = (r == 64) ? 0x3C003C00u : 0u;
    *reinterpret_cast<uint4*>(smem + st * kPStageBytes + kPKBytes + sub * kPVSub + r * 128 + c * 16) =
        make_uint4(v, v, v, v);
  }
  fence_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kPStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int t = 0; t < 2; ++t) {
      mbar_init(&q_ready[t], 4);
      mbar_init(&s_full[t], 1);
      mbar_init(&p_ready[t], 4);
      mbar_init(&pv_done[t], 1);
    }
    fence_mbar_init();
    prefetch_tmap(&tmK);
    prefetch_tmap(&tmV);
  }
  if (warp == 1) tmem_alloc(tmem_slot, kPTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp < 4) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;\n" ::"n"(kWRegsCtl));
    if (warp == 0 && lane == 0) {
      // ---------------------------------------------------------------- TMA
      const int vrow = (sq * H + h) * 64;
      for (int j = 0; j < nkt; ++j) {
        const int st = j % kPStages;
        if (!mbar_wait(&kv_empty[st], ((j / kPStages) & 1) ^ 1u, status, kStatusTimeoutEmpty)) break;
        uint8_t* sb = smem + st * kPStageBytes;
        mbar_arrive_expect_tx(&kv_full[st], kPKBytes + 2 * 64 * 64 * 2);
        tma_load_2d(sb, &tmK, &kv_full[st], D + h * 64, row_base + j * kPKT);
        tma_load_2d(sb + kPKBytes, &tmV, &kv_full[st], j * kPKT, vrow);
        tma_load_2d(sb + kPKBytes + kPVSub, &tmV, &kv_full[st], j * kPKT + 64, vrow);
      }
    } else if (warp == 1 && lane == 0) {
      // ---------------------------------------------------------------- MMA
      // Per key tile j and query tile t: O_t += P_t(j) [V_j^T; 1; 0] as soon as P_t(j) is
      // published, then at once S_t(j+1) = Q_t K_{j+1}^T into the same TMEM columns.
      // tcgen05.mma operations of one thread run in issue order, so P_t(j) is read before
      // S_t(j+1) overwrites it, and S_t(j+1) completing implies P_t(j) V_j completed.
      constexpr uint32_t idS = umma_idesc_f16(128, kPKT);
      constexpr uint32_t idO = umma_idesc_f16(128, kPVRows);
      bool ok = true;
      for (int t = 0; t < nact && ok; ++t) ok = mbar_wait(&q_ready[t], 0, status, kStatusTimeoutFull);
      if (ok) ok = mbar_wait(&kv_full[0], 0, status, kStatusTimeoutFull);
      if (ok) {
        tc_fence_after();
        const uint64_t kdesc = umma_desc_sw128(smem_u32(smem));
        for (int t = 0; t < nact; ++t) {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16_tmem_a(tmem + 128 * t, tmem + kPColQ + 32 * t + 8 * k, kdesc + 2 * k, idS, k > 0 ? 1u : 0u);
          umma_commit(&s_full[t]);
        }
      }
      for (int j = 0; j < nkt && ok; ++j) {
        const int st = j % kPStages, st1 = (j + 1) % kPStages;
        const uint8_t* sb = smem + st * kPStageBytes;
        const uint64_t kdesc1 = umma_desc_sw128(smem_u32(smem + st1 * kPStageBytes));
        bool next_ready = false;
        for (int t = 0; t < nact; ++t) {
          if (!mbar_wait(&p_ready[t], j & 1, status, kStatusTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t tO = tmem + kPColO + 80 * t, tP = tmem + 128 * t;
#pragma unroll
          for (int kk = 0; kk < 8; ++kk) {
            const uint64_t vdesc = umma_desc_sw128(smem_u32(sb + kPKBytes + (kk >> 2) * kPVSub)) + 2 * (kk & 3);
            umma_f16_tmem_a(tO, tP + 8 * kk, vdesc, idO, (j > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&pv_done[t]);
          if (j + 1 < nkt) {
            if (!next_ready) {
              if (!mbar_wait(&kv_full[st1], ((j + 1) / kPStages) & 1, status, kStatusTimeoutFull)) {
                ok = false;
                break;
              }
              tc_fence_after();
              next_ready = true;
            }
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16_tmem_a(tmem + 128 * t, tmem + kPColQ + 32 * t + 8 * k, kdesc1 + 2 * k, idS, k > 0 ? 1u : 0u);
            umma_commit(&s_full[t]);
          }
        }
        if (!ok) break;
        umma_commit(&kv_empty[st]);
      }
    }
    __syncwarp();
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;\n" ::"n"(kWRegsSoft));
    // ------------------------------------------------------------------ softmax
    const int t = (warp >> 2) - 1;
    const int qq = warp & 3;
    const int r = qq * 32 + lane;                  // query row within tile t == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>(qq * 32) << 16;
    const int qrow = q0 + 128 * t + r;             // query row within the sequence
    if (t < nact) {
      const uint32_t tS = tmem + 128 * t + lane_off;
      const uint32_t tO = tmem + kPColO + 80 * t + lane_off;
      const uint32_t tQ = tmem + kPColQ + 32 * t + lane_off;
      {
        // Q row -> TMEM lane r as 32 columns of f16 pairs (low half = even dimension)
        uint32_t qv[32];
        if (qrow < seqlen) {
          const uint4* src = reinterpret_cast<const uint4*>(qkv + static_cast<size_t>(row_base + qrow) * 3 * D + h * 64);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint4 u = src[i];
            qv[4 * i] = u.x;
            qv[4 * i + 1] = u.y;
            qv[4 * i + 2] = u.z;
            qv[4 * i + 3] = u.w;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) qv[i] = 0u;
        }
        tmem_st32(tQ, qv);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&q_ready[t]);
      }
      float m = -INFINITY;
      bool ok = true;
      for (int j = 0; j < nkt; ++j) {
        if (!mbar_wait_warp(&s_full[t], j & 1, status, kStatusTimeoutAccum)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // the whole 128-score row in registers
        float sv[128];
        {
          uint32_t ra[32], rb[32], rc[32], rd[32];
          tmem_ld32(tS, ra);
          tmem_ld32(tS + 32, rb);
          tmem_ld32(tS + 64, rc);
          tmem_ld32(tS + 96, rd);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            sv[i] = __uint_as_float(ra[i]);
            sv[32 + i] = __uint_as_float(rb[i]);
            sv[64 + i] = __uint_as_float(rc[i]);
            sv[96 + i] = __uint_as_float(rd[i]);
          }
        }
        const int kvalid = seqlen - j * kPKT;       // keys of this tile inside the sequence (>= 1)
        if (kvalid < kPKT) {  // the last tile of the sequence only (uniform branch)
#pragma unroll
          for (int i = 0; i < kPKT; ++i)
            if (i >= kvalid) sv[i] = -INFINITY;
        }
        // row max: 8 chains over columns 0..119 by three-input maxima, then 120..127
        float m8[8];
#pragma unroll
        for (int c = 0; c < 8; ++c) m8[c] = fmax3(sv[c], sv[8 + c], sv[16 + c]);
#pragma unroll
        for (int i = 24; i < 120; i += 16) {
#pragma unroll
          for (int c = 0; c < 8; ++c) m8[c] = fmax3(m8[c], sv[i + c], sv[i + 8 + c]);
        }
#pragma unroll
        for (int c = 0; c < 8; ++c) m8[c] = fmaxf(m8[c], sv[120 + c]);
        const float mt = fmaxf(fmax3(fmax3(m8[0], m8[1], m8[2]), fmax3(m8[3], m8[4], m8[5]), m8[6]), m8[7]);
        // lazy rescale (the running max is raised only when a tile's max exceeds it by
        // more than 2^8); O_t is stable here: P_t V_{j-1} was issued before S_t(j), whose
        // completion this thread waited for
        const bool need = (j > 0) && ((mt - m) * sl2 > kRescaleLog2);
        if (j == 0) m = mt;
        if (__any_sync(0xffffffffu, need)) {
          const float alpha = need ? ex2_approx((m - mt) * sl2) : 1.0f;
          uint32_t ra[32], rb[32], rc;
          tmem_ld32(tO, ra);
          tmem_ld32(tO + 32, rb);
          tmem_ld1(tO + 64, rc);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            ra[i] = __float_as_uint(__uint_as_float(ra[i]) * alpha);
            rb[i] = __float_as_uint(__uint_as_float(rb[i]) * alpha);
          }
          rc = __float_as_uint(__uint_as_float(rc) * alpha);
          tmem_st32(tO, ra);
          tmem_st32(tO + 32, rb);
          tmem_st1(tO + 64, rc);
          if (need) m = mt;
        }
        // p = 2^(s*c - m*c) as f16 pairs over the first 64 columns of S_t (the TMEM A
        // operand of O_t += P_t V): keys 0..63 -> columns 0..31, 64..127 -> 32..63
        const float mc = m * sl2;
#pragma unroll
        for (int i = 0; i < kPKT; i += 2) {
          const float2 a = __ffma2_rn(make_float2(sv[i], sv[i + 1]), make_float2(sl2, sl2), make_float2(-mc, -mc));
          sv[i] = a.x;
          sv[i + 1] = a.y;
        }
#pragma unroll
        for (int half = 0; half < 2; ++half) {
          uint32_t pk[32];
          exp2_pack64(sv + 64 * half, pk);
          tmem_st32(tS + 32 * half, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_ready[t]);
      }
      ok = __all_sync(0xffffffffu, ok);
      if (ok) ok = mbar_wait_warp(&pv_done[t], (nkt - 1) & 1, status, kStatusTimeoutAccum);
      if (ok) {
        tc_fence_after();
        float o[64];
        uint32_t ra[32], rb[32], rc;
        tmem_ld32(tO, ra);
        tmem_ld32(tO + 32, rb);
        tmem_ld1(tO + 64, rc);
        tmem_wait_ld();
        const float l = __uint_as_float(rc);
        const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          o[i] = __uint_as_float(ra[i]) * inv;
          o[32 + i] = __uint_as_float(rb[i]) * inv;
        }
        if (qrow < seqlen) {
          if (q8) {
            // Q8_0 round trip per 32-dim block (ggml quantize_row_q8_0_ref semantics)
#pragma unroll
            for (int bb = 0; bb < 2; ++bb) {
              float amax = 0.f;
#pragma unroll
              for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(o[32 * bb + i]));
              const float d = amax / 127.0f;
              const float id = d != 0.f ? 1.0f / d : 0.0f;
              const float dh = __half2float(__float2half_rn(d));
#pragma unroll
              for (int i = 0; i < 32; ++i) o[32 * bb + i] = dh * roundf(o[32 * bb + i] * id);
            }
          }
          __half* dst = out + static_cast<size_t>(row_base + qrow) * D + h * 64;
#pragma unroll
          for (int i = 0; i < 64; i += 8) {
            uint4 u;
            __half2* hh = reinterpret_cast<__half2*>(&u);
#pragma unroll
            for (int k = 0; k < 4; ++k) hh[k] = __floats2half2_rn(o[i + 2 * k], o[i + 2 * k + 1]);
            *reinterpret_cast<uint4*>(dst + i) = u;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kPTmemCols);
  }
}

}  // namespace

// qkv: [nseq*seqlen][3D] (q | k | v), vt: [nseq][H][64][ld_vt] (transposed v), out:
// [nseq*seqlen][D]. The columns of vt beyond seqlen are padding that is never read:
// the V^T tensor map is seqlen wide, so the TMA fills out-of-range keys with zeros.
// attention_tc runs the 128-query kernel (2 CTAs per SM, P in shared memory);
// $DA3B_ATTN_PP=1 (read once per process) selects the warp-specialised kernel, which is
// correct but measured slower at the C3 shape (0.92 against 0.82 ms).
// Key-range split of the 128-query kernel: -1 = automatic; 1 = never; 2-4 = that many
// shares wherever the sequence has that many key tiles (tests). Initial value from
// $DA3B_ATTN_SPLIT (0 = never), read once per process.
static std::atomic<int> g_attn_split{[] {
  const char* e = getenv("DA3B_ATTN_SPLIT");
  if (!e || !e[0]) return -1;
  const int v = atoi(e);
  return v <= 1 ? 1 : (v > 4 ? 4 : v);
}()};

void set_attention_split(int n) { g_attn_split.store(n < 0 ? -1 : (n <= 1 ? 1 : (n > 4 ? 4 : n))); }

static bool attn_pp() {
  static const bool pp = [] {
    const char* e = getenv("DA3B_ATTN_PP");
    return e && e[0] == '1';
  }();
  return pp;
}

static int attention_pp(const __half* qkv, const __half* vt, int ld_vt, int nseq, int seqlen, int H, int D,
                        __half* out, int q8, int* status, cudaStream_t s) {
  CUtensorMap tk, tv;
  int rc;
  if ((rc = make_tmap_2d(&tk, qkv, nseq * seqlen, 3 * D, 3 * D, kPKT))) return rc - 100;
  if ((rc = make_tmap_2d(&tv, vt, nseq * H * 64, seqlen, ld_vt, 64))) return rc - 200;
  static std::atomic<uint64_t> attr_set{0};  // one bit per device; first calls may race
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(attr_set.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(k_attn_ws, cudaFuncAttributeMaxDynamicSharedMemorySize, kPSmem) != cudaSuccess)
      return -3;
    attr_set.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int ntiles = (seqlen + 127) / 128;
  dim3 grid((ntiles + 1) / 2, H, nseq);
  const float sl2 = 0.125f * 1.4426950408889634f;
  // the register split (setmaxnreg) needs the kernel to launch with its full share
  static std::atomic<int> regs_fit{0};  // 0 = unchecked, 1 = fits, -1 = does not
  if (regs_fit.load(std::memory_order_acquire) == 0) {
    cudaFuncAttributes fa;
    memset(&fa, 0, sizeof(fa));
    if (cudaFuncGetAttributes(&fa, k_attn_ws) != cudaSuccess) return -5;
    const bool fits = fa.numRegs * kWThreads >= 128 * kWRegsCtl + 256 * kWRegsSoft;
    if (!fits) fprintf(stderr, "[da3b] attention: kernel has %d registers, the split needs %d\n", fa.numRegs, kWRegsLaunch);
    regs_fit.store(fits ? 1 : -1, std::memory_order_release);
  }
  if (regs_fit.load(std::memory_order_acquire) < 0) return -5;
  k_attn_ws<<<grid, kWThreads, kPSmem, s>>>(tk, tv, qkv, seqlen, H, D, out, sl2, q8, status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    cudaFuncAttributes fa;
    memset(&fa, 0, sizeof(fa));
    cudaFuncGetAttributes(&fa, k_attn_ws);
    fprintf(stderr, "[da3b] attention launch failed: %s (regs %d, max threads %d, smem %d)\n", cudaGetErrorString(e),
            fa.numRegs, fa.maxThreadsPerBlock, kPSmem);
    return -4;
  }
  return 0;
}

int attention_tc(const __half* qkv, const __half* vt, int ld_vt, int nseq, int seqlen, int H, int D, __half* out,
                 int q8, int* status, cudaStream_t s) {
  if (nseq <= 0 || seqlen <= 0) return 0;
  if (D != H * 64 || ld_vt < seqlen || ld_vt % 8 || (reinterpret_cast<uintptr_t>(out) & 15)) return -1;
  if (attn_pp()) return attention_pp(qkv, vt, ld_vt, nseq, seqlen, H, D, out, q8, status, s);
  CUtensorMap tq, tk, tv;
  int rc;
  if ((rc = make_tmap_2d(&tq, qkv, nseq * seqlen, 3 * D, 3 * D, 128))) return rc - 100;
  if ((rc = make_tmap_2d(&tk, qkv, nseq * seqlen, 3 * D, 3 * D, kKT))) return rc - 100;
  if ((rc = make_tmap_2d(&tv, vt, nseq * H * 64, seqlen, ld_vt, 64))) return rc - 200;
  // per-device "attribute set" bits; host threads may make their first call at once
  static std::atomic<uint64_t> attr_set{0};
  int dev = 0;
  cudaGetDevice(&dev);
  const uint64_t bit = uint64_t(1) << (dev & 63);
  if (!(attr_set.load(std::memory_order_acquire) & bit)) {
    if (cudaFuncSetAttribute(k_attn_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmem) != cudaSuccess) return -3;
    attr_set.fetch_or(bit, std::memory_order_acq_rel);
  }
  const int ntq = (seqlen + 127) / 128, nkt = (seqlen + kKT - 1) / kKT;
  const float sl2 = 0.125f * 1.4426950408889634f;
  // When the (query tile, head, sequence) CTAs fill fewer than the SMs' two slots each
  // (one image: 11 x 12 heads on 148 SMs), each one's key tiles are split over a
  // cluster of up to four CTAs, which merge their shares through distributed shared
  // memory: at batch 1 the softmax of one CTA per SM runs with one warp per SM
  // sub-partition and nothing to hide its latencies behind. A share keeps at least six
  // key tiles; below that the merge (about 2 us) costs more than the split saves.
  int sms = 148;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long ctas = static_cast<long long>(ntq) * H * nseq;
  const int mode = g_attn_split.load(std::memory_order_relaxed);
  int nsplit = 1;
  if (mode < 0) nsplit = static_cast<int>(std::min<long long>({4LL, (2LL * sms) / ctas, nkt / 6}));
  else if (mode > 1) nsplit = mode;
  nsplit = std::max(1, std::min(nsplit, nkt));
  if (nsplit == 1) {
    k_attn_tc<<<dim3(ntq, H, nseq), 192, kSmem, s>>>(tq, tk, tv, seqlen, H, D, out, sl2, q8, 1, status);
    return cudaGetLastError() == cudaSuccess ? 0 : -4;
  }
  cudaLaunchConfig_t cfg;
  memset(&cfg, 0, sizeof(cfg));
  cfg.gridDim = dim3(ntq * nsplit, H, nseq);
  cfg.blockDim = dim3(192, 1, 1);
  cfg.dynamicSmemBytes = kSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(nsplit);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, k_attn_tc, tq, tk, tv, seqlen, H, D, out, sl2, q8, nsplit, status) != cudaSuccess)
    return -4;
  return cudaGetLastError() == cudaSuccess ? 0 : -4;
}

}  // namespace da3b
