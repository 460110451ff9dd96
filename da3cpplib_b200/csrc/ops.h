// Host-side launchers of the device kernels (internal to libda3b).
#pragma once
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "gemm.h"

namespace da3b {

// ------------------------------------------------------------------ GEMM engine (gemm.cu)
int make_tmap_2d(CUtensorMap* map, const void* ptr, int rows, int cols, int ld, int box_rows);
int make_tmap_nhwc(CUtensorMap* map, const void* ptr, int B, int H, int W, int C, int bw, int bh);
int make_tmap_2d_typed(CUtensorMap* map, const void* ptr, CUtensorMapDataType dtype, int elem_bytes, int rows,
                       int cols, int ld, int box_cols, int box_rows, CUtensorMapSwizzle swz);
int make_tmap_nhwc_planes(CUtensorMap* map, const void* ptr, int B, int H, int W, int C, int bw, int bh);
int gemm_launch(int bn, const CUtensorMap& ta, const CUtensorMap& tb, const GemmGeom& g, const EpiArgs& e,
                int* status, cudaStream_t stream, int max_ctas);

// C[M][N] = A[M][K] * W[N][K]^T with a fused epilogue. bn <= 0 picks the N tile.
int gemm_linear(const __half* A, int M, int K, int lda, const __half* W, int N, int ldw, int bn, const EpiArgs& e,
                int* status, cudaStream_t stream);
// The same with W planar Q8_0 [N][K] (q8planar.cuh; K % 32 == 0, N % 8 == 0): the GEMM
// dequantises its weight tiles in shared memory, f16(d * q) as the staging dequantisation
// gives. Serves the one-CTA tile regime without K split only (gemm_q8p_bn(M, N, K) != 0,
// the tile width it takes, the same as the f16 route's); returns 1 without launching
// otherwise.
int gemm_q8p_bn(int M, int N, int K);
// The automatic tiles of an M x N x K linear: 1 = the one-CTA kernel with tile width bn
// and K split ksplit, 0 = CTA pairs with tile width bn, < 0 = bad arguments. Host only.
int gemm_linear_tiles(int M, int N, int K, int* bn, int* ksplit);
int gemm_linear_q8p(const __half* A, int M, int K, int lda, const uint8_t* Wq, int N, const EpiArgs& e, int* status,
                    cudaStream_t stream);
// Implicit-GEMM KxK stride-1 "same" convolution: X NHWC [B][H][W][IC] f16,
// Wp packed [OC][ksize*ksize][icp] f16 (icp = IC rounded up to 64, zero padded).
// The epilogue sees output pixel indices (b*H + y)*W + x as rows.
int conv_nhwc(const __half* X, int B, int H, int W, int IC, const __half* Wp, int OC, int ksize, int bn,
              const EpiArgs& e, int* status, cudaStream_t stream);
int pick_bn(int N);
// Fused align-corners upsample (+ UV pos-embed) -> 3x3 conv to 32 channels -> the
// kEpiOut2 epilogue (head_fused.cu): src NHWC [B][hs][ws][C] f16, output grid H x W,
// packed 3x3 weights [32][9][icp] (conv_nhwc layout), e.o2_* as for conv_nhwc.
// 3x3 conv with 128 output channels and IC % 64 == 0 (one input box per channel chunk,
// the nine taps as shifted descriptors); returns 1 without launching for other shapes
// or epilogues.
int conv3_halo(const __half* X, int B, int H, int W, int IC, const __half* Wp, int OC, const EpiArgs& e, int* status,
               cudaStream_t s);
int up_out2(const __half* src, int B, int hs, int ws, int C, const __half* pe, int H, int W, const __half* wp,
            int icp, const EpiArgs& e, int* status, cudaStream_t s);
inline int conv_icp(int IC) { return (IC + 63) / 64 * 64; }

EpiArgs epi_default();

// ------------------------------------------------------------------ elementwise (elementwise.cu)
int dequant_q8_0(const void* q8, int rows, int K, __half* out, int ldo, cudaStream_t s);
// Up to four Q8_0 matrices [rows][K/32][34 B] -> dense f16 [rows][K] in one launch;
// `first` is each segment's first 32-element block in the launch's block numbering.
// GGUF Q8_0 [N][K] -> planar Q8_0 (q8planar.cuh), the same number of bytes.
int repack_q8_0_planar(const void* raw, int N, int K, void* planar, cudaStream_t s);
// Up to four planar Q8_0 matrices -> dense f16 [rows][nblk * 32], one launch.
struct Q8Seg {
  const uint8_t* q8;  // planar Q8_0
  __half* out;
  int rows, nblk;
  long first;  // blocks of the segments before this one
};
struct Q8Segs {
  Q8Seg s[4];
  int n;
  long total;  // blocks of all segments
};
int dequant_q8p_segs(const Q8Segs& g, cudaStream_t s);
int f32_to_f16(const float* in, __half* out, size_t n, cudaStream_t s);

// Per-device status word (allocated on first use for the current device).
int* device_status_word();
int read_and_reset_status(int* word, int* out_status);

}  // namespace da3b
