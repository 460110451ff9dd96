// Launchers of the memory-bound kernels (kernels.cu) and attention (attention.cu).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace da3b {

int patchify(const uint8_t* rgb, int B, int H, int W, int P, const float* mean, const float* sd, __half* out, int ldk,
             cudaStream_t s);
// Patchify of normalised planar f32 images [B][3][H][W] (no normalisation): the
// prepared-input path.
// Legacy preprocess (floor-to-patch float bilinear + normalisation) into planar f32
// [B][3][*out_h][*out_w]; out == nullptr: size query only.
int legacy_preprocess(const uint8_t* src, int B, int w, int h, int patch, const float* mean, const float* sd,
                      float* out, int* out_w, int* out_h, cudaStream_t s);
int patchify_chw(const float* chw, int B, int H, int W, int P, __half* out, int ldk, cudaStream_t s);
int cls_rows(float* x, int B, int ntok, int D, const float* cls, const float* pos, cudaStream_t s);
int cam_rows(float* x, int nviews_total, int views_per_scene, int ntok, int D, const float* cam, cudaStream_t s);
// LayerNorm rows (D in {128,256,384,512,768,1024,1536,2048}); input row of output row r
// is (r / rm_div) * rm_mul + rm_add + r % rm_div when rm_div > 0.
// q8 = 1: Q8_0 round trip of each 32-element block of the output (ggml activation
// quantisation ahead of a Q8_0 matmul).
// dq (or null): a ViT block's planar Q8_0 staging dequantisation (ops.h), run by the
// same launch as the LayerNorm where the wide kernel serves it, else just before it.
struct Q8Segs;
int layernorm_f32(const float* in, int ld_in, int rows, int D, const float* g, const float* b, float eps, __half* out,
                  int ld_out, int col_off, int rm_div, int rm_mul, int rm_add, cudaStream_t s, int q8 = 0,
                  const Q8Segs* dq = nullptr);
int layernorm_f16(const __half* in, int ld_in, int rows, int D, const float* g, const float* b, float eps,
                  __half* out, int ld_out, int col_off, int rm_div, int rm_mul, int rm_add, cudaStream_t s);
int cast_rows(const float* in, int ld_in, int rows, int D, __half* out, int ld_out, int col_off, int rm_div, int rm_mul,
              int rm_add, cudaStream_t s);
int qk_norm_rope(__half* qkv, int M, int H, int D, int ntok, const float* qg, const float* qb, const float* kg,
                 const float* kb, const float* cs, const float* sn, cudaStream_t s);
int upsample_ac(const __half* in, int B, int hs, int ws, int C, __half* out, int H, int W, const __half* pe,
                cudaStream_t s);
int im2col_s2(const __half* in, int B, int h, int w, int C, int icp, __half* out, cudaStream_t s);
int select_ref_view(const float* x, int scenes, int S, int ntok, int D, int* b_idx, cudaStream_t s);
int permute_views(const float* src, float* dst, int scenes, int S, long view_elems, const int* b_idx, cudaStream_t s);
int unpermute_views_h(const __half* src, __half* dst, int scenes, int S, long view_elems, const int* b_idx,
                      cudaStream_t s);

// v third of qkv -> vt [nseq][H][64][ld] (the B operand layout of the tcgen05 attention).
int transpose_v(const __half* qkv, int nseq, int seqlen, int H, int D, __half* vt, int ld, cudaStream_t s);
// tcgen05 flash attention: q, k from qkv, v from vt (attention_tc.cu).
int attention_tc(const __half* qkv, const __half* vt, int ld_vt, int nseq, int seqlen, int H, int D, __half* out,
                 int q8, int* status, cudaStream_t s);
// Key-range split of attention_tc: -1 automatic (default), 1 never, 2-4 forced shares.
void set_attention_split(int n);



// Camera token capture and the camera decoder's small-M GEMV (kernels.cu).
int copy_token0(const float* x, int V, int Nt, int D, float* dst, int ld_dst, int col_off, cudaStream_t s);
int gemv_rows(const float* x, int M, int K, const __half* W, int ldw, const float* b, int N, int act, float* y,
              int ldy, int y_off, cudaStream_t s);

}  // namespace da3b
