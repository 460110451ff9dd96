// Host/device argument blocks of the persistent tcgen05 GEMM engine (gemm.cu).
//
// One kernel serves every dense contraction of the depth path:
//   * linear mode: C[M][N] = A[M][K] * B[N][K]^T  (ViT linears, 1x1 convs,
//     reassemble transposed convs, the stride-2 conv after explicit im2col);
//   * conv mode:   implicit-GEMM KxK stride-1 "same" convolution on NHWC f16,
//     where each k-block is one (tap, 64-channel chunk) of the input fetched by a
//     4-D TMA box whose out-of-range rows/columns are zero-filled (= padding).
// A and B are f16, K-major; the accumulator is f32 in TMEM; the epilogue is fused.
#pragma once
#include <stdint.h>

namespace da3b {

enum GemmMode : int { kModeLinear = 0, kModeConv = 1 };

enum EpiKind : int {
  kEpiF16 = 0,     // out = act(acc + bias + res1 + res2) as f16; optional out_relu = relu(...)
  kEpiResid = 1,   // resid_f32 += scale * (acc + bias)            (ViT proj / fc2)
  kEpiTokens = 2,  // resid_f32[row map] = acc + bias + pos[...]   (patch embed)
  kEpiConvT = 3,   // stride==kernel transposed conv: pixel-shuffle f16 store
  kEpiOut2 = 4,    // out2a(32ch) -> [LN] -> relu -> out2b (<=8ch) -> activation -> f32 planes
  kEpiQKV = 5,     // QKV linear: q|k columns to out (f16 [rows][ld_out]) and the v third
                   // transposed per (sequence, head) to vt [seq][H][64][ld_vt] for attention
};

// kActGelu and kActGeluR are both the exact-form (erf) GELU, with different erf
// approximations of published error bound (see gemm.cu): kActGeluR spends one MUFU
// operation per value instead of two.
enum Act : int { kActNone = 0, kActRelu = 1, kActGelu = 2, kActGeluR = 3 };

// Output activation of the fused out2b stage (per output channel).
enum OutAct : int {
  kOutIdentity = 0,  // raw logit
  kOutRelu = 1,      // DA2 relative: relu(l)
  kOutSigmoidScale = 2,  // DA2 metric: sigmoid(l) * out_scale
  kOutExp = 3,       // DA3 depth: exp(l)
  kOutExpP1 = 4,     // DA3 confidence / ray confidence: exp(l) + 1
};

struct GemmGeom {
  int mode;         // GemmMode
  int M, N;         // linear rows (or total output pixels in conv mode), output columns
  int K;            // linear: reduction length; conv: input channels (per tap)
  int num_kb;       // 64-wide k-blocks per tile
  int num_m_tiles, num_n_tiles;
  // conv mode
  int B, H, W;      // output (= input) spatial size and batch
  int bw, bh;       // pixel block of one M tile (bw * bh == 128)
  int tiles_x, tiles_y;
  int ksize, pad;   // kernel size, padding (stride 1)
  int ic_chunks;    // ceil(IC / 64)
  int icp;          // padded per-tap channel stride of the packed weight (ic_chunks * 64)
  int ksplit;       // 1-SM kernel: > 1 = a cluster of ksplit CTAs per tile, each a share of the k-blocks
};

struct EpiArgs {
  int kind;          // EpiKind
  int act;           // Act (kEpiF16)
  int tma_store;     // set by the launcher: 1 = f16 tile via TMA store, 2 = f32 TMA reduce-add
                     // into resid (2-SM kernel, row-major outputs without row remap)
  int q8;            // kEpiF16: round-trip each 32-column block through Q8_0 (ggml's
                     // activation quantisation before a Q8_0 matmul); needs N % 32 == 0
  const float* bias;   // [N] or null
  const float* scale;  // [N] LayerScale (kEpiResid) or null
  float* resid;        // f32 [rows][ld_resid] (kEpiResid / kEpiTokens)
  int ld_resid;
  __half* out;         // f16 output
  int ld_out;
  __half* out_relu;    // optional second f16 output relu(v), same indexing as out
  const __half* res1;  // optional f16 addend, row index = out_row % res1_mod (if res1_mod > 0)
  int ld_res1, res1_mod;
  const __half* res2;  // optional f16 addend, same indexing as out
  int ld_res2;
  // output row remap: row' = (row / rm_div) * rm_mul + rm_add + row % rm_div (rm_div > 0)
  int rm_div, rm_mul, rm_add;
  // kEpiTokens: pos-embed rows [ntok][N] f32; pos row = 1 + row % rm_div
  const float* pos;
  // kEpiConvT: input grid (Hin, Win), stride S, output channels OC
  int ct_hin, ct_win, ct_s, ct_oc;
  // kEpiOut2
  const float* o2_w;      // [o2_dim][32] 1x1 weights
  const float* o2_b;      // [o2_dim]
  const float* o2_ln_g;   // optional LayerNorm(32) gamma/beta applied before relu
  const float* o2_ln_b;
  float o2_ln_eps;
  int o2_dim;             // <= 8
  int o2_act[8];          // OutAct per output channel
  float o2_scale;         // kOutSigmoidScale factor
  float* o2_out[8];       // f32 plane per output channel, indexed by output pixel
  // kEpiQKV
  __half* vt;             // [nseq][H][64][ld_vt]
  int vt_seqlen, vt_ld, vt_d;  // tokens per attention sequence, row pitch (>= seqlen, %8), model dim D
};

#ifdef __CUDACC__
// Output activation of the fused out2b epilogue (src/dpt_head.cpp:327-338, :402-439).
__device__ __forceinline__ float out_act(float l, int a, float scale) {
  switch (a) {
    case kOutRelu: return fmaxf(l, 0.0f);
    case kOutSigmoidScale: return scale / (1.0f + expf(-l));
    case kOutExp: return expf(l);
    case kOutExpP1: return expf(l) + 1.0f;
    default: return l;
  }
}
#endif

}  // namespace da3b
