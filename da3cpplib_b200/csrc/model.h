// Model configuration and device-resident weights of the depth path.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <memory>
#include <string>
#include <vector>

#include "gguf.h"

namespace da3b {

// Mirrors da::Config (src/model_loader.hpp:11-29); same GGUF keys and defaults
// (src/model_loader.cpp:86-142).
struct Config {
  int patch_size = 14;
  int embed_dim = 0, depth = 0, num_heads = 0, head_dim = 0, mlp_hidden = 0, num_register = 0, pos_embed_grid = 0;
  int alt_start = -1, rope_start = -1, qknorm_start = -1;
  float init_values = 0.f, rope_freq = 100.f, ln_eps = 1e-6f, interp_offset = 0.1f;
  bool cat_token = true, qkv_bias = true, interp_antialias = false, head_pos_embed = true;
  std::string ffn_type = "mlp";
  int head_features = 0;
  std::vector<int32_t> out_layers, head_out_channels;
  std::vector<float> img_mean, img_std;
  int img_resize_target = 504;
  std::string img_resize_mode = "upper_bound";
  std::string checkpoint_name;
  float head_max_depth = 0.f;
  std::string arch = "depthanything3";
  bool metric_branch = false;  // read from m_vit.* / m_head.* keys (nested metric GGUF)

  bool is_da2() const { return arch == "depthanything2"; }
};

// f16 GEMM weight [N][K] (ld = ldw) with optional f32 bias [N]. A ViT block linear
// kept quantised holds its GGUF Q8_0 bytes [N][K/32][34] in q8 instead (w == nullptr);
// the engine dequantises it into its per-block staging buffer ahead of the block.
struct Lin {
  __half* w = nullptr;
  const uint8_t* q8 = nullptr;  // planar Q8_0 (q8planar.cuh) when resident quantised
  float* b = nullptr;
  int N = 0, K = 0, ldw = 0;
};
// Implicit-GEMM conv weight packed [OC][ks*ks][icp] f16, bias f32 [OC] or null.
struct Conv {
  __half* w = nullptr;
  float* b = nullptr;
  int OC = 0, IC = 0, ks = 0;
};
// Stride==kernel transposed conv as GEMM weight [S*S*OC][IC] (row (ky*S+kx)*OC+oc).
struct ConvT {
  __half* w = nullptr;
  float* b = nullptr;
  int OC = 0, IC = 0, S = 0;
};
struct Block {
  float *n1g = nullptr, *n1b = nullptr, *n2g = nullptr, *n2b = nullptr, *ls1 = nullptr, *ls2 = nullptr;
  float *qng = nullptr, *qnb = nullptr, *kng = nullptr, *knb = nullptr;
  Lin qkv, proj, fc1, fc2;
};
struct Fusion {
  bool has_rc1 = false;
  Conv rc1c1, rc1c2, rc2c1, rc2c2;
  Lin out;  // 1x1 conv as GEMM [F][F]
};
struct Head {
  float *norm_g = nullptr, *norm_b = nullptr;
  Lin proj[4];
  ConvT rs0, rs1;
  Conv rs3;  // 3x3 stride-2 (im2col + GEMM, K = 9*icp)
  Conv rn[4];
  Fusion fu[4];  // index 0..3 = refinenet1..4
  Conv out1, out2a;
  float *out2b_w = nullptr, *out2b_b = nullptr;
  int od = 0;
  bool aux = false;
  Fusion fa[4];
  Conv out1_aux[5], out2a_aux;
  float *aux_ln_g = nullptr, *aux_ln_b = nullptr, *out2b_aux_w = nullptr, *out2b_aux_b = nullptr;
  int aux_od = 0;
  // Sky head of the metric / mono DPT (src/dpt_head.cpp:205-222): 3x3 feat/2 -> 32,
  // relu, 1x1 32 -> 1 on the upsampled feature map.
  bool sky = false;
  Conv sky_out2a;
  float *sky_out2b_w = nullptr, *sky_out2b_b = nullptr;
};

// Camera decoder of DA3 (src/cam_pose.cpp:20-32): relu(bb0) -> relu(bb2) -> fc_t (3) |
// fc_q (4) | relu(fc_fov) (2) on the out-layer-3 camera token.
struct CamDec {
  bool present = false;
  Lin bb0, bb2, fc_t, fc_q, fc_fov;
};

class DeviceModel {
 public:
  ~DeviceModel();
  // Loads the GGUF, validates the architecture and uploads / repacks the weights
  // to the current device. Returns null with *err set on failure.
  static std::unique_ptr<DeviceModel> load(const std::string& path, std::string* err);

  Config cfg;
  GgufFile file;
  int patch_k = 0, patch_ldk = 0;  // 3*P*P and its padded GEMM width
  Lin patch;                       // [D][patch_ldk]
  float* cls = nullptr;            // [D]
  float* cam = nullptr;            // [2][D] or null
  float *norm_g = nullptr, *norm_b = nullptr;
  std::vector<Block> blk;
  Head head;
  CamDec camdec;
  size_t weight_bytes = 0;
  // true: the ViT block linears stay resident as Q8_0 (Lin::q8) and block_stage_elems
  // is the f16 element count of one block's four linears (the staging buffer size);
  // false ($DA3B_F16_WEIGHTS=1 at load): they are dequantised once to resident f16.
  bool q8_resident = false;
  size_t block_stage_elems = 0;

  // host views used for per-resolution tables
  const float* pos_embed_host() const;

 private:
  std::vector<void*> allocs_;
  void* dalloc(size_t bytes);
  float* up_f32(const std::string& name, bool required, std::string* err);
  bool lin_q8(const std::string& wname, const std::string& bname, Lin& out, std::string* err,
              bool keep_q8 = false);
  bool lin_f32_1x1(const std::string& wname, const std::string& bname, Lin& out, std::string* err);
  bool conv(const std::string& wname, const std::string& bname, Conv& out, std::string* err);
  bool convT(const std::string& wname, const std::string& bname, int S, ConvT& out, std::string* err);
  bool fusion(const std::string& prefix, Fusion& f, std::string* err);
};

bool read_config(const GgufFile& f, Config& c, std::string* err);

}  // namespace da3b
