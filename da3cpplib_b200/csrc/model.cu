// GGUF -> device weights. Each tensor is uploaded once and repacked into the layout
// its kernel reads (f16 K-major GEMM planes, implicit-GEMM conv packs); the GGUF file
// itself is untouched. Q8_0 linears are dequantised to f16 planes on the device.
#include "model.h"

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdlib.h>
#include <string.h>

#include "ops.h"
#include "q8planar.cuh"

namespace da3b {

int pack_conv_weight(const float* w, int OC, int IC, int ks, __half* out, cudaStream_t s);

namespace {

// w torch ConvTranspose2d [IC][OC][S][S] (ggml [KW,KH,OC,IC]) -> [(ky*S+kx)*OC + oc][IC] f16
__global__ void k_pack_convT(const float* __restrict__ w, int IC, int OC, int S, __half* __restrict__ out) {
  const long total = static_cast<long>(S) * S * OC * IC;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int ic = static_cast<int>(i % IC);
    const long r = i / IC;
    const int oc = static_cast<int>(r % OC);
    const int g = static_cast<int>(r / OC);
    const int ky = g / S, kx = g % S;
    out[i] = __float2half_rn(w[((static_cast<size_t>(ic) * OC + oc) * S + ky) * S + kx]);
  }
}

// f32 [rows][K] -> f16 [rows][ldk], zero padded
__global__ void k_cast_pad(const float* __restrict__ w, int rows, int K, int ldk, __half* __restrict__ out) {
  const long total = static_cast<long>(rows) * ldk;
  for (long i = static_cast<long>(blockIdx.x) * blockDim.x + threadIdx.x; i < total;
       i += static_cast<long>(gridDim.x) * blockDim.x) {
    const int k = static_cast<int>(i % ldk);
    const long r = i / ldk;
    out[i] = __float2half_rn(k < K ? w[r * K + k] : 0.f);
  }
}

unsigned blocks_for(long n) {
  long b = (n + 255) / 256;
  return static_cast<unsigned>(b > 65535 ? 65535 : (b < 1 ? 1 : b));
}

}  // namespace

bool read_config(const GgufFile& f, Config& c, std::string* err) {
  const std::string P = "depthanything3.";
  // A nested metric-branch file carries its structure under m_vit.* / m_head.*; its
  // head has no UV pos-embed unless m_head.pos_embed says so (src/model_loader.cpp:84-127).
  const bool metric = f.kv(P + "m_vit.embed_dim") != nullptr;
  const std::string V = P + (metric ? "m_vit." : "vit."), Hd = P + (metric ? "m_head." : "head.");
  c.patch_size = static_cast<int>(f.get_u32(P + "patch_size", 14));
  c.embed_dim = static_cast<int>(f.get_u32(V + "embed_dim", 0));
  c.depth = static_cast<int>(f.get_u32(V + "depth", 0));
  c.num_heads = static_cast<int>(f.get_u32(V + "num_heads", 0));
  c.head_dim = static_cast<int>(f.get_u32(V + "head_dim", 0));
  c.mlp_hidden = static_cast<int>(f.get_u32(V + "mlp_hidden", 0));
  c.num_register = static_cast<int>(f.get_u32(V + "num_register_tokens", 0));
  c.pos_embed_grid = static_cast<int>(f.get_u32(V + "pos_embed_grid", 0));
  c.alt_start = f.get_i32(V + "alt_start", -1);
  c.rope_start = f.get_i32(V + "rope_start", -1);
  c.qknorm_start = f.get_i32(V + "qknorm_start", -1);
  c.init_values = f.get_f32(V + "init_values", 0.f);
  c.rope_freq = f.get_f32(V + "rope_freq", 100.f);
  c.ln_eps = f.get_f32(V + "ln_eps", 1e-6f);
  c.interp_offset = f.get_f32(V + "interpolate_offset", 0.1f);
  c.cat_token = f.get_bool(V + "cat_token", true);
  c.qkv_bias = f.get_bool(V + "qkv_bias", true);
  c.interp_antialias = f.get_bool(V + "interpolate_antialias", false);
  c.ffn_type = f.get_str(V + "ffn_type", "mlp");
  c.head_features = static_cast<int>(f.get_u32(Hd + "features", 0));
  c.out_layers = f.get_i32_arr(V + "out_layers");
  c.head_out_channels = f.get_i32_arr(Hd + "out_channels");
  c.head_pos_embed = f.get_bool(Hd + "pos_embed", !metric);
  c.metric_branch = metric;
  c.img_mean = f.get_f32_arr(P + "img.mean");
  c.img_std = f.get_f32_arr(P + "img.std");
  c.img_resize_target = static_cast<int>(f.get_u32(P + "img.resize_target", 504));
  c.img_resize_mode = f.get_str(P + "img.resize_mode", "upper_bound");
  c.checkpoint_name = f.get_str(P + "checkpoint_name", "");
  c.head_max_depth = f.get_f32(P + "head.max_depth", 0.f);
  c.arch = f.get_str(P + "arch", "depthanything3");
  if (c.embed_dim <= 0 || c.depth <= 0 || c.num_heads <= 0 || c.head_dim <= 0) {
    if (err) *err = "GGUF lacks the ViT structure keys";
    return false;
  }
  if (c.head_dim != 64 || c.num_heads * c.head_dim != c.embed_dim) {
    if (err) *err = "only head_dim 64 with embed_dim = heads * 64 is supported";
    return false;
  }
  if (c.ffn_type != "mlp") {
    if (err) *err = "SwiGLU FFN (ffn_type=swiglu) is outside the supported depth path";
    return false;
  }
  if (c.out_layers.size() != 4) {
    if (err) *err = "expected 4 out_layers";
    return false;
  }
  if (c.img_mean.size() < 3 || c.img_std.size() < 3) {
    if (err) *err = "GGUF lacks img.mean / img.std";
    return false;
  }
  return true;
}

DeviceModel::~DeviceModel() {
  for (void* p : allocs_) cudaFree(p);
}

void* DeviceModel::dalloc(size_t bytes) {
  void* p = nullptr;
  if (cudaMalloc(&p, bytes < 256 ? 256 : bytes) != cudaSuccess) return nullptr;
  allocs_.push_back(p);
  weight_bytes += bytes;
  return p;
}

const float* DeviceModel::pos_embed_host() const {
  const GgufTensor* t = file.tensor("vit.pos_embed");
  return t && t->type == 0 ? reinterpret_cast<const float*>(t->data) : nullptr;
}

float* DeviceModel::up_f32(const std::string& name, bool required, std::string* err) {
  const GgufTensor* t = file.tensor(name);
  if (!t) {
    if (required && err) *err = "missing tensor " + name;
    return nullptr;
  }
  if (t->type != 0) {
    if (err) *err = "tensor " + name + " must be f32";
    return nullptr;
  }
  float* d = static_cast<float*>(dalloc(t->nbytes));
  if (!d || cudaMemcpy(d, t->data, t->nbytes, cudaMemcpyHostToDevice) != cudaSuccess) {
    if (err) *err = "upload failed for " + name;
    return nullptr;
  }
  return d;
}

bool DeviceModel::lin_q8(const std::string& wname, const std::string& bname, Lin& out, std::string* err,
                         bool keep_q8) {
  const GgufTensor* t = file.tensor(wname);
  if (!t) { if (err) *err = "missing tensor " + wname; return false; }
  const int K = static_cast<int>(t->ne[0]), N = static_cast<int>(t->ne[1]);
  out.N = N;
  out.K = K;
  out.ldw = K;
  if (K % 32) { if (err) *err = "K not a multiple of 32 in " + wname; return false; }
  if (keep_q8 && t->type == 8) {
    // resident as the GGUF's Q8_0 bytes in planar form (q8planar.cuh: the int8 plane and
    // the transposed f16 scale plane, the same byte count); per forward either the GEMM
    // dequantises its weight tiles itself or a staging kernel writes f16 ahead of a block
    if (q8p_bytes(N, K) != t->nbytes) { if (err) *err = "unexpected Q8_0 size of " + wname; return false; }
    uint8_t* q = static_cast<uint8_t*>(dalloc(t->nbytes));
    void* raw = nullptr;
    bool ok = q && cudaMalloc(&raw, t->nbytes) == cudaSuccess &&
              cudaMemcpy(raw, t->data, t->nbytes, cudaMemcpyHostToDevice) == cudaSuccess &&
              repack_q8_0_planar(raw, N, K, q, nullptr) == 0 && cudaDeviceSynchronize() == cudaSuccess;
    if (raw) cudaFree(raw);
    if (!ok) {
      if (err) *err = "Q8_0 upload failed for " + wname;
      return false;
    }
    out.q8 = q;
    if (!bname.empty()) out.b = up_f32(bname, false, err);
    return true;
  }
  out.w = static_cast<__half*>(dalloc(static_cast<size_t>(N) * K * 2));
  if (!out.w) { if (err) *err = "out of device memory"; return false; }
  if (t->type == 8) {
    void* raw = nullptr;
    if (cudaMalloc(&raw, t->nbytes) != cudaSuccess) { if (err) *err = "out of device memory"; return false; }
    bool ok = cudaMemcpy(raw, t->data, t->nbytes, cudaMemcpyHostToDevice) == cudaSuccess &&
              dequant_q8_0(raw, N, K, out.w, K, nullptr) == 0 && cudaDeviceSynchronize() == cudaSuccess;
    cudaFree(raw);
    if (!ok) { if (err) *err = "Q8_0 repack failed for " + wname; return false; }
  } else if (t->type == 0) {
    float* raw = nullptr;
    if (cudaMalloc(&raw, t->nbytes) != cudaSuccess) { if (err) *err = "out of device memory"; return false; }
    bool ok = cudaMemcpy(raw, t->data, t->nbytes, cudaMemcpyHostToDevice) == cudaSuccess;
    if (ok) {
      k_cast_pad<<<blocks_for(static_cast<long>(N) * K), 256>>>(raw, N, K, K, out.w);
      ok = cudaDeviceSynchronize() == cudaSuccess;
    }
    cudaFree(raw);
    if (!ok) { if (err) *err = "f32 linear repack failed for " + wname; return false; }
  } else {
    if (err) *err = "unsupported linear weight type in " + wname;
    return false;
  }
  if (!bname.empty()) {
    out.b = up_f32(bname, false, err);
  }
  return true;
}

bool DeviceModel::lin_f32_1x1(const std::string& wname, const std::string& bname, Lin& out, std::string* err) {
  const GgufTensor* t = file.tensor(wname);
  if (!t || t->type != 0) { if (err) *err = "missing/non-f32 tensor " + wname; return false; }
  // ggml conv kernel [1,1,IC,OC] == row-major [OC][IC]
  const int IC = static_cast<int>(t->ne[2] * t->ne[1] * t->ne[0]), OC = static_cast<int>(t->ne[3]);
  out.N = OC;
  out.K = IC;
  out.ldw = (IC + 7) / 8 * 8;
  float* raw = static_cast<float*>(nullptr);
  if (cudaMalloc(&raw, t->nbytes) != cudaSuccess) { if (err) *err = "out of device memory"; return false; }
  out.w = static_cast<__half*>(dalloc(static_cast<size_t>(OC) * out.ldw * 2));
  bool ok = out.w && cudaMemcpy(raw, t->data, t->nbytes, cudaMemcpyHostToDevice) == cudaSuccess;
  if (ok) {
    k_cast_pad<<<blocks_for(static_cast<long>(OC) * out.ldw), 256>>>(raw, OC, IC, out.ldw, out.w);
    ok = cudaDeviceSynchronize() == cudaSuccess;
  }
  cudaFree(raw);
  if (!ok) { if (err) *err = "1x1 repack failed for " + wname; return false; }
  if (!bname.empty()) out.b = up_f32(bname, false, err);
  return true;
}

bool DeviceModel::conv(const std::string& wname, const std::string& bname, Conv& out, std::string* err) {
  const GgufTensor* t = file.tensor(wname);
  if (!t || t->type != 0) { if (err) *err = "missing/non-f32 conv " + wname; return false; }
  out.ks = static_cast<int>(t->ne[0]);
  out.IC = static_cast<int>(t->ne[2]);
  out.OC = static_cast<int>(t->ne[3]);
  if (t->ne[1] != out.ks || (out.ks != 1 && out.ks != 3)) { if (err) *err = "unsupported conv kernel " + wname; return false; }
  const int icp = conv_icp(out.IC);
  float* raw = nullptr;
  if (cudaMalloc(&raw, t->nbytes) != cudaSuccess) { if (err) *err = "out of device memory"; return false; }
  out.w = static_cast<__half*>(dalloc(static_cast<size_t>(out.OC) * out.ks * out.ks * icp * 2));
  bool ok = out.w && cudaMemcpy(raw, t->data, t->nbytes, cudaMemcpyHostToDevice) == cudaSuccess &&
            pack_conv_weight(raw, out.OC, out.IC, out.ks, out.w, nullptr) == 0 && cudaDeviceSynchronize() == cudaSuccess;
  cudaFree(raw);
  if (!ok) { if (err) *err = "conv repack failed for " + wname; return false; }
  if (!bname.empty()) out.b = up_f32(bname, false, err);
  return true;
}

bool DeviceModel::convT(const std::string& wname, const std::string& bname, int S, ConvT& out, std::string* err) {
  const GgufTensor* t = file.tensor(wname);
  if (!t || t->type != 0) { if (err) *err = "missing/non-f32 convT " + wname; return false; }
  if (t->ne[0] != S || t->ne[1] != S) { if (err) *err = "convT kernel != stride in " + wname; return false; }
  out.S = S;
  out.OC = static_cast<int>(t->ne[2]);
  out.IC = static_cast<int>(t->ne[3]);
  float* raw = nullptr;
  if (cudaMalloc(&raw, t->nbytes) != cudaSuccess) { if (err) *err = "out of device memory"; return false; }
  out.w = static_cast<__half*>(dalloc(static_cast<size_t>(S) * S * out.OC * out.IC * 2));
  bool ok = out.w && cudaMemcpy(raw, t->data, t->nbytes, cudaMemcpyHostToDevice) == cudaSuccess;
  if (ok) {
    k_pack_convT<<<blocks_for(static_cast<long>(S) * S * out.OC * out.IC), 256>>>(raw, out.IC, out.OC, S, out.w);
    ok = cudaDeviceSynchronize() == cudaSuccess;
  }
  cudaFree(raw);
  if (!ok) { if (err) *err = "convT repack failed for " + wname; return false; }
  out.b = up_f32(bname, false, err);
  return true;
}

bool DeviceModel::fusion(const std::string& p, Fusion& f, std::string* err) {
  f.has_rc1 = file.tensor(p + "rc1.c1.weight") != nullptr;
  if (f.has_rc1) {
    if (!conv(p + "rc1.c1.weight", p + "rc1.c1.bias", f.rc1c1, err)) return false;
    if (!conv(p + "rc1.c2.weight", p + "rc1.c2.bias", f.rc1c2, err)) return false;
  }
  if (!conv(p + "rc2.c1.weight", p + "rc2.c1.bias", f.rc2c1, err)) return false;
  if (!conv(p + "rc2.c2.weight", p + "rc2.c2.bias", f.rc2c2, err)) return false;
  return lin_f32_1x1(p + "out.weight", p + "out.bias", f.out, err);
}

std::unique_ptr<DeviceModel> DeviceModel::load(const std::string& path, std::string* err) {
  std::unique_ptr<DeviceModel> m(new DeviceModel());
  if (!m->file.open(path, err)) return nullptr;
  if (!read_config(m->file, m->cfg, err)) return nullptr;
  const Config& c = m->cfg;
  const int D = c.embed_dim, P = c.patch_size;
  // patch embed [D][3][P][P] f32 -> f16 [D][ldk]
  {
    const GgufTensor* t = m->file.tensor("vit.patch_embed.weight");
    if (!t || t->type != 0 || t->ne[3] != D) { if (err) *err = "bad vit.patch_embed.weight"; return nullptr; }
    m->patch_k = 3 * P * P;
    m->patch_ldk = (m->patch_k + 63) / 64 * 64;
    float* raw = nullptr;
    if (cudaMalloc(&raw, t->nbytes) != cudaSuccess) { if (err) *err = "out of device memory"; return nullptr; }
    m->patch.w = static_cast<__half*>(m->dalloc(static_cast<size_t>(D) * m->patch_ldk * 2));
    bool ok = m->patch.w && cudaMemcpy(raw, t->data, t->nbytes, cudaMemcpyHostToDevice) == cudaSuccess;
    if (ok) {
      k_cast_pad<<<blocks_for(static_cast<long>(D) * m->patch_ldk), 256>>>(raw, D, m->patch_k, m->patch_ldk, m->patch.w);
      ok = cudaDeviceSynchronize() == cudaSuccess;
    }
    cudaFree(raw);
    if (!ok) { if (err) *err = "patch embed repack failed"; return nullptr; }
    m->patch.N = D;
    m->patch.K = m->patch_k;
    m->patch.ldw = m->patch_ldk;
    if (!(m->patch.b = m->up_f32("vit.patch_embed.bias", true, err))) return nullptr;
  }
  if (!(m->cls = m->up_f32("vit.cls_token", true, err))) return nullptr;
  if (!m->pos_embed_host()) { if (err) *err = "missing f32 vit.pos_embed"; return nullptr; }
  m->cam = m->file.tensor("vit.camera_token") ? m->up_f32("vit.camera_token", true, err) : nullptr;
  if (!(m->norm_g = m->up_f32("vit.norm.weight", true, err))) return nullptr;
  m->norm_b = m->up_f32("vit.norm.bias", false, err);
  m->blk.resize(c.depth);
  {
    const GgufTensor* q0 = m->file.tensor("vit.blk.0.attn_qkv.weight");
    const char* f16 = getenv("DA3B_F16_WEIGHTS");
    m->q8_resident = q0 && q0->type == 8 && !(f16 && f16[0] == '1');
  }
  for (int i = 0; i < c.depth; ++i) {
    const std::string p = "vit.blk." + std::to_string(i) + ".";
    Block& b = m->blk[i];
    if (!(b.n1g = m->up_f32(p + "norm1.weight", true, err))) return nullptr;
    b.n1b = m->up_f32(p + "norm1.bias", false, err);
    if (!(b.n2g = m->up_f32(p + "norm2.weight", true, err))) return nullptr;
    b.n2b = m->up_f32(p + "norm2.bias", false, err);
    b.ls1 = m->up_f32(p + "ls1", false, err);
    b.ls2 = m->up_f32(p + "ls2", false, err);
    if (m->file.tensor(p + "attn_qnorm.weight")) {
      b.qng = m->up_f32(p + "attn_qnorm.weight", true, err);
      b.qnb = m->up_f32(p + "attn_qnorm.bias", false, err);
      b.kng = m->up_f32(p + "attn_knorm.weight", true, err);
      b.knb = m->up_f32(p + "attn_knorm.bias", false, err);
      if (!b.qng || !b.kng) return nullptr;
    }
    const bool kq = m->q8_resident;
    if (!m->lin_q8(p + "attn_qkv.weight", p + "attn_qkv.bias", b.qkv, err, kq)) return nullptr;
    if (!m->lin_q8(p + "attn_proj.weight", p + "attn_proj.bias", b.proj, err, kq)) return nullptr;
    if (!m->lin_q8(p + "mlp_fc1.weight", p + "mlp_fc1.bias", b.fc1, err, kq)) return nullptr;
    if (!m->lin_q8(p + "mlp_fc2.weight", p + "mlp_fc2.bias", b.fc2, err, kq)) return nullptr;
    if (b.qkv.N != 3 * D || b.qkv.K != D || b.fc1.K != D || b.fc2.N != D || b.proj.N != D || b.proj.K != D ||
        b.fc2.K != b.fc1.N) {
      if (err) *err = "inconsistent block shapes in block " + std::to_string(i);
      return nullptr;
    }
    // a model whose block linears are Q8_0 keeps all of them quantised; a block with
    // another weight type there is rejected rather than mixed
    if (kq && !(b.qkv.q8 && b.proj.q8 && b.fc1.q8 && b.fc2.q8)) {
      if (err) *err = "block " + std::to_string(i) + " mixes Q8_0 and other linear weight types";
      return nullptr;
    }
    const size_t st = static_cast<size_t>(b.qkv.N) * D + static_cast<size_t>(D) * D +
                      static_cast<size_t>(b.fc1.N) * D * 2;
    if (st > m->block_stage_elems) m->block_stage_elems = st;
  }
  if (m->file.tensor("cam.bb0.weight")) {
    CamDec& cd = m->camdec;
    if (!m->lin_q8("cam.bb0.weight", "cam.bb0.bias", cd.bb0, err) ||
        !m->lin_q8("cam.bb2.weight", "cam.bb2.bias", cd.bb2, err) ||
        !m->lin_q8("cam.fc_t.weight", "cam.fc_t.bias", cd.fc_t, err) ||
        !m->lin_q8("cam.fc_q.weight", "cam.fc_q.bias", cd.fc_q, err) ||
        !m->lin_q8("cam.fc_fov.weight", "cam.fc_fov.bias", cd.fc_fov, err))
      return nullptr;
    if (cd.bb2.K != cd.bb0.N || cd.fc_t.K != cd.bb2.N || cd.fc_q.K != cd.bb2.N || cd.fc_fov.K != cd.bb2.N ||
        cd.fc_t.N != 3 || cd.fc_q.N != 4 || cd.fc_fov.N != 2) {
      if (err) *err = "camera decoder shapes do not chain";
      return nullptr;
    }
    cd.present = true;
  }
  // ---- DPT head (tensor names: src/dpt_head.cpp:108-272)
  Head& h = m->head;
  if (m->file.tensor("head.norm.weight")) {
    if (!(h.norm_g = m->up_f32("head.norm.weight", true, err))) return nullptr;
    h.norm_b = m->up_f32("head.norm.bias", false, err);
  }
  for (int s = 0; s < 4; ++s) {
    const std::string ss = std::to_string(s);
    if (!m->lin_f32_1x1("head.proj." + ss + ".weight", "head.proj." + ss + ".bias", h.proj[s], err)) return nullptr;
  }
  if (!m->convT("head.resize.0.weight", "head.resize.0.bias", 4, h.rs0, err)) return nullptr;
  if (!m->convT("head.resize.1.weight", "head.resize.1.bias", 2, h.rs1, err)) return nullptr;
  if (!m->conv("head.resize.3.weight", "head.resize.3.bias", h.rs3, err)) return nullptr;
  for (int s = 0; s < 4; ++s)
    if (!m->conv("head.scratch.layer" + std::to_string(s + 1) + "_rn.weight", "", h.rn[s], err)) return nullptr;
  for (int r = 0; r < 4; ++r)
    if (!m->fusion("head.scratch.rn" + std::to_string(r + 1) + ".", h.fu[r], err)) return nullptr;
  if (!m->conv("head.scratch.out1.weight", "head.scratch.out1.bias", h.out1, err)) return nullptr;
  if (!m->conv("head.scratch.out2a.weight", "head.scratch.out2a.bias", h.out2a, err)) return nullptr;
  if (h.out2a.OC != 32) { if (err) *err = "out2a must have 32 output channels"; return nullptr; }
  {
    const GgufTensor* t = m->file.tensor("head.scratch.out2b.weight");
    if (!t || t->ne[2] != 32 || t->ne[3] < 1 || t->ne[3] > 8) { if (err) *err = "bad head.scratch.out2b.weight"; return nullptr; }
    h.od = static_cast<int>(t->ne[3]);
    if (!(h.out2b_w = m->up_f32("head.scratch.out2b.weight", true, err))) return nullptr;
    if (!(h.out2b_b = m->up_f32("head.scratch.out2b.bias", true, err))) return nullptr;
  }
  if (m->file.tensor("head.scratch.sky_out2b.weight")) {
    if (!m->conv("head.scratch.sky_out2a.weight", "head.scratch.sky_out2a.bias", h.sky_out2a, err)) return nullptr;
    const GgufTensor* t = m->file.tensor("head.scratch.sky_out2b.weight");
    if (h.sky_out2a.OC != 32 || h.sky_out2a.ks != 3 || h.sky_out2a.IC != h.out2a.IC || t->ne[2] != 32 || t->ne[3] != 1) {
      if (err) *err = "sky head must be 3x3 feat/2 -> 32 then 1x1 32 -> 1";
      return nullptr;
    }
    if (!(h.sky_out2b_w = m->up_f32("head.scratch.sky_out2b.weight", true, err))) return nullptr;
    if (!(h.sky_out2b_b = m->up_f32("head.scratch.sky_out2b.bias", true, err))) return nullptr;
    h.sky = true;
  }
  h.aux = m->file.tensor("head.scratch.rn1_aux.out.weight") != nullptr;
  if (h.aux) {
    for (int r = 0; r < 4; ++r)
      if (!m->fusion("head.scratch.rn" + std::to_string(r + 1) + "_aux.", h.fa[r], err)) return nullptr;
    for (int i = 0; i < 5; ++i) {
      const std::string p = "head.scratch.out1_aux." + std::to_string(i) + ".";
      if (!m->conv(p + "weight", p + "bias", h.out1_aux[i], err)) return nullptr;
    }
    if (!m->conv("head.scratch.out2a_aux.weight", "head.scratch.out2a_aux.bias", h.out2a_aux, err)) return nullptr;
    if (!(h.aux_ln_g = m->up_f32("head.scratch.out2_aux_ln.weight", true, err))) return nullptr;
    h.aux_ln_b = m->up_f32("head.scratch.out2_aux_ln.bias", false, err);
    const GgufTensor* t = m->file.tensor("head.scratch.out2b_aux.weight");
    if (!t || t->ne[2] != 32 || t->ne[3] < 1 || t->ne[3] > 8) { if (err) *err = "bad out2b_aux"; return nullptr; }
    h.aux_od = static_cast<int>(t->ne[3]);
    if (!(h.out2b_aux_w = m->up_f32("head.scratch.out2b_aux.weight", true, err))) return nullptr;
    if (!(h.out2b_aux_b = m->up_f32("head.scratch.out2b_aux.bias", true, err))) return nullptr;
    if (h.out2a_aux.OC != 32) { if (err) *err = "out2a_aux must have 32 channels"; return nullptr; }
  }
  if (cudaDeviceSynchronize() != cudaSuccess) { if (err) *err = "device error during load"; return nullptr; }
  return m;
}

}  // namespace da3b
