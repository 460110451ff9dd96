// Forward of the depth path on one device.
//
// Backbone (per ViT block, M = n_views * tokens rows; the residual stream x is f32):
//   LN1 -> QKV GEMM(+bias) -> [QK-norm + RoPE] -> flash attention -> proj GEMM with
//   x += ls1*(acc+b) epilogue -> LN2 -> fc1 GEMM(+bias, erf-GELU) -> fc2 GEMM with
//   x += ls2*(acc+b); out-layer features are LayerNormed straight into the head's
//   NHWC input (src/vit_block.cpp:30-58, src/dino_backbone.cpp:80-311, :462-616).
// DPT head (NHWC f16, all views batched): projections (+UV PE), reassemble convT as
// GEMM with a pixel-shuffle store, stride-2 conv via im2col, layer_rn convs, four
// fusion levels whose residual adds / ReLUs live in the conv epilogues, out1,
// upsample(+PE) and out2a with out2b + the output activation fused in its epilogue
// (src/dpt_head.cpp:75-275, src/dpt_blocks.cpp:18-143).
#include "engine.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <type_traits>

#include "kernels.h"
#include "ops.h"

namespace da3b {

// ------------------------------------------------------------------ per-shape plan
struct Arena {
  char* base = nullptr;
  size_t size = 0, used = 0;
  template <typename T>
  T* take(size_t count) {
    const size_t bytes = (count * sizeof(T) + 255) / 256 * 256;
    if (!base) {  // sizing pass
      used += bytes;
      return nullptr;
    }
    if (used + bytes > size) return nullptr;
    T* p = reinterpret_cast<T*>(base + used);
    used += bytes;
    return p;
  }
};

struct Level {
  int h = 0, w = 0;
  __half *T = nullptr, *Y1 = nullptr, *Y1r = nullptr, *Y2 = nullptr, *Z = nullptr;
};

struct Plan {
  int V = 0, S = 0, scenes = 0, H = 0, W = 0, gh = 0, gw = 0, Np = 0, Ntok = 0, M = 0;
  bool rays = false;
  // true: upsample + output_conv2 run fused (up_out2, no full-resolution feature map);
  // false ($DA3B_UNFUSED_UP=1 at plan creation): upsample_ac into O1u, then conv_nhwc
  bool fused_up = true;
  int ho3 = 0, wo3 = 0;  // stride-2 stage grid
  int Cf = 0;            // feature channels (D or 2D)
  Arena arena;
  // inputs / outputs owned by the plan (the captured graph reads / writes these)
  uint8_t* rgb = nullptr;
  float *depth = nullptr, *conf = nullptr, *raysbuf = nullptr, *sky = nullptr;
  // backbone
  float *x = nullptr, *x2 = nullptr, *pos = nullptr;
  float *rl_cos = nullptr, *rl_sin = nullptr, *rn_cos = nullptr, *rn_sin = nullptr;
  __half *patchA = nullptr, *xn = nullptr, *qkv = nullptr, *attn = nullptr, *hid = nullptr;
  __half* vt = nullptr;   // transposed V [nseq][H][64][ld] written by the QKV epilogue
  int ld_vt_local = 0, ld_vt_global = 0;
  __half* feats[4] = {nullptr, nullptr, nullptr, nullptr};
  __half* ftmp[4] = {nullptr, nullptr, nullptr, nullptr};
  __half* featn[4] = {nullptr, nullptr, nullptr, nullptr};  // head-LayerNormed features (DA3)
  int* b_idx = nullptr;
  float* resid_cap = nullptr;  // [depth][M][D] residual after each block (capture mode only)
  // head
  __half* P[4] = {nullptr, nullptr, nullptr, nullptr};
  __half *L0 = nullptr, *L1 = nullptr, *L3 = nullptr, *A3 = nullptr;
  __half* RN[4] = {nullptr, nullptr, nullptr, nullptr};
  __half* RNr[4] = {nullptr, nullptr, nullptr, nullptr};
  Level lv[4];  // 0 = 4gh (refinenet1) ... 3 = stride-2 grid (refinenet4)
  __half* U[4] = {nullptr, nullptr, nullptr, nullptr};  // upsampled outputs at lv2, lv1, lv0, 8gh
  __half *O1 = nullptr, *O1u = nullptr, *auxA = nullptr, *auxB = nullptr;
  __half* pe_proj[4] = {nullptr, nullptr, nullptr, nullptr};
  __half *pe_full = nullptr, *pe_aux = nullptr;
  int launches = 0;
  cudaGraphExec_t graph = nullptr;
  bool warmed = false;
  // prepared input (infer_preprocessed): normalised planar f32 [V][3][H][W], allocated on
  // first use, with its own captured graph (the first kernel reads it instead of rgb)
  float* chw = nullptr;
  bool prepared = false;
  // camera tokens of out-layer 3 in processing order [V][Cf] f32 and the camera
  // decoder's activations [V][hidden] x 2 and pose encodings [V][9] (DA3 with cam.*)
  float *cam = nullptr, *cam_h1 = nullptr, *cam_h2 = nullptr, *cam_pe = nullptr;
  cudaGraphExec_t graph_pre = nullptr;
  bool warmed_pre = false;
  ~Plan() {
    if (graph) cudaGraphExecDestroy(graph);
    if (graph_pre) cudaGraphExecDestroy(graph_pre);
    if (chw) cudaFree(chw);
    if (arena.base) cudaFree(arena.base);
  }
};

Engine::~Engine() {
  if (device_ >= 0) cudaSetDevice(device_);
  plans_.clear();
  if (wstage_) cudaFree(wstage_);
  for (auto& st : side_)
    if (st) cudaStreamDestroy(st);
  for (auto& ev : ev_)
    if (ev) cudaEventDestroy(ev);
  model_.reset();
}

std::unique_ptr<Engine> Engine::create(const std::string& path, int device, std::string* err) {
  if (cudaSetDevice(device) != cudaSuccess) {
    if (err) *err = "cannot select CUDA device " + std::to_string(device);
    return nullptr;
  }
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess || prop.major < 10) {
    if (err) *err = "libda3b needs an sm_100 (Blackwell B200) device";
    return nullptr;
  }
  std::unique_ptr<Engine> e(new Engine());
  e->device_ = device;
  e->status_ = device_status_word();
  if (!e->status_) {
    if (err) *err = "cannot allocate the device status word";
    return nullptr;
  }
  e->model_ = DeviceModel::load(path, err);
  if (!e->model_) return nullptr;
  if (e->model_->q8_resident &&
      cudaMalloc(&e->wstage_, e->model_->block_stage_elems * sizeof(__half)) != cudaSuccess) {
    e->wstage_ = nullptr;
    if (err) *err = "cannot allocate the block weight staging buffer";
    return nullptr;
  }
  if (const char* g = getenv("DA3B_GRAPH")) e->use_graph_ = strcmp(g, "0") != 0;
  if (const char* q = getenv("DA3B_Q8_TILES")) e->q8_tiles_ = q[0] == '1';
  for (auto& st : e->side_)
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
      st = nullptr;
      if (err) *err = "cannot create the head's side streams";
      return nullptr;
    }
  for (auto& ev : e->ev_)
    if (cudaEventCreateWithFlags(&ev, cudaEventDisableTiming) != cudaSuccess) {
      ev = nullptr;
      if (err) *err = "cannot create the head's events";
      return nullptr;
    }
  return e;
}

void Engine::set_act_quant(bool on) {
  if (on == act_quant_) return;
  act_quant_ = on;
  cudaSetDevice(device_);
  cudaDeviceSynchronize();
  last_ = nullptr;
  plans_.clear();
}

void Engine::set_capture_residuals(bool on) {
  if (on == capture_resid_) return;
  capture_resid_ = on;
  cudaSetDevice(device_);
  cudaDeviceSynchronize();
  last_ = nullptr;
  plans_.clear();
}

void Engine::set_raw_logits(bool on) {
  if (on == raw_logits_) return;
  raw_logits_ = on;
  cudaSetDevice(device_);
  cudaDeviceSynchronize();
  last_ = nullptr;
  plans_.clear();
}

HeadKind Engine::head_kind() const {
  const Config& c = model_->cfg;
  if (c.is_da2()) return c.head_max_depth > 0.f ? HeadKind::Da2Metric : HeadKind::Da2Relative;
  return HeadKind::Da3;
}

int Engine::status() {
  int st = 0;
  if (read_and_reset_status(status_, &st)) return -1;
  return st;
}

// ------------------------------------------------------------------ host tables
namespace {

float cubic_a075(float x) {  // Catmull-Rom with a = -0.75 (PyTorch bicubic)
  const float a = -0.75f;
  x = std::fabs(x);
  if (x < 1) return ((a + 2) * x - (a + 3)) * x * x + 1;
  if (x < 2) return (((x - 5) * x + 8) * x - 4) * a;
  return 0;
}

// Bicubic interpolation of the pos-embed grid to gh x gw with the +offset scale and
// border clamp, always applied (src/dino_backbone.cpp:18-56). Row 0 (CLS) copied.
std::vector<float> interp_pos(const float* p, int E, int Mg, int gh, int gw, float offset) {
  std::vector<float> out(static_cast<size_t>(1 + gh * gw) * E);
  for (int ch = 0; ch < E; ++ch) out[ch] = p[ch];
  const float sx = static_cast<float>(gw + offset) / Mg, sy = static_cast<float>(gh + offset) / Mg;
  for (int oy = 0; oy < gh; ++oy) {
    const float iy = (oy + 0.5f) / sy - 0.5f;
    const int y0 = static_cast<int>(std::floor(iy));
    const float fy = iy - y0;
    float wy[4];
    int yy[4];
    for (int m = -1; m <= 2; ++m) {
      wy[m + 1] = cubic_a075(fy - m);
      yy[m + 1] = std::min(std::max(y0 + m, 0), Mg - 1);
    }
    for (int ox = 0; ox < gw; ++ox) {
      const float ix = (ox + 0.5f) / sx - 0.5f;
      const int x0 = static_cast<int>(std::floor(ix));
      const float fx = ix - x0;
      float wx[4];
      int xx[4];
      for (int n = -1; n <= 2; ++n) {
        wx[n + 1] = cubic_a075(fx - n);
        xx[n + 1] = std::min(std::max(x0 + n, 0), Mg - 1);
      }
      float* o = &out[static_cast<size_t>(1 + oy * gw + ox) * E];
      for (int ch = 0; ch < E; ++ch) {
        float acc = 0;
        for (int m = 0; m < 4; ++m)
          for (int n = 0; n < 4; ++n) acc += wy[m] * wx[n] * p[static_cast<size_t>(1 + yy[m] * Mg + xx[n]) * E + ch];
        o[ch] = acc;
      }
    }
  }
  return out;
}

// 2-D RoPE tables (src/rope2d.cpp:4-27) for token positions (y, x): [tokens][64].
void rope_tables(const std::vector<float>& pos, int tokens, float freq, std::vector<float>& cs,
                 std::vector<float>& sn) {
  const int hd = 64, half = 32, quart = 16;
  cs.assign(static_cast<size_t>(hd) * tokens, 0.f);
  sn.assign(static_cast<size_t>(hd) * tokens, 0.f);
  for (int t = 0; t < tokens; ++t) {
    const float y = pos[2 * t], x = pos[2 * t + 1];
    for (int j = 0; j < quart; ++j) {
      const float invf = std::pow(freq, -2.f * static_cast<float>(j) / static_cast<float>(half));
      const float ay = y * invf, ax = x * invf;
      float* c = &cs[static_cast<size_t>(t) * hd];
      float* s = &sn[static_cast<size_t>(t) * hd];
      c[j] = c[j + quart] = std::cos(ay);
      s[j] = s[j + quart] = std::sin(ay);
      c[half + j] = c[half + j + quart] = std::cos(ax);
      s[half + j] = s[half + j + quart] = std::sin(ax);
    }
  }
}

// 0.1 * UV sinusoidal embedding as NHWC [ph*pw][C] f16 (src/uv_posembed.cpp:15-73,
// src/dpt_head.cpp:22-50).
std::vector<__half> uv_table(int pw, int ph, int C, float aspect, float ratio) {
  std::vector<__half> out(static_cast<size_t>(pw) * ph * C);
  const double diag = std::sqrt(static_cast<double>(aspect) * aspect + 1.0);
  const double span_x = aspect / diag, span_y = 1.0 / diag;
  const double left_x = -span_x * (pw - 1) / pw, right_x = span_x * (pw - 1) / pw;
  const double top_y = -span_y * (ph - 1) / ph, bottom_y = span_y * (ph - 1) / ph;
  const int D = C / 2, F = D / 2;
  std::vector<double> om(F);
  for (int j = 0; j < F; ++j) om[j] = 1.0 / std::pow(100.0, static_cast<double>(j) / (static_cast<double>(D) / 2.0));
  for (int y = 0; y < ph; ++y) {
    const double yc = ph == 1 ? top_y : top_y + y * ((bottom_y - top_y) / (ph - 1));
    for (int x = 0; x < pw; ++x) {
      const double xc = pw == 1 ? left_x : left_x + x * ((right_x - left_x) / (pw - 1));
      __half* o = &out[(static_cast<size_t>(y) * pw + x) * C];
      for (int j = 0; j < F; ++j) {
        o[j] = __float2half(ratio * static_cast<float>(std::sin(xc * om[j])));
        o[F + j] = __float2half(ratio * static_cast<float>(std::cos(xc * om[j])));
        o[D + j] = __float2half(ratio * static_cast<float>(std::sin(yc * om[j])));
        o[D + F + j] = __float2half(ratio * static_cast<float>(std::cos(yc * om[j])));
      }
    }
  }
  return out;
}

bool is_global(const Config& c, int i) { return c.alt_start >= 0 && i >= c.alt_start && (i % 2 == 1); }

}  // namespace

// ------------------------------------------------------------------ plan creation
Plan* Engine::plan_for(int V, int S, int H, int W, bool rays) {
  auto key = std::make_tuple(V, S, H, W, rays);
  auto it = plans_.find(key);
  if (it != plans_.end()) return it->second.get();
  const Config& c = model_->cfg;
  const Head& hd = model_->head;
  const int P = c.patch_size, D = c.embed_dim;
  std::unique_ptr<Plan> p(new Plan());
  p->V = V;
  p->S = S;
  p->scenes = V / S;
  p->H = H;
  p->W = W;
  p->gh = H / P;
  p->gw = W / P;
  p->Np = p->gh * p->gw;
  p->Ntok = 1 + p->Np;
  p->M = V * p->Ntok;
  p->rays = rays && hd.aux;
  {
    const char* u = getenv("DA3B_UNFUSED_UP");
    const int Fh = (c.head_features > 0 ? c.head_features : hd.rn[0].OC) / 2;
    p->fused_up = !(u && u[0] == '1') && Fh >= 16 && Fh <= 128 && (Fh & (Fh - 1)) == 0;
  }
  p->ho3 = (p->gh + 2 - 3) / 2 + 1;
  p->wo3 = (p->gw + 2 - 3) / 2 + 1;
  p->Cf = (c.cat_token ? 2 : 1) * D;
  const int F = c.head_features > 0 ? c.head_features : hd.rn[0].OC;
  const int* oc = nullptr;
  int ocv[4];
  for (int s = 0; s < 4; ++s) ocv[s] = hd.proj[s].N;
  oc = ocv;
  const size_t V_ = static_cast<size_t>(V), M_ = static_cast<size_t>(p->M), Np = static_cast<size_t>(p->Np);
  const int gh = p->gh, gw = p->gw;
  // ---- size the arena (two passes: count, then carve)
  auto carve = [&](Arena& a) -> bool {
    bool ok = true;
    auto T = [&](auto*& dst, size_t count) {
      using E = std::remove_reference_t<decltype(*dst)>;
      dst = a.template take<E>(count);
      if (!dst && a.base) ok = false;
    };
    T(p->rgb, V_ * H * W * 3);
    T(p->depth, V_ * H * W);
    T(p->conf, V_ * H * W);
    if (p->rays) T(p->raysbuf, static_cast<size_t>(hd.aux_od) * V_ * (8 * gh) * (8 * gw));
    if (hd.sky) T(p->sky, V_ * H * W);
    T(p->x, M_ * D);
    if (S >= 3 && c.alt_start >= 0) T(p->x2, M_ * D);
    T(p->pos, static_cast<size_t>(p->Ntok) * D);
    T(p->rl_cos, static_cast<size_t>(p->Ntok) * 64);
    T(p->rl_sin, static_cast<size_t>(p->Ntok) * 64);
    T(p->rn_cos, static_cast<size_t>(p->Ntok) * 64);
    T(p->rn_sin, static_cast<size_t>(p->Ntok) * 64);
    T(p->patchA, V_ * Np * model_->patch_ldk);
    T(p->xn, M_ * D);
    T(p->qkv, M_ * 3 * D);
    p->ld_vt_local = (p->Ntok + 7) / 8 * 8;
    p->ld_vt_global = (S * p->Ntok + 7) / 8 * 8;
    T(p->vt, std::max(V_ * D * p->ld_vt_local, static_cast<size_t>(p->scenes) * D * p->ld_vt_global));
    T(p->attn, M_ * D);
    T(p->hid, M_ * c.mlp_hidden);
    for (int o = 0; o < 4; ++o) T(p->feats[o], V_ * Np * p->Cf);
    if (S >= 3 && c.alt_start >= 0)
      for (int o = 0; o < 4; ++o) T(p->ftmp[o], V_ * Np * p->Cf);
    if (hd.norm_g)
      for (int o = 0; o < 4; ++o) T(p->featn[o], V_ * Np * p->Cf);
    T(p->b_idx, static_cast<size_t>(std::max(1, p->scenes)));
    if (capture_resid_) T(p->resid_cap, static_cast<size_t>(c.depth) * M_ * D);
    if (model_->camdec.present) {
      T(p->cam, V_ * p->Cf);
      T(p->cam_h1, V_ * model_->camdec.bb0.N);
      T(p->cam_h2, V_ * model_->camdec.bb2.N);
      T(p->cam_pe, V_ * 9);
    }
    for (int s = 0; s < 4; ++s) T(p->P[s], V_ * Np * oc[s]);
    T(p->L0, V_ * (4 * gh) * (4 * gw) * oc[0]);
    T(p->L1, V_ * (2 * gh) * (2 * gw) * oc[1]);
    T(p->A3, V_ * p->ho3 * p->wo3 * 9 * conv_icp(oc[3]));
    T(p->L3, V_ * p->ho3 * p->wo3 * oc[3]);
    const int lh[4] = {4 * gh, 2 * gh, gh, p->ho3}, lw[4] = {4 * gw, 2 * gw, gw, p->wo3};
    for (int s = 0; s < 4; ++s) {
      T(p->RN[s], V_ * lh[s] * lw[s] * F);
      T(p->RNr[s], V_ * lh[s] * lw[s] * F);
      Level& L = p->lv[s];
      L.h = lh[s];
      L.w = lw[s];
      const size_t n = V_ * lh[s] * lw[s] * F;
      T(L.T, n);
      T(L.Y1, n);
      T(L.Y1r, n);
      T(L.Y2, n);
      T(L.Z, n);
    }
    T(p->U[0], V_ * gh * gw * F);                  // refinenet4 -> lv2
    T(p->U[1], V_ * (2 * gh) * (2 * gw) * F);      // refinenet3 -> lv1
    T(p->U[2], V_ * (4 * gh) * (4 * gw) * F);      // refinenet2 -> lv0
    T(p->U[3], V_ * (8 * gh) * (8 * gw) * F);      // refinenet1 -> 8gh
    T(p->O1, V_ * (8 * gh) * (8 * gw) * (F / 2));
    if (!p->fused_up) T(p->O1u, V_ * H * W * (F / 2));
    if (p->rays) {
      T(p->auxA, V_ * (8 * gh) * (8 * gw) * F);
      T(p->auxB, V_ * (8 * gh) * (8 * gw) * F);
    }
    if (c.head_pos_embed) {
      for (int s = 0; s < 4; ++s) T(p->pe_proj[s], Np * oc[s]);
      T(p->pe_full, static_cast<size_t>(H) * W * (F / 2));
      if (p->rays) T(p->pe_aux, static_cast<size_t>(8 * gh) * (8 * gw) * (F / 2));
    }
    return ok;
  };
  Arena count;  // sizing pass (base == nullptr)
  carve(count);
  const size_t bytes = count.used;
  if (cudaMalloc(&p->arena.base, bytes) != cudaSuccess) {
    err_ = "out of device memory for a plan of " + std::to_string(bytes >> 20) + " MiB";
    return nullptr;
  }
  p->arena.size = bytes;
  p->arena.used = 0;
  if (!carve(p->arena)) {
    err_ = "plan arena overflow";
    return nullptr;
  }
  // padded im2col columns must read as zero
  cudaMemset(p->A3, 0, V_ * p->ho3 * p->wo3 * 9 * conv_icp(oc[3]) * sizeof(__half));
  // ---- tables
  {
    std::vector<float> pos = interp_pos(model_->pos_embed_host(), D, c.pos_embed_grid, gh, gw, c.interp_offset);
    cudaMemcpy(p->pos, pos.data(), pos.size() * 4, cudaMemcpyHostToDevice);
    std::vector<float> pl(2 * p->Ntok, 0.f), pn(2 * p->Ntok, 0.f);
    for (int t = 1; t < p->Ntok; ++t) {  // (src/dino_backbone.cpp:92-95)
      const int idx = t - 1;
      pl[2 * t] = static_cast<float>(idx / gw + 1);
      pl[2 * t + 1] = static_cast<float>(idx % gw + 1);
      pn[2 * t] = pn[2 * t + 1] = 1.f;
    }
    std::vector<float> cs, sn;
    rope_tables(pl, p->Ntok, c.rope_freq, cs, sn);
    cudaMemcpy(p->rl_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(p->rl_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    rope_tables(pn, p->Ntok, c.rope_freq, cs, sn);
    cudaMemcpy(p->rn_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(p->rn_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice);
    if (c.head_pos_embed) {
      const float aspect = static_cast<float>(W) / static_cast<float>(H);
      for (int s = 0; s < 4; ++s) {
        auto t = uv_table(gw, gh, oc[s], aspect, 0.1f);
        cudaMemcpy(p->pe_proj[s], t.data(), t.size() * 2, cudaMemcpyHostToDevice);
      }
      auto t = uv_table(W, H, F / 2, aspect, 0.1f);
      cudaMemcpy(p->pe_full, t.data(), t.size() * 2, cudaMemcpyHostToDevice);
      if (p->rays) {
        auto ta = uv_table(8 * gw, 8 * gh, F / 2, aspect, 0.1f);
        cudaMemcpy(p->pe_aux, ta.data(), ta.size() * 2, cudaMemcpyHostToDevice);
      }
    }
  }
  if (cudaDeviceSynchronize() != cudaSuccess) {
    err_ = "device error while building a plan";
    return nullptr;
  }
  Plan* raw = p.get();
  plans_[key] = std::move(p);
  return raw;
}

// ------------------------------------------------------------------ forward
#define CK(call)                                                             \
  do {                                                                       \
    const int rc_ = (call);                                                  \
    ++p.launches;                                                            \
    if (rc_ != 0) {                                                          \
      err_ = std::string("launch failed (") + #call + ") rc=" + std::to_string(rc_); \
      return rc_ < 0 ? rc_ : -rc_;                                           \
    }                                                                        \
  } while (0)

static EpiArgs epi_f16(__half* out, int ld, const float* bias, int act) {
  EpiArgs e = epi_default();
  e.kind = kEpiF16;
  e.out = out;
  e.ld_out = ld;
  e.bias = bias;
  e.act = act;
  return e;
}

int Engine::backbone(Plan& p, cudaStream_t s) {
  const DeviceModel& m = *model_;
  const Config& c = m.cfg;
  const int D = c.embed_dim, Hh = c.num_heads, Np = p.Np, Nt = p.Ntok, V = p.V, M = p.M;
  const bool select = p.S >= 3 && c.alt_start >= 0;
  float* mean = const_cast<float*>(c.img_mean.data());
  float* sd = const_cast<float*>(c.img_std.data());
  // ---- tokens: patchify -> patch-embed GEMM (+bias +pos into rows 1..Np) ; CLS row
  if (p.prepared) CK(patchify_chw(p.chw, V, p.H, p.W, c.patch_size, p.patchA, m.patch_ldk, s));
  else CK(patchify(p.rgb, V, p.H, p.W, c.patch_size, mean, sd, p.patchA, m.patch_ldk, s));
  {
    EpiArgs e = epi_default();
    e.kind = kEpiTokens;
    e.resid = p.x;
    e.ld_resid = D;
    e.bias = m.patch.b;
    e.pos = p.pos;
    e.rm_div = Np;
    e.rm_mul = Nt;
    e.rm_add = 1;
    CK(gemm_linear(p.patchA, V * Np, m.patch_k, m.patch_ldk, m.patch.w, D, m.patch.ldw, 0, e, status_, s));
  }
  CK(cls_rows(p.x, V, Nt, D, m.cls, p.pos, s));

  // local_x bookkeeping (src/dino_backbone.cpp:143-161): after local block j, x is the
  // local_x of every out-layer L >= j whose blocks in (j, L] are all global.
  auto write_local = [&](int j) -> int {
    if (!c.cat_token) return 0;
    for (int o = 0; o < 4; ++o) {
      const int L = c.out_layers[o];
      if (L < j) continue;
      bool all_global = true;
      for (int i = j + 1; i <= L; ++i)
        if (!is_global(c, i)) all_global = false;
      if (all_global) {
        CK(cast_rows(p.x, D, V * Np, D, p.feats[o], p.Cf, 0, Np, Nt, 1, s));
        if (o == 3 && p.cam) CK(copy_token0(p.x, V, Nt, D, p.cam, p.Cf, 0, s));  // local half of the camera token
      }
    }
    return 0;
  };
  if (int rc = write_local(-1)) return rc;

  for (int i = 0; i < c.depth; ++i) {
    const Block& b = m.blk[i];
    // this block's linears: the resident f16 planes; or, resident as planar Q8_0,
    // dequantised into the staging buffer by the LN1 launch (in stream order after the
    // previous block's last GEMM) for the f16 GEMMs (default), or ($DA3B_Q8_TILES=1, few rows: every
    // linear on one-CTA tiles) read by GEMMs that dequantise their weight tiles in
    // shared memory. The two give the same bits; the staging route is the faster at
    // one image (ViT-B: QKV 12.6 + 2.2 us against 18.1 us, fc1 14.6 + 2.7 against 20.3).
    const __half *w_qkv = b.qkv.w, *w_proj = b.proj.w, *w_fc1 = b.fc1.w, *w_fc2 = b.fc2.w;
    const bool q8_tiles = m.q8_resident && q8_tiles_ && gemm_q8p_bn(M, b.qkv.N, b.qkv.K) &&
                          gemm_q8p_bn(M, b.proj.N, b.proj.K) && gemm_q8p_bn(M, b.fc1.N, b.fc1.K) &&
                          gemm_q8p_bn(M, b.fc2.N, b.fc2.K);
    auto linear = [&](const __half* A, int lda, const Lin& L, const __half* w_f16, const EpiArgs& e) -> int {
      if (q8_tiles) return gemm_linear_q8p(A, M, L.K, lda, L.q8, L.N, e, status_, s);
      return gemm_linear(A, M, L.K, lda, w_f16, L.N, L.ldw, 0, e, status_, s);
    };
    Q8Segs g;
    memset(&g, 0, sizeof(g));
    if (m.q8_resident && !q8_tiles) {
      const Lin* L4[4] = {&b.qkv, &b.proj, &b.fc1, &b.fc2};
      const __half** ptrs[4] = {&w_qkv, &w_proj, &w_fc1, &w_fc2};
      __half* dst = wstage_;
      long first = 0;
      for (int k = 0; k < 4; ++k) {
        g.s[k] = Q8Seg{L4[k]->q8, dst, L4[k]->N, L4[k]->K / 32, first};
        *ptrs[k] = dst;
        first += static_cast<long>(L4[k]->N) * (L4[k]->K / 32);
        dst += static_cast<size_t>(L4[k]->N) * L4[k]->K;
      }
      g.n = 4;
      g.total = first;
    }
    if (select && i == c.alt_start - 1) {
      // reference-view selection on the views' token 0 after blocks [0, alt_start-1)
      // (pass A, src/dino_backbone.cpp:427-441); the local blocks before are per view,
      // so the pass-B recomputation reduces to permuting the views in place.
      CK(select_ref_view(p.x, p.scenes, p.S, Nt, D, p.b_idx, s));
      CK(permute_views(p.x, p.x2, p.scenes, p.S, static_cast<long>(Nt) * D, p.b_idx, s));
      std::swap(p.x, p.x2);
    }
    if (c.alt_start >= 0 && i == c.alt_start && m.cam) CK(cam_rows(p.x, V, p.S, Nt, D, m.cam, s));
    const bool global = is_global(c, i);
    const bool use_rope = c.rope_start >= 0 && i >= c.rope_start;
    // ---- attention half
    const int q8 = act_quant_ ? 1 : 0;
    // LN1, with this block's staging dequantisation in the same launch
    CK(layernorm_f32(p.x, D, M, D, b.n1g, b.n1b, c.ln_eps, p.xn, D, 0, 0, 0, 0, s, q8, g.n ? &g : nullptr));
    const int seqlen = global ? p.S * Nt : Nt, nseq = global ? p.scenes : V;
    const int ld_vt = global ? p.ld_vt_global : p.ld_vt_local;
    {
      EpiArgs e = epi_f16(p.qkv, 3 * D, b.qkv.b, kActNone);
      e.kind = kEpiQKV;
      e.vt = p.vt;
      e.vt_seqlen = seqlen;
      e.vt_ld = ld_vt;
      e.vt_d = D;
      CK(linear(p.xn, D, b.qkv, w_qkv, e));
    }
    if (b.qng || use_rope) {
      const float* cs = use_rope ? (global ? p.rn_cos : p.rl_cos) : nullptr;
      const float* sn = use_rope ? (global ? p.rn_sin : p.rl_sin) : nullptr;
      CK(qk_norm_rope(p.qkv, M, Hh, D, Nt, b.qng, b.qnb, b.kng, b.knb, cs, sn, s));
    }
    CK(attention_tc(p.qkv, p.vt, ld_vt, nseq, seqlen, Hh, D, p.attn, q8, status_, s));
    {
      EpiArgs e = epi_default();
      e.kind = kEpiResid;
      e.resid = p.x;
      e.ld_resid = D;
      e.bias = b.proj.b;
      e.scale = b.ls1;
      CK(linear(p.attn, D, b.proj, w_proj, e));
    }
    // ---- MLP half
    CK(layernorm_f32(p.x, D, M, D, b.n2g, b.n2b, c.ln_eps, p.xn, D, 0, 0, 0, 0, s, q8));
    {
      EpiArgs e = epi_f16(p.hid, b.fc1.N, b.fc1.b, kActGelu);
      e.q8 = q8;
      CK(linear(p.xn, D, b.fc1, w_fc1, e));
    }
    {
      EpiArgs e = epi_default();
      e.kind = kEpiResid;
      e.resid = p.x;
      e.ld_resid = D;
      e.bias = b.fc2.b;
      e.scale = b.ls2;
      CK(linear(p.hid, b.fc2.K, b.fc2, w_fc2, e));
    }
    if (p.resid_cap &&
        cudaMemcpyAsync(p.resid_cap + static_cast<size_t>(i) * M * D, p.x, static_cast<size_t>(M) * D * sizeof(float),
                        cudaMemcpyDeviceToDevice, s) != cudaSuccess) {
      err_ = "residual capture copy failed";
      return -30;
    }
    if (!global)
      if (int rc = write_local(i)) return rc;
    for (int o = 0; o < 4; ++o) {
      if (c.out_layers[o] != i) continue;
      // DA2: LN(x) (host double LN in the reference, src/dino_backbone.cpp:183-196);
      // DA3: cat[local_x, LN(x)] (src/dino_backbone.cpp:296-306). Token 0 dropped.
      CK(layernorm_f32(p.x, D, V * Np, D, m.norm_g, m.norm_b, c.ln_eps, p.feats[o], p.Cf, c.cat_token ? D : 0, Np, Nt,
                       1, s));
      if (o == 3 && p.cam) CK(copy_token0(p.x, V, Nt, D, p.cam, p.Cf, c.cat_token ? D : 0, s));  // raw x half
    }
  }
  if (select) {
    for (int o = 0; o < 4; ++o) {
      CK(unpermute_views_h(p.feats[o], p.ftmp[o], p.scenes, p.S, static_cast<long>(Np) * p.Cf, p.b_idx, s));
      std::swap(p.feats[o], p.ftmp[o]);  // swapped back at the end of the forward
    }
  }
  return 0;
}

// One fusion pyramid (refinenet4 .. refinenet1) over the layer_rn maps; writes the
// x2-upsampled refinenet1 output into u_out (8gh x 8gw). lateral_ready (or null): per
// level r < 3 an event after which RN[r] / RNr[r] and the first conv of the level's RCU1
// (into lv[r].T) are done on another stream; the pyramid then waits for it before level
// r and skips that conv.
int Engine::pyramid(Plan& p, const void* fw, __half* u_out, cudaStream_t s, const cudaEvent_t* lateral_ready) {
  const Fusion* fu = static_cast<const Fusion*>(fw);
  const int V = p.V;
  const int F = fu[0].rc2c1.OC;
  // level index: 3 = refinenet4 (stride-2 grid), 2, 1, 0 = refinenet1
  const __half* top = nullptr;
  for (int r = 3; r >= 0; --r) {
    Level& L = p.lv[r];
    const Fusion& f = fu[r];
    const int hh = L.h, ww = L.w;
    const __half* y = nullptr;
    if (r == 3) {
      y = p.RN[3];
    } else {
      // y1 = top + RCU1(lateral): relu -> conv1 -> relu -> conv2 + lateral (+ top)
      if (lateral_ready) {
        if (cudaStreamWaitEvent(s, lateral_ready[r], 0) != cudaSuccess) {
          err_ = "stream wait failed";
          return -51;
        }
      } else {
        EpiArgs e1 = epi_f16(L.T, F, f.rc1c1.b, kActRelu);
        CK(conv_nhwc(p.RNr[r], V, hh, ww, f.rc1c1.IC, f.rc1c1.w, F, 3, 0, e1, status_, s));
      }
      EpiArgs e2 = epi_f16(L.Y1, F, f.rc1c2.b, kActNone);
      e2.res1 = p.RN[r];
      e2.ld_res1 = F;
      e2.res2 = top;
      e2.ld_res2 = F;
      e2.out_relu = L.Y1r;
      CK(conv_nhwc(L.T, V, hh, ww, F, f.rc1c2.w, F, 3, 0, e2, status_, s));
      y = L.Y1;
    }
    // RCU2: relu(y) -> conv1 -> relu -> conv2 + y
    const __half* yr = (r == 3) ? p.RNr[3] : L.Y1r;
    EpiArgs e3 = epi_f16(L.T, F, f.rc2c1.b, kActRelu);
    CK(conv_nhwc(yr, V, hh, ww, F, f.rc2c1.w, F, 3, 0, e3, status_, s));
    EpiArgs e4 = epi_f16(L.Y2, F, f.rc2c2.b, kActNone);
    e4.res1 = y;
    e4.ld_res1 = F;
    CK(conv_nhwc(L.T, V, hh, ww, F, f.rc2c2.w, F, 3, 0, e4, status_, s));
    // out 1x1 conv at the low resolution, then the align-corners resize: the two
    // commute (bilinear weights sum to one), so the conv runs on 4x fewer pixels.
    CK(gemm_linear(L.Y2, V * hh * ww, F, F, f.out.w, F, f.out.ldw, 0, epi_f16(L.Z, F, f.out.b, kActNone), status_, s));
    int th, tw;
    __half* dst;
    if (r == 3) { th = p.gh; tw = p.gw; dst = p.U[0]; }
    else if (r == 2) { th = 2 * p.gh; tw = 2 * p.gw; dst = p.U[1]; }
    else if (r == 1) { th = 4 * p.gh; tw = 4 * p.gw; dst = p.U[2]; }
    else { th = 2 * hh; tw = 2 * ww; dst = u_out; }
    CK(upsample_ac(L.Z, V, hh, ww, F, dst, th, tw, nullptr, s));
    top = dst;
  }
  return 0;
}

int Engine::head(Plan& p, cudaStream_t s) {
  const DeviceModel& m = *model_;
  const Config& c = m.cfg;
  const Head& h = m.head;
  const int V = p.V, Np = p.Np, gh = p.gh, gw = p.gw, Cf = p.Cf;
  const int F = h.rn[0].OC;
  // ---- head LayerNorm (DA3, eps 1e-5, src/dpt_head.cpp:91-103) over the feature channels
  const __half* fin[4] = {p.feats[0], p.feats[1], p.feats[2], p.feats[3]};
  if (h.norm_g)
    for (int o = 0; o < 4; ++o) {
      CK(layernorm_f16(p.feats[o], Cf, V * Np, Cf, h.norm_g, h.norm_b, 1e-5f, p.featn[o], Cf, 0, 0, 0, 0, s));
      fin[o] = p.featn[o];
    }
  // ---- the four lateral branches: projection (+0.1 UV PE) -> resize -> layer_rn (raw +
  // relu copies) and, for levels 0-2, the first conv of the level's RCU1. They depend on
  // nothing but the features, and only refinenet4 (level 3) needs its branch before the
  // fusion chain starts, so branches 0-2 run on side streams (forked and joined by
  // events, which a graph capture turns into parallel branches) while branch 3 and
  // then the chain run on s; the chain waits for branch r just before level r. At one
  // image these launches fill 6-148 of the SMs each.
  const Fusion* fu = h.fu;
  auto branch = [&](int st, cudaStream_t bs) -> int {
    {
      const Lin& L = h.proj[st];
      EpiArgs e = epi_f16(p.P[st], L.N, L.b, kActNone);
      if (c.head_pos_embed) {
        e.res1 = p.pe_proj[st];
        e.ld_res1 = L.N;
        e.res1_mod = Np;
      }
      CK(gemm_linear(fin[st], V * Np, Cf, Cf, L.w, L.N, L.ldw, 0, e, status_, bs));
    }
    if (st == 0 || st == 1) {
      const ConvT& rs = st == 0 ? h.rs0 : h.rs1;
      const int sc = st == 0 ? 4 : 2;
      EpiArgs e = epi_f16(st == 0 ? p.L0 : p.L1, rs.OC, rs.b, kActNone);
      e.kind = kEpiConvT;
      e.ct_hin = gh;
      e.ct_win = gw;
      e.ct_s = sc;
      e.ct_oc = rs.OC;
      CK(gemm_linear(p.P[st], V * Np, rs.IC, rs.IC, rs.w, sc * sc * rs.OC, rs.IC, 0, e, status_, bs));
    } else if (st == 3) {
      const int icp3 = conv_icp(h.rs3.IC);
      CK(im2col_s2(p.P[3], V, gh, gw, h.rs3.IC, icp3, p.A3, bs));
      CK(gemm_linear(p.A3, V * p.ho3 * p.wo3, 9 * icp3, 9 * icp3, h.rs3.w, h.rs3.OC, 9 * icp3, 0,
                     epi_f16(p.L3, h.rs3.OC, h.rs3.b, kActNone), status_, bs));
    }
    const __half* Ls[4] = {p.L0, p.L1, p.P[2], p.L3};
    {
      EpiArgs e = epi_f16(p.RN[st], F, nullptr, kActNone);
      e.out_relu = p.RNr[st];
      CK(conv_nhwc(Ls[st], V, p.lv[st].h, p.lv[st].w, h.rn[st].IC, h.rn[st].w, F, 3, 0, e, status_, bs));
    }
    if (st < 3) {
      const Fusion& f = fu[st];
      EpiArgs e1 = epi_f16(p.lv[st].T, F, f.rc1c1.b, kActRelu);
      CK(conv_nhwc(p.RNr[st], V, p.lv[st].h, p.lv[st].w, f.rc1c1.IC, f.rc1c1.w, F, 3, 0, e1, status_, bs));
    }
    return 0;
  };
  if (cudaEventRecord(ev_[0], s) != cudaSuccess) {
    err_ = "event record failed";
    return -52;
  }
  for (int st = 0; st < 3; ++st) {
    if (cudaStreamWaitEvent(side_[st], ev_[0], 0) != cudaSuccess) {
      err_ = "stream wait failed";
      return -52;
    }
    if (int rc = branch(st, side_[st])) return rc;
    if (cudaEventRecord(ev_[1 + st], side_[st]) != cudaSuccess) {
      err_ = "event record failed";
      return -52;
    }
  }
  if (int rc = branch(3, s)) return rc;
  // ---- main fusion pyramid -> out1 -> upsample(+PE) -> out2a + out2b + activation
  if (int rc = pyramid(p, h.fu, p.U[3], s, ev_ + 1)) return rc;
  const int h8 = 8 * gh, w8 = 8 * gw;
  CK(conv_nhwc(p.U[3], V, h8, w8, F, h.out1.w, h.out1.OC, 3, 0, epi_f16(p.O1, h.out1.OC, h.out1.b, kActNone), status_,
               s));
  const __half* pe_full = c.head_pos_embed ? p.pe_full : nullptr;
  if (!p.fused_up) CK(upsample_ac(p.O1, V, h8, w8, h.out1.OC, p.O1u, p.H, p.W, pe_full, s));
  // output_conv2: 3x3 -> 32, relu, 1x1 -> output_dim, activation, on the upsampled map
  auto out2 = [&](const Conv& cv, const EpiArgs& e) -> int {
    if (p.fused_up) return up_out2(p.O1, V, h8, w8, h.out1.OC, pe_full, p.H, p.W, cv.w, conv_icp(cv.IC), e, status_, s);
    return conv_nhwc(p.O1u, V, p.H, p.W, cv.IC, cv.w, 32, 3, 32, e, status_, s);
  };
  {
    EpiArgs e = epi_default();
    e.kind = kEpiOut2;
    e.bias = h.out2a.b;
    e.o2_w = h.out2b_w;
    e.o2_b = h.out2b_b;
    e.o2_dim = h.od;
    const HeadKind k = head_kind();
    for (int i = 0; i < h.od; ++i) {
      if (raw_logits_) e.o2_act[i] = kOutIdentity;
      else if (k == HeadKind::Da2Relative) e.o2_act[i] = kOutRelu;
      else if (k == HeadKind::Da2Metric) e.o2_act[i] = kOutSigmoidScale;
      else e.o2_act[i] = (i == 0) ? kOutExp : kOutExpP1;
      e.o2_out[i] = (i == 0) ? p.depth : p.conf;
    }
    if (h.od > 2) {
      err_ = "more than two main-head output channels";
      return -50;
    }
    e.o2_scale = c.head_max_depth;
    CK(out2(h.out2a, e));
  }
  // ---- sky head (metric / mono DPT, src/dpt_head.cpp:205-222 and the relu at
  // src/dpt_head.cpp:334-338) on the same upsampled feature map
  if (h.sky) {
    EpiArgs e = epi_default();
    e.kind = kEpiOut2;
    e.bias = h.sky_out2a.b;
    e.o2_w = h.sky_out2b_w;
    e.o2_b = h.sky_out2b_b;
    e.o2_dim = 1;
    e.o2_act[0] = raw_logits_ ? kOutIdentity : kOutRelu;
    e.o2_out[0] = p.sky;
    CK(out2(h.sky_out2a, e));
  }
  // ---- aux ray head (DualDPT, src/dpt_head.cpp:225-272)
  if (p.rays) {
    if (int rc = pyramid(p, h.fa, p.auxA, s, nullptr)) return rc;
    __half* a = p.auxA;
    __half* b = p.auxB;
    for (int i = 0; i < 5; ++i) {
      const Conv& cv = h.out1_aux[i];
      EpiArgs e = epi_f16(b, cv.OC, cv.b, kActNone);
      if (i == 4 && c.head_pos_embed) {
        e.res1 = p.pe_aux;
        e.ld_res1 = cv.OC;
        e.res1_mod = h8 * w8;
      }
      CK(conv_nhwc(a, V, h8, w8, cv.IC, cv.w, cv.OC, 3, 0, e, status_, s));
      std::swap(a, b);
    }
    EpiArgs e = epi_default();
    e.kind = kEpiOut2;
    e.bias = h.out2a_aux.b;
    e.o2_w = h.out2b_aux_w;
    e.o2_b = h.out2b_aux_b;
    e.o2_dim = h.aux_od;
    e.o2_ln_g = h.aux_ln_g;
    e.o2_ln_b = h.aux_ln_b;
    e.o2_ln_eps = 1e-5f;
    const size_t plane = static_cast<size_t>(V) * h8 * w8;
    for (int i = 0; i < h.aux_od; ++i) {
      e.o2_act[i] = (i == h.aux_od - 1 && !raw_logits_) ? kOutExpP1 : kOutIdentity;
      e.o2_out[i] = p.raysbuf + i * plane;
    }
    CK(conv_nhwc(a, V, h8, w8, h.out2a_aux.IC, h.out2a_aux.w, 32, 3, 32, e, status_, s));
  }
  return 0;
}

int Engine::forward(Plan& p, cudaStream_t s) {
  p.launches = 0;
  // Buffers swapped by the view permutation are swapped back afterwards so every
  // forward (and the captured graph) of a plan addresses the same buffers.
  float* x0 = p.x;
  __half* f0[4] = {p.feats[0], p.feats[1], p.feats[2], p.feats[3]};
  __half* t0[4] = {p.ftmp[0], p.ftmp[1], p.ftmp[2], p.ftmp[3]};
  int rc = backbone(p, s);
  if (!rc) rc = head(p, s);
  last_x_ = p.x;
  for (int o = 0; o < 4; ++o) last_feat_[o] = p.feats[o];
  if (p.x != x0) std::swap(p.x, p.x2);
  for (int o = 0; o < 4; ++o) {
    p.feats[o] = f0[o];
    p.ftmp[o] = t0[o];
  }
  return rc;
}

int Engine::run(const uint8_t* rgb, int V, int S, int H, int W, float* depth, float* conf, float* rays,
                cudaStream_t s) {
  int code = 0;
  Plan* p = checked_plan(V, S, H, W, rays != nullptr, &code);
  if (!p) return code;
  const size_t HW = static_cast<size_t>(H) * W;
  if (cudaMemcpyAsync(p->rgb, rgb, static_cast<size_t>(V) * HW * 3, cudaMemcpyDefault, s) != cudaSuccess) {
    err_ = "input copy failed";
    return -5;
  }
  const int rc = launch(p, false, s);
  return rc ? rc : copy_out(p, depth, conf, rays, s);
}

int Engine::run_with_rays(const uint8_t* rgb, int V, int S, int H, int W, float* depth, float* conf, cudaStream_t s) {
  if (!model_->head.aux) {
    err_ = "this GGUF has no auxiliary ray head";
    return -70;
  }
  int code = 0;
  Plan* p = checked_plan(V, S, H, W, true, &code);
  if (!p) return code;
  const size_t HW = static_cast<size_t>(H) * W;
  if (cudaMemcpyAsync(p->rgb, rgb, static_cast<size_t>(V) * HW * 3, cudaMemcpyDefault, s) != cudaSuccess) {
    err_ = "input copy failed";
    return -5;
  }
  const int rc = launch(p, false, s);
  return rc ? rc : copy_out(p, depth, conf, nullptr, s);
}

const float* Engine::last_rays(int* n_views, int* ray_h, int* ray_w) const {
  if (!last_ || !last_->rays || !last_->raysbuf) return nullptr;
  if (n_views) *n_views = last_->V;
  if (ray_h) *ray_h = 8 * last_->gh;
  if (ray_w) *ray_w = 8 * last_->gw;
  return last_->raysbuf;
}

Plan* Engine::checked_plan(int V, int S, int H, int W, bool rays, int* code) {
  const Config& c = model_->cfg;
  if (V <= 0 || S <= 0 || V % S || H <= 0 || W <= 0 || H % c.patch_size || W % c.patch_size) {
    err_ = "bad shape: n_views must be a positive multiple of views_per_scene and H, W multiples of the patch size";
    if (code) *code = -2;
    return nullptr;
  }
  if (rays && !model_->head.aux) {
    err_ = "this GGUF has no auxiliary ray head";
    if (code) *code = -3;
    return nullptr;
  }
  cudaSetDevice(device_);
  Plan* p = plan_for(V, S, H, W, rays);
  if (!p) {
    if (code) *code = -4;
    return nullptr;
  }
  last_ = p;
  return p;
}

float* Engine::prepared_input(int V, int S, int H, int W, size_t* bytes) {
  Plan* p = checked_plan(V, S, H, W, false, nullptr);
  if (!p) return nullptr;
  const size_t n = static_cast<size_t>(V) * 3 * H * W;
  if (!p->chw && cudaMalloc(&p->chw, n * sizeof(float)) != cudaSuccess) {
    p->chw = nullptr;
    err_ = "out of device memory for the prepared input";
    return nullptr;
  }
  if (bytes) *bytes = n * sizeof(float);
  return p->chw;
}

int Engine::run_prepared(int V, int S, int H, int W, float* depth, float* conf, cudaStream_t s) {
  if (!prepared_input(V, S, H, W, nullptr)) return -4;
  Plan* p = last_;
  const int rc = launch(p, true, s);
  return rc ? rc : copy_out(p, depth, conf, nullptr, s);
}

// One forward of a plan: eager on its first run (plan warm-up), then replays of the
// graph captured for this input mode.
int Engine::launch(Plan* p, bool prepared, cudaStream_t s) {
  p->prepared = prepared;
  bool& warmed = prepared ? p->warmed_pre : p->warmed;
  cudaGraphExec_t& graph = prepared ? p->graph_pre : p->graph;
  if (!use_graph_ || !warmed) {
    const int rc = forward(*p, s);
    if (rc) return rc;
    warmed = true;
    return 0;
  }
  if (!graph) {
    cudaStream_t cs;
    cudaStreamCreateWithFlags(&cs, cudaStreamNonBlocking);
    cudaGraph_t g = nullptr;
    int rc = 0;
    if (cudaStreamBeginCapture(cs, cudaStreamCaptureModeThreadLocal) != cudaSuccess) rc = -6;
    if (!rc) rc = forward(*p, cs);
    if (cudaStreamEndCapture(cs, &g) != cudaSuccess && !rc) rc = -7;
    if (!rc && cudaGraphInstantiate(&graph, g, 0) != cudaSuccess) rc = -8;
    if (g) cudaGraphDestroy(g);
    cudaStreamDestroy(cs);
    if (rc) {
      if (err_.empty()) err_ = "CUDA graph capture failed";
      graph = nullptr;
      return rc;
    }
  }
  if (cudaGraphLaunch(graph, s) != cudaSuccess) {
    err_ = "graph launch failed";
    return -9;
  }
  return 0;
}

int Engine::copy_out(Plan* p, float* depth, float* conf, float* rays, cudaStream_t s) {
  const size_t HW = static_cast<size_t>(p->H) * p->W;
  const int V = p->V;
  if (depth && cudaMemcpyAsync(depth, p->depth, static_cast<size_t>(V) * HW * 4, cudaMemcpyDefault, s) != cudaSuccess)
    return -10;
  if (conf && model_->head.od >= 2 &&
      cudaMemcpyAsync(conf, p->conf, static_cast<size_t>(V) * HW * 4, cudaMemcpyDefault, s) != cudaSuccess)
    return -11;
  if (rays) {
    const size_t n = static_cast<size_t>(model_->head.aux_od) * V * (8 * p->gh) * (8 * p->gw);
    if (cudaMemcpyAsync(rays, p->raysbuf, n * 4, cudaMemcpyDefault, s) != cudaSuccess) return -12;
  }
  return 0;
}

// Camera decoder on the camera tokens of the last run (CamPose::pose,
// src/cam_pose.cpp:20-38): pose encodings [V][9], in the original view order.
int Engine::sky(float* dst, size_t count, cudaStream_t s) {
  if (!model_->head.sky) {
    err_ = "this GGUF has no sky head (head.scratch.sky_out2*)";
    return -60;
  }
  if (!last_) {
    err_ = "no forward has run yet";
    return -61;
  }
  const size_t n = static_cast<size_t>(last_->V) * last_->H * last_->W;
  if (count != n) {
    err_ = "the last run produced " + std::to_string(n) + " sky values, not " + std::to_string(count);
    return -63;
  }
  if (cudaMemcpyAsync(dst, last_->sky, n * 4, cudaMemcpyDefault, s) != cudaSuccess) {
    err_ = "sky copy failed";
    return -62;
  }
  return 0;
}

int Engine::poses(std::vector<float>& pe, cudaStream_t s) {
  const CamDec& cd = model_->camdec;
  if (!cd.present) {
    err_ = "this GGUF has no camera decoder (cam.*)";
    return -1;
  }
  if (!last_ || !last_->cam) {
    err_ = "no run to take camera tokens from";
    return -2;
  }
  Plan& p = *last_;
  const int V = p.V;
  if (cd.bb0.K != p.Cf) {
    err_ = "camera decoder input width does not match the camera token";
    return -3;
  }
  cudaSetDevice(device_);
  int rc = gemv_rows(p.cam, V, cd.bb0.K, cd.bb0.w, cd.bb0.ldw, cd.bb0.b, cd.bb0.N, 1, p.cam_h1, cd.bb0.N, 0, s);
  if (!rc) rc = gemv_rows(p.cam_h1, V, cd.bb2.K, cd.bb2.w, cd.bb2.ldw, cd.bb2.b, cd.bb2.N, 1, p.cam_h2, cd.bb2.N, 0, s);
  if (!rc) rc = gemv_rows(p.cam_h2, V, cd.fc_t.K, cd.fc_t.w, cd.fc_t.ldw, cd.fc_t.b, 3, 0, p.cam_pe, 9, 0, s);
  if (!rc) rc = gemv_rows(p.cam_h2, V, cd.fc_q.K, cd.fc_q.w, cd.fc_q.ldw, cd.fc_q.b, 4, 0, p.cam_pe, 9, 3, s);
  if (!rc) rc = gemv_rows(p.cam_h2, V, cd.fc_fov.K, cd.fc_fov.w, cd.fc_fov.ldw, cd.fc_fov.b, 2, 1, p.cam_pe, 9, 7, s);
  std::vector<float> proc(static_cast<size_t>(V) * 9);
  if (rc || cudaMemcpyAsync(proc.data(), p.cam_pe, proc.size() * 4, cudaMemcpyDeviceToHost, s) != cudaSuccess ||
      cudaStreamSynchronize(s) != cudaSuccess) {
    err_ = "camera decoder launch failed";
    return -4;
  }
  pe.assign(proc.size(), 0.f);
  const bool select = p.S >= 3 && model_->cfg.alt_start >= 0;
  std::vector<int> ref(p.scenes, 0);
  if (select) {
    if (cudaMemcpy(ref.data(), p.b_idx, ref.size() * sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -5;
  }
  for (int sc = 0; sc < p.scenes; ++sc)
    for (int q = 0; q < p.S; ++q) {
      // processing position q holds original view: the reference view first, then the
      // others in order (src/dino_backbone.cpp:427-441)
      const int b = ref[sc];
      const int t = !select ? q : (q == 0 ? b : (q <= b ? q - 1 : q));
      std::copy(&proc[(static_cast<size_t>(sc) * p.S + q) * 9], &proc[(static_cast<size_t>(sc) * p.S + q) * 9] + 9,
                &pe[(static_cast<size_t>(sc) * p.S + t) * 9]);
    }
  return 0;
}

void Engine::last_size(int* H, int* W) const {
  *H = last_ ? last_->H : 0;
  *W = last_ ? last_->W : 0;
}

std::vector<int> Engine::last_ref_views(cudaStream_t s) {
  std::vector<int> out;
  if (!last_ || last_->S < 3) return out;
  out.resize(last_->scenes);
  cudaMemcpyAsync(out.data(), last_->b_idx, out.size() * sizeof(int), cudaMemcpyDeviceToHost, s);
  cudaStreamSynchronize(s);
  return out;
}

int Engine::launches(int V, int S, int H, int W, bool rays) const {
  auto it = plans_.find(std::make_tuple(V, S, H, W, rays));
  return it == plans_.end() ? 0 : it->second->launches;
}

const __half* Engine::debug_feat(int o, int* rows, int* cols) const {
  if (!last_ || o < 0 || o > 3) return nullptr;
  *rows = last_->V * last_->Np;
  *cols = last_->Cf;
  return last_feat_[o];
}
const float* Engine::debug_x(int* rows, int* cols) const {
  if (!last_) return nullptr;
  *rows = last_->M;
  *cols = model_->cfg.embed_dim;
  return last_x_;
}

const float* Engine::debug_resid(int layer, int* rows, int* cols) const {
  if (!last_ || !last_->resid_cap || layer < 0 || layer >= model_->cfg.depth) return nullptr;
  *rows = last_->M;
  *cols = model_->cfg.embed_dim;
  return last_->resid_cap + static_cast<size_t>(layer) * last_->M * model_->cfg.embed_dim;
}

}  // namespace da3b
