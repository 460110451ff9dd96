// C ABI over DA3cpplib's own host-side sources, compiled unmodified from the reference
// checkout into oracle/_ref/ — test infrastructure only, never part of libda3b.
//
// Compiled: src/preprocess.cpp (the real/legacy preprocess and the uint8 cubic/area
// resizers), src/uv_posembed.cpp, src/nested.cpp (the nested metric alignment),
// src/ray_pose.cpp + src/linalg.cpp (the ray->pose solver), and src/rope2d.cpp +
// src/dino_backbone.cpp for their host functions: the 2-D RoPE tables, the bicubic
// pos-embed interpolation and the multi-view reference-view selection. The last two
// files also build ggml graphs; ggml's source is absent from the checkout, so the ggml
// names they use are declared in oracle/ref_shim/ and defined to abort in
// oracle/ref_stubs.cpp. None of the functions called here reaches them.
#include <cstdint>
#include <cstring>
#include <deque>
#include <functional>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <vector>

#include "dino_backbone.hpp"
#include "linalg.hpp"
#include "model_loader.hpp"
#include "nested.hpp"
#include "ray_pose.hpp"
#include "preprocess.hpp"
#include "rope2d.hpp"
#include "uv_posembed.hpp"

#define REF_API extern "C" __attribute__((visibility("default")))

namespace {
da::Config make_cfg(int patch, int target, int upper, const float* mean, const float* std_) {
  da::Config c;
  c.patch_size = static_cast<uint32_t>(patch);
  c.img_resize_target = static_cast<uint32_t>(target);
  c.img_resize_mode = upper ? "upper_bound" : "lower_bound";
  c.img_mean.assign(mean, mean + 3);
  c.img_std.assign(std_, std_ + 3);
  return c;
}
da::Image make_img(const uint8_t* rgb, int w, int h) {
  da::Image im;
  im.w = w;
  im.h = h;
  im.rgb.assign(rgb, rgb + static_cast<size_t>(w) * h * 3);
  return im;
}
}  // namespace

// preprocess_real (legacy = 0) or preprocess (legacy = 1). Writes at most cap floats of
// CHW output and, when rgb_out is non-null (real path only), the resized uint8 HWC
// image (cap_rgb bytes at most). Returns 0 on success, -1 when the reference returns
// false, -2 when an output buffer is too small.
REF_API int ref_preprocess(const uint8_t* rgb, int w, int h, int patch, int target, int upper, const float* mean,
                           const float* std_, int legacy, float* chw, int64_t cap, int* H, int* W, uint8_t* rgb_out,
                           int64_t cap_rgb) {
  const da::Config c = make_cfg(patch, target, upper, mean, std_);
  const da::Image im = make_img(rgb, w, h);
  da::Preprocessed p;
  std::vector<uint8_t> u8;
  const bool ok = legacy ? da::preprocess(im, c, p) : da::preprocess_real(im, c, p, rgb_out ? &u8 : nullptr);
  if (!ok) return -1;
  *H = p.H;
  *W = p.W;
  if (static_cast<int64_t>(p.chw.size()) > cap) return -2;
  std::memcpy(chw, p.chw.data(), p.chw.size() * sizeof(float));
  if (rgb_out && !legacy) {
    if (static_cast<int64_t>(u8.size()) > cap_rgb) return -2;
    std::memcpy(rgb_out, u8.data(), u8.size());
  }
  return 0;
}

// resize_cubic (mode 0) / resize_area (mode 1) of a uint8 HWC RGB image.
REF_API int ref_resize(const uint8_t* rgb, int w, int h, int dw, int dh, int mode, uint8_t* out) {
  const da::Image im = make_img(rgb, w, h);
  const da::Image r = mode == 0 ? da::resize_cubic(im, dw, dh) : da::resize_area(im, dw, dh);
  if (r.w != dw || r.h != dh) return -1;
  std::memcpy(out, r.rgb.data(), r.rgb.size());
  return 0;
}

// uv_pos_embed: [ph][pw][C] row-major, raw (not multiplied by the 0.1 ratio).
REF_API int ref_uv_pos_embed(int pw, int ph, int C, float aspect, float* out) {
  const std::vector<float> v = da::uv_pos_embed(pw, ph, C, aspect);
  if (v.size() != static_cast<size_t>(pw) * ph * C) return -1;
  std::memcpy(out, v.data(), v.size() * sizeof(float));
  return 0;
}

// NestedAligner::process_mono_sky on metric_depth (in place), then NestedAligner::align.
// Returns the scale factor.
REF_API float ref_nested_align(const float* any_depth, const float* any_conf, const float* any_ext,
                               const float* any_intr, float* metric_depth, const float* sky, int64_t n,
                               float* out_depth, float* out_ext) {
  const size_t N = static_cast<size_t>(n);
  da::AnyviewOut any;
  any.depth.assign(any_depth, any_depth + N);
  any.depth_conf.assign(any_conf, any_conf + N);
  for (int k = 0; k < 12; ++k) any.extrinsics[k] = any_ext[k];
  for (int k = 0; k < 9; ++k) any.intrinsics[k] = any_intr[k];
  da::MetricOut m;
  m.depth.assign(metric_depth, metric_depth + N);
  m.sky.assign(sky, sky + N);
  da::NestedAligner::process_mono_sky(m.depth, m.sky);
  std::memcpy(metric_depth, m.depth.data(), N * sizeof(float));
  // align() takes H and W only for their product
  const da::NestedOut r = da::NestedAligner::align(any, m, 1, static_cast<int>(N));
  std::memcpy(out_depth, r.depth.data(), N * sizeof(float));
  for (int k = 0; k < 12; ++k) out_ext[k] = r.extrinsics[k];
  return r.scale_factor;
}

// da::solve_ray_pose with its production defaults (no fed indices), as
// Engine::depth_pose_rays_native calls it. diag as in the oracle's or_ray_pose.
REF_API int ref_ray_pose(const float* ray, const float* conf, int Hy, int Wx, int img_h, int img_w, float* ext,
                         float* intr, double* diag) {
  da::RayPoseParams p;
  da::RayPoseOut o;
  if (!da::solve_ray_pose(ray, conf, Hy, Wx, img_h, img_w, nullptr, nullptr, nullptr, 0, p, o)) return -1;
  std::memcpy(ext, o.extrinsics.data(), 12 * sizeof(float));
  std::memcpy(intr, o.intrinsics.data(), 9 * sizeof(float));
  if (diag) {
    std::memcpy(diag, o.R, 9 * sizeof(double));
    std::memcpy(diag + 9, o.T, 3 * sizeof(double));
    diag[12] = o.focal[0];
    diag[13] = o.focal[1];
    diag[14] = o.pp[0];
    diag[15] = o.pp[1];
    std::memcpy(diag + 16, o.A, 9 * sizeof(double));
    diag[25] = o.n_inlier_best;
  }
  return 0;
}

REF_API void ref_qr(const double* a, int n, double* q, double* r) { da::linalg::householder_qr(a, n, q, r); }
REF_API void ref_ql3(const double* a, double* q, double* l) { da::linalg::ql_decomposition(a, q, l); }
REF_API void ref_smallest_eigvec(const double* m, int n, double* v) { da::linalg::smallest_eigvec(m, n, v); }
REF_API int ref_homography(const double* src, const double* dst, const double* w, int M, double* H) {
  return da::linalg::homography_weighted(src, dst, w, M, H) ? 0 : -1;
}

// ---------------------------------------------------------------- DA3 backbone host code
// Access to private members of the reference's classes without editing its headers:
// an explicit template instantiation may name a private member (the access rules do
// not apply to explicit instantiations), and it exports the member pointer through a
// friend function.
namespace {
template <typename Tag, typename Tag::type M>
struct Expose {
  friend typename Tag::type get(Tag) { return M; }
};
struct CfgTag {
  typedef da::Config da::ModelLoader::*type;
  friend type get(CfgTag);
};
struct InterpTag {
  typedef std::vector<float> (da::DinoBackbone::*type)(int, int) const;
  friend type get(InterpTag);
};
struct SaddleTag {
  typedef int (da::DinoBackbone::*type)(const std::vector<std::vector<float>>&, int) const;
  friend type get(SaddleTag);
};
}  // namespace
template struct Expose<CfgTag, &da::ModelLoader::cfg_>;
template struct Expose<InterpTag, &da::DinoBackbone::interp_pos_embed>;
template struct Expose<SaddleTag, &da::DinoBackbone::select_reference_view_saddle>;

// The checker's ModelLoader: model_loader.cpp (GGUF reading) is not compiled; tensor()
// serves the tensors registered by the entry points below.
namespace {
std::mutex g_ml_mu;
std::map<std::string, ggml_tensor> g_ml_tensors;
// interp_pos_embed caches its result by the pos_embed data pointer, so every call gets
// a buffer that stays alive (and therefore at a fresh address) until the library unloads.
std::deque<std::vector<float>> g_pe_keep;
}  // namespace
da::ModelLoader::~ModelLoader() {}
ggml_tensor* da::ModelLoader::tensor(const std::string& name) const {
  auto it = g_ml_tensors.find(name);
  return it == g_ml_tensors.end() ? nullptr : &it->second;
}

// build_rope_tables (src/rope2d.cpp:4-27): cos / sin [tokens][head_dim] for positions
// pos_yx [tokens][2] (y, x).
REF_API int ref_rope_tables(const float* pos_yx, int tokens, int head_dim, float freq, float* cos_out,
                            float* sin_out) {
  const std::vector<float> pos(pos_yx, pos_yx + static_cast<size_t>(tokens) * 2);
  const da::RopeTables rt = da::build_rope_tables(pos, tokens, head_dim, freq);
  const size_t n = static_cast<size_t>(tokens) * head_dim;
  if (rt.cos.size() != n || rt.sin.size() != n) return -1;
  std::memcpy(cos_out, rt.cos.data(), n * sizeof(float));
  std::memcpy(sin_out, rt.sin.data(), n * sizeof(float));
  return 0;
}

// DinoBackbone::interp_pos_embed (src/dino_backbone.cpp:18-56) of a pos-embed table
// [1 + grid^2][embed] to gh x gw: out [1 + gh*gw][embed].
REF_API int ref_interp_pos_embed(const float* pos_embed, int embed, int grid, float offset, int gh, int gw,
                                 float* out) {
  std::lock_guard<std::mutex> lk(g_ml_mu);
  g_pe_keep.emplace_back(pos_embed, pos_embed + static_cast<size_t>(1 + grid * grid) * embed);
  ggml_tensor t{};
  t.type = GGML_TYPE_F32;
  t.ne[0] = embed;
  t.ne[1] = 1 + grid * grid;
  t.ne[2] = t.ne[3] = 1;
  t.data = g_pe_keep.back().data();
  g_ml_tensors["vit.pos_embed"] = t;
  da::ModelLoader ml;
  da::Config& cfg = ml.*get(CfgTag());
  cfg.embed_dim = static_cast<uint32_t>(embed);
  cfg.pos_embed_grid = static_cast<uint32_t>(grid);
  cfg.interp_offset = offset;
  da::Backend be;
  da::DinoBackbone bb(ml, be);
  const std::vector<float> v = (bb.*get(InterpTag()))(gh, gw);
  if (v.size() != static_cast<size_t>(1 + gh * gw) * embed) return -1;
  std::memcpy(out, v.data(), v.size() * sizeof(float));
  return 0;
}

// DinoBackbone::select_reference_view_saddle (src/dino_backbone.cpp:372-412) on S views'
// CLS features cls [S][embed]; returns the selected view.
REF_API int ref_select_saddle(const float* cls, int S, int embed) {
  std::vector<std::vector<float>> c(S);
  for (int s = 0; s < S; ++s) c[s].assign(cls + static_cast<size_t>(s) * embed, cls + static_cast<size_t>(s + 1) * embed);
  da::ModelLoader ml;
  da::Backend be;
  da::DinoBackbone bb(ml, be);
  return (bb.*get(SaddleTag()))(c, embed);
}
