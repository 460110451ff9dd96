// C ABI over DA3cpplib's own host-only sources, compiled unmodified from the reference
// checkout into oracle/_ref/ — test infrastructure only, never part of libda3b.
//
// Only src/preprocess.cpp (the real/legacy preprocess and the uint8 cubic/area
// resizers), src/uv_posembed.cpp, src/nested.cpp (the nested metric alignment) and
// src/ray_pose.cpp + src/linalg.cpp (the ray->pose solver) are compiled: they need
// nothing from ggml beyond
// the opaque type names that model_loader.hpp mentions (oracle/ref_shim/). Everything
// else on the depth path goes through ggml graphs, whose source is absent from the
// reference checkout, so it cannot be built here.
#include <cstdint>
#include <cstring>
#include <vector>

#include "linalg.hpp"
#include "nested.hpp"
#include "ray_pose.hpp"
#include "preprocess.hpp"
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
