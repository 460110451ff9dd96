// Nested metric alignment (src/nested.cpp:7-96), host side. The two branches' outputs
// are already on the host when this runs; the order statistics use selection rather
// than a full sort (linear instead of n log n, identical values).
#include "nested.h"

#include <algorithm>
#include <cmath>
#include <vector>

namespace da3b {

float quantile_linear(float* v, size_t n, float q) {
  if (n == 0) return 0.0f;
  if (n == 1) return v[0];
  const double pos = static_cast<double>(q) * static_cast<double>(n - 1);
  const double lo_d = std::floor(pos);
  const size_t lo = static_cast<size_t>(lo_d);
  size_t hi = static_cast<size_t>(std::ceil(pos));
  if (hi >= n) hi = n - 1;
  std::nth_element(v, v + lo, v + n);
  const float a = v[lo];
  const float b = hi == lo ? a : *std::min_element(v + lo + 1, v + n);
  const double frac = pos - lo_d;
  return static_cast<float>(static_cast<double>(a) + frac * (static_cast<double>(b) - static_cast<double>(a)));
}

namespace {
inline bool non_sky(float s) { return s < 0.3f; }
}  // namespace

void mono_sky_fill(float* depth, const float* sky, size_t n) {
  if (n == 0) return;
  std::vector<float> ns;
  ns.reserve(n);
  for (size_t i = 0; i < n; ++i)
    if (non_sky(sky[i])) ns.push_back(depth[i]);
  const size_t n_sky = n - ns.size();
  if (ns.size() <= 10 || n_sky <= 10) return;
  const float fill = quantile_linear(ns.data(), ns.size(), 0.99f);
  for (size_t i = 0; i < n; ++i)
    if (!non_sky(sky[i])) depth[i] = fill;
}

float nested_align(const float* any_depth, const float* any_conf, const float any_ext[12], const float any_intr[9],
                   const float* metric_depth, const float* sky, size_t n, float* out_depth, float out_ext[12]) {
  // metric depth scaled by the anyview focal length / 300
  const float focal = (any_intr[0] + any_intr[4]) * 0.5f;
  const float metric_scale = focal / 300.0f;
  // median confidence over the non-sky pixels
  std::vector<float> buf;
  buf.reserve(n);
  for (size_t i = 0; i < n; ++i)
    if (non_sky(sky[i])) buf.push_back(any_conf[i]);
  const float median_conf = quantile_linear(buf.data(), buf.size(), 0.5f);
  // least-squares scale sum(a*b) / sum(b*b) over confident non-sky pixels with valid depths
  double num = 0.0, den = 0.0;
  for (size_t i = 0; i < n; ++i) {
    const float md = metric_depth[i] * metric_scale;
    if (non_sky(sky[i]) && any_conf[i] >= median_conf && md > 1e-2f && any_depth[i] > 1e-3f) {
      const double a = md, b = any_depth[i];
      num += a * b;
      den += b * b;
    }
  }
  if (den < 1e-12) den = 1e-12;
  const float scale = static_cast<float>(num / den);
  for (int k = 0; k < 12; ++k) out_ext[k] = any_ext[k];
  out_ext[3] *= scale;
  out_ext[7] *= scale;
  out_ext[11] *= scale;
  for (size_t i = 0; i < n; ++i) out_depth[i] = any_depth[i] * scale;
  // sky pixels -> min(0.99 quantile of the scaled non-sky depth, 200)
  buf.clear();
  for (size_t i = 0; i < n; ++i)
    if (non_sky(sky[i])) buf.push_back(out_depth[i]);
  float fill = quantile_linear(buf.data(), buf.size(), 0.99f);
  if (fill > 200.0f) fill = 200.0f;
  for (size_t i = 0; i < n; ++i)
    if (!non_sky(sky[i])) out_depth[i] = fill;
  return scale;
}

}  // namespace da3b
