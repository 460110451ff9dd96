// Ray -> pose solver of DA3 (use_ray_pose, src/ray_pose.cpp:95-252 with
// src/linalg.cpp:8-203): camera-to-world extrinsics and intrinsics from the aux ray
// head's per-pixel ray field by a weighted homography RANSAC and a QL decomposition.
//
// The data-parallel parts run on the GPU in double precision with no fused
// multiply-add contraction (this file's kernels are built with -fmad=false), so every
// value equals the reference's host double arithmetic: the ray cloud, a stable radix
// sort of the points by weight, the 100 hypothesis fits, the inlier masks (100 x N),
// the ordered inlier-weight sums, the confidence-weighted mean origin and the refit's
// normal matrix. The host keeps what is sequential by nature: the seeded draws and the
// shuffle (same std::mt19937 / std::uniform_int_distribution / std::shuffle calls as
// the reference), the refit's 9x9 eigenproblem and the 3x3 QL.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace da3b {

struct RayPoseResult {
  float ext[12];   // camera-to-world 3x4, row-major
  float intr[9];   // 3x3, row-major
  double R[9], T[3], focal[2], pp[2], A[9];
  int n_inlier_best = 0;
};

class RaySolver {
 public:
  RaySolver() = default;
  ~RaySolver();
  RaySolver(const RaySolver&) = delete;
  RaySolver& operator=(const RaySolver&) = delete;

  // rays: device f32 planes [7][n_views][Hy][Wx] (direction xyz, origin xyz, confidence
  // after exp+1), the aux ray head's layout; solves view `view`. Returns 0, 1 when the
  // reference reports a degenerate field (no pose), or a negative error code (*err set).
  // Synchronises `s` twice (after the RANSAC and after the refit's normal matrix).
  int solve(const float* rays, int n_views, int view, int Hy, int Wx, int img_h, int img_w, cudaStream_t s,
            RayPoseResult* out, std::string* err);

 private:
  bool reserve(int N, std::string* err);
  void release();
  int cap_ = 0, draws_for_ = -1;
  // device
  double2* dst_ = nullptr;  // z-normalised direction per point
  double *w_ = nullptr, *H_ = nullptr, *scores_ = nullptr, *sums_ = nullptr, *ata_ = nullptr;
  uint32_t* keys_[2] = {nullptr, nullptr};
  int* hist_ = nullptr;
  int *vals_[2] = {nullptr, nullptr}, *draws_ = nullptr, *fit_ok_ = nullptr, *best_ = nullptr, *refit_ = nullptr;
  uint8_t *mask_ = nullptr, *bestmask_ = nullptr;
  // pinned host
  int* h_order_ = nullptr;
  uint8_t* h_mask_ = nullptr;
  double* h_small_ = nullptr;  // [4] origin / confidence sums, [4] best iteration
  int* h_refit_ = nullptr;
  double* h_ata_ = nullptr;
};

// Host helpers shared with the solver (same arithmetic as src/linalg.cpp).
double det3(const double a[9]);
void ql3(const double a[9], double q[9], double l[9]);

}  // namespace da3b
