// Camera pose from DA3's 9-value pose encoding [t(3), quaternion xyzw (4), fov h/w (2)]:
// pose_encoding_to_extri_intri of CamPose::pose (src/cam_pose.cpp:40-83), in f32 with
// the same operations. ext: world-to-camera 3x4 row-major [R^T | -R^T t] of the
// camera-to-world [R | t]; intr: 3x3 row-major with the principal point at the image
// centre of the processed size H x W.
#pragma once
#include <algorithm>
#include <cmath>

namespace da3b {

inline void pose_to_ext_intr(const float* pe, int H, int W, float* ext, float* intr) {
  const float qi = pe[3], qj = pe[4], qk = pe[5], qr = pe[6];
  const float sc = 2.0f / (qi * qi + qj * qj + qk * qk + qr * qr);
  const float R[3][3] = {{1.0f - sc * (qj * qj + qk * qk), sc * (qi * qj - qk * qr), sc * (qi * qk + qj * qr)},
                         {sc * (qi * qj + qk * qr), 1.0f - sc * (qi * qi + qk * qk), sc * (qj * qk - qi * qr)},
                         {sc * (qi * qk - qj * qr), sc * (qj * qk + qi * qr), 1.0f - sc * (qi * qi + qj * qj)}};
  for (int r = 0; r < 3; ++r) {
    float acc = 0.0f;
    for (int k = 0; k < 3; ++k) acc += R[k][r] * pe[k];
    for (int k = 0; k < 3; ++k) ext[r * 4 + k] = R[k][r];
    ext[r * 4 + 3] = -acc;
  }
  const float fy = (H / 2.0f) / std::max(std::tan(pe[7] / 2.0f), 1e-6f);
  const float fx = (W / 2.0f) / std::max(std::tan(pe[8] / 2.0f), 1e-6f);
  for (int i = 0; i < 9; ++i) intr[i] = 0.0f;
  intr[0] = fx;
  intr[4] = fy;
  intr[2] = W / 2.0f;
  intr[5] = H / 2.0f;
  intr[8] = 1.0f;
}

}  // namespace da3b
