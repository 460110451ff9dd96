// C++ API check of libda3b (include/da3cpp/da3.h), built and run by tests/test_cpp_api_gpu.py.
//
//   da3_api_check <da3 gguf> <da2 gguf> <size> [<mono gguf> <metric-branch gguf>]
//
// 1. load_model + model_info on a DA3 checkpoint;
// 2. infer() on a seeded RGB8 image at the processed size;
// 3. infer_preprocessed() on the same image, normalised here exactly as the reference's
//    preprocess does ((v / 255 - mean) / std in f32, planar [3][H][W]) and uploaded by
//    the callback into the device buffer the library hands out: depth and confidence
//    must be bit-identical to step 2;
// 4. the reference's refusals: infer_preprocessed on a DA2 checkpoint, infer() on an
//    image whose data size does not match, both return false with an empty Result;
// 5. InferOptions::ray_pose with with_pose: the ray->pose solver's camera-to-world pose
//    equals da3b_ray_pose on the ray field da3b_infer_device writes for the same image;
//    ray_pose without with_pose, with legacy_resize, or on DA2 is refused;
// 6. (with the optional models) DA3 mono: kind, depth + sky and no confidence, refusal of
//    with_pose and infer_preprocessed; nested: load_nested_model with the DA3 model as the
//    anyview branch, kind / camera pose / metric flags, depth + pose without confidence or
//    sky, and the infer_preprocessed refusal (src/api.cpp:95-161, :184).
// Prints "OK" and exits 0 when every check holds.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "da3b.h"
#include "da3cpp/da3.h"
#include "da3cpp/da3_c.h"

#define CHECK(c)                                         \
  do {                                                   \
    if (!(c)) {                                          \
      std::printf("FAIL %s:%d %s\n", __FILE__, __LINE__, #c); \
      return 1;                                          \
    }                                                    \
  } while (0)

int main(int argc, char** argv) {
  if (argc < 4) return 2;
  const int n = std::atoi(argv[3]);
  da3::Params p;
  p.model_path = argv[1];
  auto model = da3::load_model(p);
  CHECK(model);
  const da3::ModelInfo info = da3::model_info(*model);
  CHECK(info.patch_size == 14);

  da3::Image img;
  img.width = n;
  img.height = n;
  img.data.resize(static_cast<size_t>(n) * n * 3);
  std::mt19937_64 rng(20260101);
  for (auto& v : img.data) v = static_cast<uint8_t>(rng() & 255);

  da3::Result a;
  CHECK(da3::infer(*model, img, a));
  CHECK(a.width == n && a.height == n && a.depth.size() == static_cast<size_t>(n) * n);

  std::vector<float> chw(static_cast<size_t>(3) * n * n);
  for (int c = 0; c < 3; ++c)
    for (int i = 0; i < n * n; ++i)
      chw[static_cast<size_t>(c) * n * n + i] = (static_cast<float>(img.data[static_cast<size_t>(i) * 3 + c]) / 255.f -
                                                  info.mean[c]) / info.std[c];
  bool called = false;
  da3::Result b;
  CHECK(da3::infer_preprocessed(*model, n, n, [&](const da3::UploadTarget& t) {
    called = t.device && t.bytes == chw.size() * sizeof(float) &&
             cudaMemcpy(t.destination, chw.data(), t.bytes, cudaMemcpyHostToDevice) == cudaSuccess;
  }, b));
  CHECK(called);
  CHECK(b.width == n && b.height == n);
  CHECK(b.depth.size() == a.depth.size() && std::memcmp(b.depth.data(), a.depth.data(), a.depth.size() * 4) == 0);
  CHECK(b.confidence.size() == a.confidence.size() &&
        std::memcmp(b.confidence.data(), a.confidence.data(), a.confidence.size() * 4) == 0);

  da3::Params p2;
  p2.model_path = argv[2];
  auto da2 = da3::load_model(p2);
  CHECK(da2);
  da3::Result c;
  CHECK(!da3::infer_preprocessed(*da2, n, n, [&](const da3::UploadTarget&) {}, c));
  CHECK(c.depth.empty());
  da3::Image bad = img;
  bad.data.pop_back();
  CHECK(!da3::infer(*model, bad, c));
  CHECK(c.depth.empty());

  {
    da3::InferOptions rp;
    rp.with_pose = true;
    rp.ray_pose = true;
    da3::Result rr;
    CHECK(da3::infer(*model, img, rr, rp));
    CHECK(rr.has_pose && rr.depth.size() == a.depth.size());
    CHECK(std::memcmp(rr.depth.data(), a.depth.data(), a.depth.size() * 4) == 0);
    da_ctx* ctx = da3b_load(argv[1], 0);
    CHECK(ctx);
    const int g = 8 * (n / 14);
    void *d_img = nullptr, *d_depth = nullptr, *d_conf = nullptr, *d_rays = nullptr;
    CHECK(cudaMalloc(&d_img, img.data.size()) == cudaSuccess);
    CHECK(cudaMalloc(&d_depth, static_cast<size_t>(n) * n * 4) == cudaSuccess);
    CHECK(cudaMalloc(&d_conf, static_cast<size_t>(n) * n * 4) == cudaSuccess);
    CHECK(cudaMalloc(&d_rays, static_cast<size_t>(7) * g * g * 4) == cudaSuccess);
    CHECK(cudaMemcpy(d_img, img.data.data(), img.data.size(), cudaMemcpyHostToDevice) == cudaSuccess);
    CHECK(da3b_infer_device(ctx, d_img, 1, 1, n, n, d_depth, d_conf, d_rays, nullptr) == 0);
    CHECK(cudaDeviceSynchronize() == cudaSuccess);
    float ext[12], intr[9];
    CHECK(da3b_ray_pose(ctx, static_cast<const float*>(d_rays), 1, 0, g, g, n, n, ext, intr, nullptr, nullptr) == 0);
    CHECK(std::memcmp(ext, rr.extrinsics.data(), sizeof(ext)) == 0);
    CHECK(std::memcmp(intr, rr.intrinsics.data(), sizeof(intr)) == 0);
    cudaFree(d_img);
    cudaFree(d_depth);
    cudaFree(d_conf);
    cudaFree(d_rays);
    da_capi_free(ctx);
    da3::InferOptions only_rays;
    only_rays.ray_pose = true;
    CHECK(!da3::infer(*model, img, rr, only_rays) && rr.depth.empty());
    rp.legacy_resize = true;
    CHECK(!da3::infer(*model, img, rr, rp) && rr.depth.empty());
    rp.legacy_resize = false;
    CHECK(!da3::infer(*da2, img, rr, rp) && rr.depth.empty());
  }

  if (argc >= 6) {
    da3::Params pm;
    pm.model_path = argv[4];
    auto mono = da3::load_model(pm);
    CHECK(mono);
    const da3::ModelInfo mi = da3::model_info(*mono);
    CHECK(mi.kind == da3::ModelKind::da3_mono && mi.is_metric && !mi.has_camera_pose);
    da3::Result r;
    CHECK(da3::infer(*mono, img, r));
    CHECK(r.depth.size() == static_cast<size_t>(n) * n && r.sky.size() == r.depth.size() && r.confidence.empty());
    CHECK(!r.has_pose && r.is_metric);
    da3::InferOptions wp;
    wp.with_pose = true;
    CHECK(!da3::infer(*mono, img, r, wp) && r.depth.empty());
    CHECK(!da3::infer_preprocessed(*mono, n, n, [&](const da3::UploadTarget&) {}, r));

    da3::NestedParams np;
    np.anyview_model_path = argv[1];
    np.metric_model_path = argv[5];
    auto nested = da3::load_nested_model(np);
    CHECK(nested);
    const da3::ModelInfo ni = da3::model_info(*nested);
    CHECK(ni.kind == da3::ModelKind::da3_nested && ni.is_metric && ni.has_camera_pose);
    da3::Result q;
    CHECK(da3::infer(*nested, img, q));
    CHECK(q.depth.size() == static_cast<size_t>(n) * n && q.confidence.empty() && q.sky.empty());
    CHECK(q.has_pose && q.is_metric && q.intrinsics[8] == 1.f);
    CHECK(!da3::infer_preprocessed(*nested, n, n, [&](const da3::UploadTarget&) {}, q));
    np.metric_model_path.clear();
    CHECK(!da3::load_nested_model(np));
  }
  std::printf("OK\n");
  return 0;
}
