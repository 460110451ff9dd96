// C++ API check of libda3b (include/da3cpp/da3.h), built and run by tests/test_cpp_api_gpu.py.
//
//   da3_api_check <da3 gguf> <da2 gguf> <size>
//
// 1. load_model + model_info on a DA3 checkpoint;
// 2. infer() on a seeded RGB8 image at the processed size;
// 3. infer_preprocessed() on the same image, normalised here exactly as the reference's
//    preprocess does ((v / 255 - mean) / std in f32, planar [3][H][W]) and uploaded by
//    the callback into the device buffer the library hands out: depth and confidence
//    must be bit-identical to step 2;
// 4. the reference's refusals: infer_preprocessed on a DA2 checkpoint, infer() on an
//    image whose data size does not match, both return false with an empty Result.
// Prints "OK" and exits 0 when every check holds.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>
#include <random>
#include <vector>

#include "da3cpp/da3.h"

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
  std::printf("OK\n");
  return 0;
}
