// da3.h — C++ API of libda3b, source-compatible with DA3cpplib's public header
// (include/da3cpp/da3.h in DA3cpplib: Params :45-49, NestedParams :51-55, Image :58-62, ModelInfo :64-78,
// Result :80-90, InferOptions :92-103, load_model :105, load_nested_model :106, model_info :107,
// infer :109-110, infer_file :111-112, infer_preprocessed :119-126).
//
// Same types, names, argument meaning and error behaviour (bool false / nullptr,
// Result reset on entry, Result::depth empty on failure). The depth path runs on a
// B200 through libda3b's own sm_100a kernels; there is no CPU or ggml fallback.
#pragma once

#include <array>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#define DA3CPP_VERSION_MAJOR 0
#define DA3CPP_VERSION_MINOR 2
#define DA3CPP_VERSION_PATCH 0
#define DA3CPP_VERSION "0.2.0"

#if defined(__GNUC__)
#define DA3_API __attribute__((visibility("default")))
#else
#define DA3_API
#endif

namespace da3 {

struct Model;

// Kept for source compatibility. libda3b never runs TensorRT: with enabled=true and
// fallback_to_ggml=false load_model fails (as the reference does when TensorRT is
// unavailable); otherwise the request is ignored and the native path runs.
struct TensorRtParams {
  bool enabled = false;
  std::string onnx_path;
  std::string cache_dir;
  bool fp16 = true;
  bool fallback_to_ggml = true;
  std::size_t workspace_bytes = std::size_t{2} << 30;
};

enum class ModelKind {
  da3,
  da3_mono,
  da3_nested,
  da2_relative,
  da2_metric,
};

struct Params {
  std::string model_path;
  int n_threads = 4;  // host threads (unused by the GPU path)
  TensorRtParams tensorrt;
  int device = -1;    // CUDA device ordinal; -1 = $DA3B_DEVICE or 0
};

// Nested metric model (reference :51-55): DA3 anyview model + metric branch.
struct NestedParams {
  std::string anyview_model_path;
  std::string metric_model_path;
  int n_threads = 4;  // host threads (unused by the GPU path)
};

// Interleaved RGB8 image (width * height * 3 bytes).
struct Image {
  int width = 0;
  int height = 0;
  std::vector<std::uint8_t> data;
};

struct ModelInfo {
  ModelKind kind = ModelKind::da3;
  std::string checkpoint_name;
  int patch_size = 0;
  int resize_target = 0;
  std::array<float, 3> mean{};
  std::array<float, 3> std{};
  bool is_metric = false;
  bool has_camera_pose = false;
  bool has_aux_ray_head = false;
  bool tensorrt_enabled = false;
  bool tensorrt_active = false;
  std::string device_name = "cpu";
  bool gpu_active = false;
};

struct Result {
  int width = 0;
  int height = 0;
  std::vector<float> depth;
  std::vector<float> confidence;
  std::vector<float> sky;
  std::array<float, 12> extrinsics{};  // 3x4 row-major
  std::array<float, 9> intrinsics{};   // 3x3 row-major
  bool is_metric = false;
  bool has_pose = false;
};

struct InferOptions {
  bool with_pose = false;
  bool ray_pose = false;
  bool legacy_resize = false;
};

DA3_API std::shared_ptr<Model> load_model(const Params& params);
DA3_API std::shared_ptr<Model> load_nested_model(const NestedParams& params);
DA3_API ModelInfo model_info(const Model& model);

DA3_API bool infer(Model& model, const Image& image, Result& result, const InferOptions& options = {});
DA3_API bool infer_file(Model& model, const std::string& image_path, Result& result,
                        const InferOptions& options = {});

// Zero-copy input path: the callback receives the device buffer of the planar,
// already resized and normalised f32 image [3][H][W] and must fill it synchronously
// (device = true). DA3 cat-token models only, as in the reference.
struct UploadTarget {
  void* destination = nullptr;
  std::size_t bytes = 0;
  bool device = false;
};
using UploadCallback = std::function<void(const UploadTarget&)>;
DA3_API bool infer_preprocessed(Model& model, int height, int width, const UploadCallback& upload, Result& result);

// Batched extension (not in the reference): n RGB8 images of identical processed
// size (multiples of the patch size, no resize needed) in one forward.
DA3_API bool infer_batch(Model& model, const std::vector<Image>& images, std::vector<Result>& results);

}  // namespace da3
