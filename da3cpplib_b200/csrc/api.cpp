// Public boundary of libda3b: the DA3cpplib-compatible C++ API (da3::), its C ABI
// (da_capi_*), and the model-level batched entry points (da3b_*). Everything here is
// host code; inference runs through Engine on the GPU.
#include <cuda_runtime.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <memory>
#include <string>
#include <vector>

#include "da3b.h"
#include "da3cpp/da3.h"
#include "da3cpp/da3_c.h"
#include "engine.h"
#include "kernels.h"
#include "nested.h"
#include "pose.h"
#include "preprocess.h"
#include "raypose.h"

#define DA_LOG(...)                     \
  do {                                  \
    fprintf(stderr, "[da3b] ");         \
    fprintf(stderr, __VA_ARGS__);       \
    fprintf(stderr, "\n");              \
  } while (0)

struct da_ctx {
  std::unique_ptr<da3b::Engine> engine;
  // nested metric models (src/engine.cpp:67-77): the metric branch next to the anyview
  // engine above, on the same device and stream
  std::unique_ptr<da3b::Engine> metric;
  std::string last_error;
  cudaStream_t stream = nullptr;
  // preprocess_real on the GPU for inputs that need a resize: original image upload
  // buffer and processed-size output (grow-only), tap tables and scratch
  std::unique_ptr<da3b::Resizer> resizer;
  // ray -> pose solver scratch (InferOptions::ray_pose, da3b_ray_pose)
  std::unique_ptr<da3b::RaySolver> raysolver;
  uint8_t* in_dev = nullptr;
  size_t in_cap = 0;
  uint8_t* pre_dev = nullptr;
  size_t pre_cap = 0;
  ~da_ctx() {
    if (engine) cudaSetDevice(engine->device());
    if (stream) cudaStreamSynchronize(stream);
    resizer.reset();
    raysolver.reset();
    if (in_dev) cudaFree(in_dev);
    if (pre_dev) cudaFree(pre_dev);
    if (stream) cudaStreamDestroy(stream);
  }
};

namespace {

int default_device() {
  if (const char* d = getenv("DA3B_DEVICE")) return atoi(d);
  return 0;
}

// Processed size (src/preprocess.cpp:26-41 legacy, :157-197 real policy).
void processed_size(const da3b::Config& c, int w, int h, bool legacy, int* ow, int* oh) {
  const int patch = c.patch_size;
  if (legacy) {
    int dw = (w / patch) * patch, dh = (h / patch) * patch;
    *ow = dw == 0 ? patch : dw;
    *oh = dh == 0 ? patch : dh;
    return;
  }
  const int target = c.img_resize_target > 0 ? c.img_resize_target : 504;
  const bool upper = c.img_resize_mode.rfind("lower", 0) != 0;
  int cw = w, ch = h;
  const int bound = upper ? std::max(cw, ch) : std::min(cw, ch);
  if (bound != target) {
    const double scale = static_cast<double>(target) / bound;
    cw = std::max(1, static_cast<int>(std::nearbyint(cw * scale)));
    ch = std::max(1, static_cast<int>(std::nearbyint(ch * scale)));
  }
  auto nearest = [](int x, int p) {
    const int down = (x / p) * p, up = down + p;
    return (std::abs(up - x) <= std::abs(x - down)) ? up : down;
  };
  *ow = std::max(1, nearest(cw, patch));
  *oh = std::max(1, nearest(ch, patch));
}

bool read_ppm(const char* path, int* w, int* h, std::vector<uint8_t>& rgb, std::string* err) {
  FILE* f = fopen(path, "rb");
  if (!f) { *err = std::string("cannot open image ") + path; return false; }
  char magic[3] = {0, 0, 0};
  int maxv = 0;
  bool ok = fscanf(f, "%2s", magic) == 1 && strcmp(magic, "P6") == 0 && fscanf(f, "%d %d %d", w, h, &maxv) == 3 &&
            maxv == 255 && *w > 0 && *h > 0;
  if (ok) {
    fgetc(f);
    rgb.resize(static_cast<size_t>(*w) * *h * 3);
    ok = fread(rgb.data(), 1, rgb.size(), f) == rgb.size();
  }
  fclose(f);
  if (!ok) *err = std::string("image decode supports binary PPM (P6, 8-bit) only: ") + path;
  return ok;
}

bool is_mono(const da3b::Engine& e) { return e.has_sky() && e.output_dim() == 1; }

bool is_nested(const da_ctx* c) { return c->metric != nullptr; }

// Metric-scale checkpoints by name (src/da_capi.cpp:41-52, src/api.cpp:21-30).
bool name_is_metric(const da3b::Config& c) {
  if (c.head_max_depth > 0.f) return true;
  std::string n = c.checkpoint_name;
  std::transform(n.begin(), n.end(), n.begin(), [](unsigned char ch) { return static_cast<char>(tolower(ch)); });
  return n.find("metric") != std::string::npos || n.find("nested") != std::string::npos ||
         n.find("mono") != std::string::npos;
}

// Legacy preprocess on the GPU (src/preprocess.cpp:8-41, bit-exact): upload n views,
// float bilinear to the floor-to-patch size and normalisation straight into the plan's
// planar f32 input, then the forward from it (scenes of S views).
bool run_legacy(da_ctx* c, const uint8_t* rgb, int n, int S, int w, int h, std::vector<float>& depth,
                std::vector<float>* conf, int* oh, int* ow) {
  da3b::Engine& e = *c->engine;
  cudaSetDevice(e.device());
  const auto& cfg = e.config();
  int W = 0, H = 0;
  if (da3b::legacy_preprocess(nullptr, n, w, h, cfg.patch_size, cfg.img_mean.data(), cfg.img_std.data(), nullptr, &W,
                              &H, c->stream) != 0) {
    c->last_error = "preprocess: bad legacy size";
    return false;
  }
  const size_t in_bytes = static_cast<size_t>(n) * w * h * 3;
  if (in_bytes > c->in_cap) {
    if (c->in_dev) {
      cudaStreamSynchronize(c->stream);
      cudaFree(c->in_dev);
    }
    c->in_dev = nullptr;
    c->in_cap = 0;
    if (cudaMalloc(&c->in_dev, in_bytes) != cudaSuccess) {
      c->last_error = "preprocess: out of device memory";
      return false;
    }
    c->in_cap = in_bytes;
  }
  float* chw = e.prepared_input(n, S, H, W, nullptr);
  if (!chw || cudaMemcpyAsync(c->in_dev, rgb, in_bytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
      da3b::legacy_preprocess(c->in_dev, n, w, h, cfg.patch_size, cfg.img_mean.data(), cfg.img_std.data(), chw, &W, &H,
                              c->stream) != 0) {
    c->last_error = "preprocess: legacy resize failed " + e.last_error();
    return false;
  }
  depth.resize(static_cast<size_t>(n) * H * W);
  const bool want_conf = conf && e.output_dim() >= 2;
  if (want_conf) conf->resize(depth.size());
  const int rc = e.run_prepared(n, S, H, W, depth.data(), want_conf ? conf->data() : nullptr, c->stream);
  if (rc != 0 || cudaStreamSynchronize(c->stream) != cudaSuccess || e.status() != 0) {
    c->last_error = "depth: forward failed: " + e.last_error();
    return false;
  }
  *oh = H;
  *ow = W;
  return true;
}

// Single-image inference at the processed size (H2D, forward, D2H). rays: also run the
// aux ray head, leaving its planes on the device (Engine::last_rays).
bool run_one(da_ctx* c, const uint8_t* rgb, int w, int h, bool legacy, std::vector<float>& depth,
             std::vector<float>* conf, int* oh, int* ow, bool rays = false) {
  da3b::Engine& e = *c->engine;
  int W = 0, H = 0;
  processed_size(e.config(), w, h, legacy, &W, &H);
  if (W != w || H != h) {
    if (legacy) return run_legacy(c, rgb, 1, 1, w, h, depth, conf, oh, ow);
    // preprocess_real on the GPU (src/preprocess.cpp:157-197): upload, resize, then the
    // processed image feeds the forward below
    cudaSetDevice(e.device());
    const size_t in_bytes = static_cast<size_t>(w) * h * 3, pre_bytes = static_cast<size_t>(W) * H * 3;
    auto grow = [&](uint8_t*& p, size_t& cap, size_t need) -> bool {
      if (need <= cap) return true;
      if (p) {
        cudaStreamSynchronize(c->stream);
        cudaFree(p);
      }
      p = nullptr;
      cap = 0;
      if (cudaMalloc(&p, need) != cudaSuccess) return false;
      cap = need;
      return true;
    };
    if (!c->resizer) c->resizer.reset(new da3b::Resizer());
    const auto& cfg = e.config();
    int rw = 0, rh = 0;
    if (!grow(c->in_dev, c->in_cap, in_bytes) || !grow(c->pre_dev, c->pre_cap, pre_bytes) ||
        cudaMemcpyAsync(c->in_dev, rgb, in_bytes, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
        c->resizer->preprocess_real(c->in_dev, 1, w, h, cfg.patch_size,
                                    cfg.img_resize_target > 0 ? cfg.img_resize_target : 504,
                                    cfg.img_resize_mode.rfind("lower", 0) != 0, c->pre_dev, &rw, &rh, c->stream) != 0 ||
        rw != W || rh != H) {
      c->last_error = "preprocess: GPU resize to " + std::to_string(W) + "x" + std::to_string(H) + " failed";
      return false;
    }
    rgb = c->pre_dev;
  }
  depth.resize(static_cast<size_t>(H) * W);
  const bool want_conf = conf && e.output_dim() >= 2;
  if (want_conf) conf->resize(static_cast<size_t>(H) * W);
  cudaSetDevice(e.device());
  const int rc = rays ? e.run_with_rays(rgb, 1, 1, H, W, depth.data(), want_conf ? conf->data() : nullptr, c->stream)
                      : e.run(rgb, 1, 1, H, W, depth.data(), want_conf ? conf->data() : nullptr, nullptr, c->stream);
  if (rc != 0 || cudaStreamSynchronize(c->stream) != cudaSuccess || e.status() != 0) {
    c->last_error = "depth: forward failed: " + e.last_error();
    return false;
  }
  *oh = H;
  *ow = W;
  return true;
}

// Sky plane of the last forward (relu of the sky logits), host copy.
bool fetch_sky(da_ctx* c, da3b::Engine& e, size_t n, std::vector<float>& sky) {
  sky.resize(n);
  if (e.sky(sky.data(), n, c->stream) != 0 || cudaStreamSynchronize(c->stream) != cudaSuccess) {
    c->last_error = "sky: " + e.last_error();
    sky.clear();
    return false;
  }
  return true;
}

// Nested metric depth of one image (src/engine.cpp:416-451): the legacy preprocess
// feeds both branches; anyview -> depth, confidence and camera pose; metric -> depth and
// sky; then the sky fill and the alignment on the host (src/nested.cpp:22-96).
bool run_nested(da_ctx* c, const uint8_t* rgb, int w, int h, std::vector<float>& depth, float ext[12],
                float intr[9], int* oh, int* ow) {
  da3b::Engine& a = *c->engine;
  da3b::Engine& m = *c->metric;
  std::vector<float> conf;
  int H = 0, W = 0;
  if (!run_legacy(c, rgb, 1, 1, w, h, depth, &conf, &H, &W)) return false;
  if (conf.size() != depth.size()) {
    c->last_error = "nested: the anyview model has no confidence channel";
    return false;
  }
  std::vector<float> pe;
  if (a.poses(pe, c->stream) != 0) {
    c->last_error = "nested: camera pose failed: " + a.last_error();
    return false;
  }
  float any_ext[12];
  da3b::pose_to_ext_intr(pe.data(), H, W, any_ext, intr);
  // same normalised input for the metric branch: device copy of the anyview plan's input
  size_t bytes = 0, bytes_m = 0;
  float* src = a.prepared_input(1, 1, H, W, &bytes);
  float* dst = m.prepared_input(1, 1, H, W, &bytes_m);
  const size_t n = static_cast<size_t>(H) * W;
  std::vector<float> mdepth(n), sky;
  if (!src || !dst || bytes != bytes_m ||
      cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, c->stream) != cudaSuccess ||
      m.run_prepared(1, 1, H, W, mdepth.data(), nullptr, c->stream) != 0 ||
      cudaStreamSynchronize(c->stream) != cudaSuccess || m.status() != 0) {
    c->last_error = "nested: metric branch failed: " + m.last_error();
    return false;
  }
  if (!fetch_sky(c, m, n, sky)) return false;
  da3b::mono_sky_fill(mdepth.data(), sky.data(), n);
  da3b::nested_align(depth.data(), conf.data(), any_ext, intr, mdepth.data(), sky.data(), n, depth.data(), ext);
  *oh = H;
  *ow = W;
  return true;
}

da_ctx* make_ctx(const char* path, int device, std::string* err) {
  if (!path) { *err = "null path"; return nullptr; }
  auto e = da3b::Engine::create(path, device, err);
  if (!e) return nullptr;
  auto* c = new da_ctx();
  c->engine = std::move(e);
  cudaSetDevice(device);
  cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking);
  return c;
}

}  // namespace

// ====================================================================== da3:: C++ API
namespace da3 {

struct Model {
  std::unique_ptr<da_ctx> ctx;
};

std::shared_ptr<Model> load_model(const Params& params) {
  if (params.model_path.empty()) return nullptr;
  if (params.tensorrt.enabled && !params.tensorrt.fallback_to_ggml) {
    DA_LOG("load_model: TensorRT is not part of this library and fallback is disabled");
    return nullptr;
  }
  std::string err;
  da_ctx* c = make_ctx(params.model_path.c_str(), params.device >= 0 ? params.device : default_device(), &err);
  if (!c) {
    DA_LOG("load_model: %s", err.c_str());
    return nullptr;
  }
  auto m = std::make_shared<Model>();
  m->ctx.reset(c);
  return m;
}

// src/api.cpp:69-78 / src/engine.cpp:67-77: the anyview model plus the metric branch
// (a metric-branch GGUF with m_vit.* / m_head.* or any DPT with a sky head).
std::shared_ptr<Model> load_nested_model(const NestedParams& params) {
  if (params.anyview_model_path.empty() || params.metric_model_path.empty()) return nullptr;
  da_ctx* c = da_capi_load_nested(params.anyview_model_path.c_str(), params.metric_model_path.c_str(),
                                  params.n_threads);
  if (!c) return nullptr;
  auto m = std::make_shared<Model>();
  m->ctx.reset(c);
  return m;
}

ModelInfo model_info(const Model& model) {
  ModelInfo info;
  if (!model.ctx || !model.ctx->engine) return info;
  const da3b::Engine& e = *model.ctx->engine;
  const da3b::Config& c = e.config();
  info.checkpoint_name = c.checkpoint_name;
  info.patch_size = c.patch_size;
  info.resize_target = c.img_resize_target;
  for (int i = 0; i < 3; ++i) {
    info.mean[i] = c.img_mean[i];
    info.std[i] = c.img_std[i];
  }
  info.is_metric = name_is_metric(c) || is_nested(model.ctx.get());
  info.has_aux_ray_head = e.has_aux();
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, e.device()) == cudaSuccess) info.device_name = prop.name;
  info.gpu_active = true;
  if (is_nested(model.ctx.get())) {
    info.kind = ModelKind::da3_nested;
    info.has_camera_pose = true;
  } else if (c.is_da2()) info.kind = c.head_max_depth > 0.f ? ModelKind::da2_metric : ModelKind::da2_relative;
  else if (is_mono(e)) info.kind = ModelKind::da3_mono;
  else {
    info.kind = ModelKind::da3;
    info.has_camera_pose = true;
  }
  return info;
}

bool infer(Model& model, const Image& image, Result& result, const InferOptions& options) {
  result = {};
  if (!model.ctx || !model.ctx->engine) return false;
  if (image.width <= 0 || image.height <= 0 ||
      image.data.size() != static_cast<size_t>(image.width) * image.height * 3)
    return false;
  da_ctx* c = model.ctx.get();
  const da3b::Engine& e = *c->engine;
  if (is_nested(c)) {
    // src/api.cpp:123-129: both branches + alignment; options do not apply
    int H = 0, W = 0;
    if (!run_nested(c, image.data.data(), image.width, image.height, result.depth, result.extrinsics.data(),
                    result.intrinsics.data(), &H, &W)) {
      DA_LOG("infer: %s", c->last_error.c_str());
      result = {};
      return false;
    }
    result.height = H;
    result.width = W;
    result.is_metric = true;
    result.has_pose = true;
    return !result.depth.empty();
  }
  // src/api.cpp:130-158: the ray solver only with with_pose, never with legacy_resize,
  // and only for DA3 models with the aux ray head
  if (options.ray_pose && (!options.with_pose || options.legacy_resize || e.config().is_da2() || is_mono(e) ||
                           !e.has_aux()))
    return false;
  if (options.with_pose && !options.ray_pose && (e.config().is_da2() || is_mono(e) || !e.has_camera())) return false;
  // DA2 and mono always use preprocess_real (src/engine.cpp:105-130); DA3 uses it
  // unless legacy_resize (src/api.cpp:151-157).
  const bool mono = is_mono(e);
  const bool legacy = !e.config().is_da2() && !mono && options.legacy_resize;
  int H = 0, W = 0;
  if (!run_one(c, image.data.data(), image.width, image.height, legacy, result.depth, &result.confidence, &H, &W,
               options.ray_pose) ||
      (mono && !fetch_sky(c, *c->engine, result.depth.size(), result.sky))) {
    DA_LOG("infer: %s", c->last_error.c_str());
    result = {};
    return false;
  }
  result.height = H;
  result.width = W;
  result.is_metric = model_info(model).is_metric;
  if (options.ray_pose) {
    // Engine::depth_pose_rays_native (src/engine.cpp:296-328): the solver on this
    // forward's ray field; camera-to-world extrinsics
    int nv = 0, rh = 0, rw = 0;
    const float* rays = c->engine->last_rays(&nv, &rh, &rw);
    if (!c->raysolver) c->raysolver.reset(new da3b::RaySolver());
    da3b::RayPoseResult rp;
    std::string err;
    const int rc = rays ? c->raysolver->solve(rays, nv, 0, rh, rw, H, W, c->stream, &rp, &err) : -1;
    if (rc != 0) {
      DA_LOG("infer: ray->pose solver failed (%d) %s", rc, err.c_str());
      result = {};
      return false;
    }
    memcpy(result.extrinsics.data(), rp.ext, sizeof(rp.ext));
    memcpy(result.intrinsics.data(), rp.intr, sizeof(rp.intr));
    result.has_pose = true;
  } else if (options.with_pose) {
    // CamPose::pose on this forward's camera token (src/api.cpp:136-150, src/engine.cpp:271-286)
    std::vector<float> pe;
    if (c->engine->poses(pe, c->stream) != 0) {
      DA_LOG("infer: camera pose failed: %s", c->engine->last_error().c_str());
      result = {};
      return false;
    }
    da3b::pose_to_ext_intr(pe.data(), H, W, result.extrinsics.data(), result.intrinsics.data());
    result.has_pose = true;
  }
  return !result.depth.empty();
}

bool infer_file(Model& model, const std::string& image_path, Result& result, const InferOptions& options) {
  Image img;
  std::string err;
  if (!read_ppm(image_path.c_str(), &img.width, &img.height, img.data, &err)) {
    DA_LOG("infer_file: %s", err.c_str());
    result = {};
    return false;
  }
  return infer(model, img, result, options);
}

// src/api.cpp:178-193: DA3 (not DA2, mono or nested) only; the caller fills the device
// buffer of the normalised planar f32 image [3][height][width] synchronously inside the
// callback; depth (+ confidence) at that size.
bool infer_preprocessed(Model& model, int height, int width, const UploadCallback& upload, Result& result) {
  result = {};
  if (!model.ctx || !model.ctx->engine || !upload || height <= 0 || width <= 0) return false;
  da_ctx* c = model.ctx.get();
  da3b::Engine& e = *c->engine;
  if (is_nested(c) || e.config().is_da2() || is_mono(e)) return false;
  size_t bytes = 0;
  float* dst = e.prepared_input(1, 1, height, width, &bytes);
  if (!dst) {
    DA_LOG("infer_preprocessed: %s", e.last_error().c_str());
    return false;
  }
  upload(UploadTarget{dst, bytes, true});
  result.depth.resize(static_cast<size_t>(height) * width);
  const bool want_conf = e.output_dim() >= 2;
  if (want_conf) result.confidence.resize(result.depth.size());
  cudaSetDevice(e.device());
  const int rc = e.run_prepared(1, 1, height, width, result.depth.data(),
                                want_conf ? result.confidence.data() : nullptr, c->stream);
  if (rc != 0 || cudaStreamSynchronize(c->stream) != cudaSuccess || e.status() != 0) {
    DA_LOG("infer_preprocessed: forward failed: %s", e.last_error().c_str());
    result = {};
    return false;
  }
  result.height = height;
  result.width = width;
  result.is_metric = model_info(model).is_metric;
  return true;
}

bool infer_batch(Model& model, const std::vector<Image>& images, std::vector<Result>& results) {
  results.clear();
  if (!model.ctx || !model.ctx->engine || images.empty()) return false;
  da_ctx* c = model.ctx.get();
  da3b::Engine& e = *c->engine;
  if (is_nested(c)) return false;
  const int w = images[0].width, h = images[0].height, n = static_cast<int>(images.size());
  std::vector<uint8_t> rgb(static_cast<size_t>(n) * w * h * 3);
  for (int i = 0; i < n; ++i) {
    if (images[i].width != w || images[i].height != h ||
        images[i].data.size() != static_cast<size_t>(w) * h * 3)
      return false;
    memcpy(&rgb[static_cast<size_t>(i) * w * h * 3], images[i].data.data(), images[i].data.size());
  }
  const size_t HW = static_cast<size_t>(w) * h;
  std::vector<float> depth(n * HW), conf(e.output_dim() >= 2 ? n * HW : 0);
  if (da3b_infer_host(c, rgb.data(), n, 1, h, w, depth.data(), conf.empty() ? nullptr : conf.data(), nullptr) != 0) {
    DA_LOG("infer_batch: %s", c->last_error.c_str());
    return false;
  }
  std::vector<float> sky;
  if (e.has_sky() && !fetch_sky(c, e, depth.size(), sky)) return false;
  const bool metric = model_info(model).is_metric;
  results.resize(n);
  for (int i = 0; i < n; ++i) {
    Result& r = results[i];
    r.width = w;
    r.height = h;
    r.is_metric = metric;
    r.depth.assign(depth.begin() + i * HW, depth.begin() + (i + 1) * HW);
    if (!conf.empty()) r.confidence.assign(conf.begin() + i * HW, conf.begin() + (i + 1) * HW);
    if (!sky.empty()) r.sky.assign(sky.begin() + i * HW, sky.begin() + (i + 1) * HW);
  }
  return true;
}

}  // namespace da3

// ====================================================================== C ABI
extern "C" {

DA_CAPI int da_capi_abi_version(void) { return 4; }

DA_CAPI da_ctx* da_capi_load(const char* path, int n_threads) {
  (void)n_threads;
  std::string err;
  da_ctx* c = make_ctx(path, default_device(), &err);
  if (!c) DA_LOG("da_capi_load: %s", err.c_str());
  return c;
}

DA_CAPI da_ctx* da_capi_load_nested(const char* anyview, const char* metric, int n_threads) {
  (void)n_threads;
  if (!anyview || !metric) return nullptr;
  std::string err;
  const int dev = default_device();
  da_ctx* c = make_ctx(anyview, dev, &err);
  if (!c) {
    DA_LOG("da_capi_load_nested: anyview: %s", err.c_str());
    return nullptr;
  }
  c->metric = da3b::Engine::create(metric, dev, &err);
  if (!c->metric) {
    DA_LOG("da_capi_load_nested: metric: %s", err.c_str());
    delete c;
    return nullptr;
  }
  if (!c->metric->has_sky() || c->engine->config().is_da2() || !c->engine->has_camera() ||
      c->engine->output_dim() < 2) {
    DA_LOG("da_capi_load_nested: needs a DA3 anyview model with camera decoder and confidence, and a metric "
           "model with a sky head");
    delete c;
    return nullptr;
  }
  return c;
}

DA_CAPI void da_capi_free(da_ctx* c) { delete c; }

DA_CAPI char* da_capi_info_json(da_ctx* c) {
  if (!c || !c->engine) return nullptr;
  const da3b::Config& cfg = c->engine->config();
  std::string name;
  for (char ch : cfg.checkpoint_name) {
    if (ch == '"' || ch == '\\') name += '\\';
    if (static_cast<unsigned char>(ch) >= 0x20) name += ch;
  }
  const std::string j = "{\"checkpoint\":\"" + name + "\",\"embed_dim\":" + std::to_string(cfg.embed_dim) +
                        ",\"depth\":" + std::to_string(cfg.depth) + ",\"num_heads\":" + std::to_string(cfg.num_heads) +
                        ",\"tensorrt_enabled\":false,\"tensorrt_active\":false}";
  char* p = static_cast<char*>(malloc(j.size() + 1));
  if (p) memcpy(p, j.c_str(), j.size() + 1);
  return p;
}

DA_CAPI void da_capi_free_string(char* s) { free(s); }
DA_CAPI const char* da_capi_last_error(da_ctx* c) { return c ? c->last_error.c_str() : ""; }
DA_CAPI void da_capi_free_floats(float* p) { free(p); }
DA_CAPI void da_capi_free_bytes(unsigned char* p) { free(p); }

// src/da_capi.cpp:97-117: nested -> both branches + alignment; DA2 -> depth_relative
// (preprocess_real); DA3 -> depth (legacy floor-to-patch preprocess).
DA_CAPI float* da_capi_depth_path(da_ctx* c, const char* image_path, int* out_h, int* out_w) {
  if (!c || !c->engine || !image_path) {
    if (c) c->last_error = "depth: bad args";
    return nullptr;
  }
  int w = 0, h = 0;
  std::vector<uint8_t> rgb;
  if (!read_ppm(image_path, &w, &h, rgb, &c->last_error)) return nullptr;
  std::vector<float> depth;
  int H = 0, W = 0;
  const bool legacy = !c->engine->config().is_da2();
  if (is_nested(c)) {
    float ext[12], intr[9];
    if (!run_nested(c, rgb.data(), w, h, depth, ext, intr, &H, &W)) return nullptr;
  } else if (!run_one(c, rgb.data(), w, h, legacy, depth, nullptr, &H, &W)) {
    return nullptr;
  }
  float* p = static_cast<float*>(malloc(depth.size() * sizeof(float)));
  if (!p) {
    c->last_error = "depth: oom";
    return nullptr;
  }
  memcpy(p, depth.data(), depth.size() * sizeof(float));
  if (out_h) *out_h = H;
  if (out_w) *out_w = W;
  return p;
}

// src/da_capi.cpp:119-129: legacy preprocess, one view, camera-token pose.
DA_CAPI int da_capi_pose_path(da_ctx* c, const char* image_path, float out_ext[12], float out_intr[9]) {
  if (!c || !c->engine || !image_path) {
    if (c) c->last_error = "pose: bad args";
    return -1;
  }
  if (c->engine->config().is_da2() || !c->engine->has_camera()) {
    c->last_error = "pose: this model has no camera pose";
    return -1;
  }
  int w = 0, h = 0;
  std::vector<uint8_t> rgb;
  if (!read_ppm(image_path, &w, &h, rgb, &c->last_error)) return -1;
  std::vector<float> depth, conf, pe;
  int H = 0, W = 0;
  if (is_nested(c)) {
    // src/da_capi.cpp:123-124: the nested pose is the anyview pose, translation scaled
    float ext[12], intr[9];
    if (!run_nested(c, rgb.data(), w, h, depth, ext, intr, &H, &W)) return -1;
    if (out_ext) memcpy(out_ext, ext, sizeof(ext));
    if (out_intr) memcpy(out_intr, intr, sizeof(intr));
    return 0;
  }
  if (!run_one(c, rgb.data(), w, h, true, depth, &conf, &H, &W)) return -1;
  if (c->engine->poses(pe, c->stream) != 0) {
    c->last_error = "pose: " + c->engine->last_error();
    return -1;
  }
  float ext[12], intr[9];
  da3b::pose_to_ext_intr(pe.data(), H, W, ext, intr);
  if (out_ext) memcpy(out_ext, ext, sizeof(ext));
  if (out_intr) memcpy(out_intr, intr, sizeof(intr));
  return 0;
}

// src/da_capi.cpp:130-155: legacy preprocess, one backbone pass over all views.
DA_CAPI float* da_capi_depth_pose_multi(da_ctx* c, const char** paths, int n, int* out_h, int* out_w, int* out_n,
                                        float* out_ext, float* out_intr) {
  if (!c || !c->engine || !paths || n <= 0) {
    if (c) c->last_error = "depth_multi: bad args";
    return nullptr;
  }
  int w0 = 0, h0 = 0;
  std::vector<uint8_t> all;
  for (int i = 0; i < n; ++i) {
    int w = 0, h = 0;
    std::vector<uint8_t> rgb;
    if (!paths[i] || !read_ppm(paths[i], &w, &h, rgb, &c->last_error)) return nullptr;
    if (i == 0) { w0 = w; h0 = h; }
    else if (w != w0 || h != h0) { c->last_error = "depth_multi: views differ in H,W"; return nullptr; }
    all.insert(all.end(), rgb.begin(), rgb.end());
  }
  int W = 0, H = 0;
  processed_size(c->engine->config(), w0, h0, true, &W, &H);
  float* p = nullptr;
  if (W != w0 || H != h0) {
    std::vector<float> d;
    if (!run_legacy(c, all.data(), n, n, w0, h0, d, nullptr, &H, &W)) return nullptr;
    p = static_cast<float*>(malloc(d.size() * sizeof(float)));
    if (!p) { c->last_error = "depth_multi: oom"; return nullptr; }
    memcpy(p, d.data(), d.size() * sizeof(float));
  } else {
    const size_t per = static_cast<size_t>(H) * W;
    p = static_cast<float*>(malloc(static_cast<size_t>(n) * per * sizeof(float)));
    if (!p) { c->last_error = "depth_multi: oom"; return nullptr; }
    if (da3b_infer_host(c, all.data(), n, n, H, W, p, nullptr, nullptr) != 0) {
      free(p);
      return nullptr;
    }
  }
  if (out_ext || out_intr) {
    // CamPose::pose per view (src/engine.cpp:372-381), original view order
    std::vector<float> pe;
    if (!c->engine->has_camera() || c->engine->poses(pe, c->stream) != 0) {
      c->last_error = "depth_multi: camera pose failed: " + c->engine->last_error();
      free(p);
      return nullptr;
    }
    for (int i = 0; i < n; ++i) {
      float ext[12], intr[9];
      da3b::pose_to_ext_intr(&pe[static_cast<size_t>(i) * 9], H, W, ext, intr);
      if (out_ext) memcpy(out_ext + static_cast<size_t>(i) * 12, ext, sizeof(ext));
      if (out_intr) memcpy(out_intr + static_cast<size_t>(i) * 9, intr, sizeof(intr));
    }
  }
  if (out_h) *out_h = H;
  if (out_w) *out_w = W;
  if (out_n) *out_n = n;
  return p;
}

// src/da_capi.cpp:202-285: nested -> aligned depth and pose (no conf / sky); DA2 ->
// depth only; mono -> depth and sky; DA3 -> depth, confidence and camera pose. Every
// path but nested uses preprocess_real.
DA_CAPI int da_capi_depth_dense(da_ctx* c, const char* image_path, int* out_h, int* out_w, float** out_depth,
                                float** out_conf, float** out_sky, float out_ext[12], float out_intr[9],
                                int* out_is_metric) {
  if (!c || !c->engine || !image_path) {
    if (c) c->last_error = "depth_dense: bad args";
    return -1;
  }
  if (out_depth) *out_depth = nullptr;
  if (out_conf) *out_conf = nullptr;
  if (out_sky) *out_sky = nullptr;
  if (out_ext) memset(out_ext, 0, 12 * sizeof(float));
  if (out_intr) memset(out_intr, 0, 9 * sizeof(float));
  int w = 0, h = 0;
  std::vector<uint8_t> rgb;
  if (!read_ppm(image_path, &w, &h, rgb, &c->last_error)) return -1;
  da3b::Engine& e = *c->engine;
  std::vector<float> depth, second;
  float ext[12] = {0}, intr[9] = {0};
  bool has_pose = false;
  int H = 0, W = 0;
  int metric = name_is_metric(e.config()) ? 1 : 0;
  if (is_nested(c)) {
    if (!run_nested(c, rgb.data(), w, h, depth, ext, intr, &H, &W)) return -1;
    has_pose = true;
    metric = 1;
  } else {
    const bool mono = is_mono(e);
    if (!run_one(c, rgb.data(), w, h, false, depth, mono ? nullptr : &second, &H, &W)) return -1;
    if (e.config().is_da2()) {
      second.clear();
      metric = e.config().head_max_depth > 0.f ? 1 : 0;
    } else if (mono) {
      if (!fetch_sky(c, e, depth.size(), second)) return -1;
    } else {
      std::vector<float> pe;
      if (!e.has_camera() || e.poses(pe, c->stream) != 0) {
        c->last_error = "depth_dense: depth+pose failed: " + e.last_error();
        return -1;
      }
      da3b::pose_to_ext_intr(pe.data(), H, W, ext, intr);
      has_pose = true;
    }
    if (!mono && second.size() != depth.size()) second.clear();
    if (mono) {
      if (out_sky && !second.empty()) {
        *out_sky = static_cast<float*>(malloc(second.size() * sizeof(float)));
        if (!*out_sky) { c->last_error = "depth_dense: oom"; return -1; }
        memcpy(*out_sky, second.data(), second.size() * sizeof(float));
      }
    } else if (out_conf && !second.empty()) {
      *out_conf = static_cast<float*>(malloc(second.size() * sizeof(float)));
      if (!*out_conf) { c->last_error = "depth_dense: oom"; return -1; }
      memcpy(*out_conf, second.data(), second.size() * sizeof(float));
    }
  }
  if (out_depth) {
    *out_depth = static_cast<float*>(malloc(depth.size() * sizeof(float)));
    if (!*out_depth) {
      if (out_conf && *out_conf) { free(*out_conf); *out_conf = nullptr; }
      if (out_sky && *out_sky) { free(*out_sky); *out_sky = nullptr; }
      c->last_error = "depth_dense: oom";
      return -1;
    }
    memcpy(*out_depth, depth.data(), depth.size() * sizeof(float));
  }
  if (has_pose) {
    if (out_ext) memcpy(out_ext, ext, sizeof(ext));
    if (out_intr) memcpy(out_intr, intr, sizeof(intr));
  }
  if (out_h) *out_h = H;
  if (out_w) *out_w = W;
  if (out_is_metric) *out_is_metric = metric;
  return 0;
}

DA_CAPI int da_capi_points(da_ctx* c, const char*, float, int*, float**, unsigned char**) {
  if (c) c->last_error = "points: point clouds are outside the depth path of this library";
  return -1;
}
DA_CAPI int da_capi_export_glb(da_ctx* c, const char*, const char*) {
  if (c) c->last_error = "export_glb: exporters are outside the depth path of this library";
  return -1;
}
DA_CAPI int da_capi_export_colmap(da_ctx* c, const char*, const char*, int) {
  if (c) c->last_error = "export_colmap: exporters are outside the depth path of this library";
  return -1;
}

// ---------------------------------------------------------------------- da3b_*
DA3B_API da_ctx* da3b_load(const char* gguf_path, int device) {
  std::string err;
  da_ctx* c = make_ctx(gguf_path, device, &err);
  if (!c) DA_LOG("da3b_load: %s", err.c_str());
  return c;
}

DA3B_API int da3b_processed_size(da_ctx* c, int w, int h, int legacy, int* out_h, int* out_w, int* needs_resize) {
  if (!c || !c->engine || w <= 0 || h <= 0) return -1;
  int W = 0, H = 0;
  processed_size(c->engine->config(), w, h, legacy != 0, &W, &H);
  if (out_h) *out_h = H;
  if (out_w) *out_w = W;
  if (needs_resize) *needs_resize = (W != w || H != h) ? 1 : 0;
  return 0;
}

DA3B_API int da3b_infer_device(da_ctx* c, const void* rgb_dev, int n_views, int views_per_scene, int h, int w,
                               void* depth_dev, void* conf_dev, void* rays_dev, void* stream) {
  if (!c || !c->engine || !rgb_dev || !depth_dev) return -1;
  cudaSetDevice(c->engine->device());
  const int rc = c->engine->run(static_cast<const uint8_t*>(rgb_dev), n_views, views_per_scene, h, w,
                                static_cast<float*>(depth_dev), static_cast<float*>(conf_dev),
                                static_cast<float*>(rays_dev), static_cast<cudaStream_t>(stream));
  if (rc) c->last_error = c->engine->last_error();
  return rc;
}

DA3B_API int da3b_last_pose(da_ctx* c, int n_views, float* pose_enc, float* ext, float* intr) {
  if (!c || !c->engine || n_views <= 0) return -1;
  std::vector<float> pe;
  const int rc = c->engine->poses(pe, c->stream);
  if (rc) {
    c->last_error = c->engine->last_error();
    return rc - 10;
  }
  if (static_cast<int>(pe.size()) != n_views * 9) {
    c->last_error = "last_pose: the last run had " + std::to_string(pe.size() / 9) + " views";
    return -2;
  }
  int H = 0, W = 0;
  c->engine->last_size(&H, &W);
  for (int v = 0; v < n_views; ++v) {
    if (pose_enc) memcpy(pose_enc + v * 9, &pe[static_cast<size_t>(v) * 9], 9 * sizeof(float));
    float e[12], k[9];
    da3b::pose_to_ext_intr(&pe[static_cast<size_t>(v) * 9], H, W, e, k);
    if (ext) memcpy(ext + v * 12, e, sizeof(e));
    if (intr) memcpy(intr + v * 9, k, sizeof(k));
  }
  return 0;
}

DA3B_API int da3b_ray_pose(da_ctx* c, const float* rays_dev, int n_views, int view, int ray_h, int ray_w, int img_h,
                           int img_w, float* ext, float* intr, double* diag, void* stream) {
  if (!c || !c->engine || !rays_dev || !ext || !intr) return -1;
  cudaSetDevice(c->engine->device());
  if (!c->raysolver) c->raysolver.reset(new da3b::RaySolver());
  da3b::RayPoseResult r;
  std::string err;
  const int rc = c->raysolver->solve(rays_dev, n_views, view, ray_h, ray_w, img_h, img_w,
                                     stream ? static_cast<cudaStream_t>(stream) : c->stream, &r, &err);
  if (rc < 0) {
    c->last_error = err;
    return rc;
  }
  if (rc > 0) {
    c->last_error = "ray pose: degenerate ray field";
    return rc;
  }
  memcpy(ext, r.ext, sizeof(r.ext));
  memcpy(intr, r.intr, sizeof(r.intr));
  if (diag) {
    memcpy(diag, r.R, 9 * sizeof(double));
    memcpy(diag + 9, r.T, 3 * sizeof(double));
    diag[12] = r.focal[0];
    diag[13] = r.focal[1];
    diag[14] = r.pp[0];
    diag[15] = r.pp[1];
    memcpy(diag + 16, r.A, 9 * sizeof(double));
    diag[25] = r.n_inlier_best;
  }
  return 0;
}

DA3B_API int da3b_last_sky(da_ctx* c, int n_views, float* sky) {
  if (!c || !c->engine || !sky || n_views <= 0) return -1;
  da3b::Engine& e = *c->engine;
  int H = 0, W = 0;
  e.last_size(&H, &W);
  const size_t n = static_cast<size_t>(n_views) * H * W;
  if (e.sky(sky, n, c->stream) != 0 || cudaStreamSynchronize(c->stream) != cudaSuccess) {
    c->last_error = "last_sky: " + e.last_error();
    return -2;
  }
  return 0;
}

DA3B_API float da3b_nested_align(const float* any_depth, const float* any_conf, const float* any_ext,
                                 const float* any_intr, float* metric_depth, const float* sky, int64_t n,
                                 float* out_depth, float* out_ext) {
  if (!any_depth || !any_conf || !any_ext || !any_intr || !metric_depth || !sky || !out_depth || !out_ext || n < 0)
    return -1.0f;
  da3b::mono_sky_fill(metric_depth, sky, static_cast<size_t>(n));
  return da3b::nested_align(any_depth, any_conf, any_ext, any_intr, metric_depth, sky, static_cast<size_t>(n),
                            out_depth, out_ext);
}

DA3B_API int da3b_infer_prepared(da_ctx* c, const float* chw, int n_views, int h, int w, float* depth, float* conf,
                                 void* stream) {
  if (!c || !c->engine || !chw || !depth || n_views <= 0 || h <= 0 || w <= 0) return -1;
  da3b::Engine& e = *c->engine;
  size_t bytes = 0;
  float* dst = e.prepared_input(n_views, 1, h, w, &bytes);
  if (!dst) {
    c->last_error = e.last_error();
    return -2;
  }
  cudaStream_t s = stream ? static_cast<cudaStream_t>(stream) : c->stream;
  if (cudaMemcpyAsync(dst, chw, bytes, cudaMemcpyDefault, s) != cudaSuccess) return -3;
  const int rc = e.run_prepared(n_views, 1, h, w, depth, conf, s);
  if (rc) {
    c->last_error = e.last_error();
    return rc;
  }
  return 0;
}

DA3B_API int da3b_infer_host(da_ctx* c, const void* rgb_host, int n_views, int views_per_scene, int h, int w,
                             float* depth_host, float* conf_host, float* rays_host) {
  if (!c || !c->engine || !rgb_host || !depth_host) return -1;
  cudaSetDevice(c->engine->device());
  int rc = c->engine->run(static_cast<const uint8_t*>(rgb_host), n_views, views_per_scene, h, w, depth_host,
                          conf_host, rays_host, c->stream);
  if (rc) {
    c->last_error = c->engine->last_error();
    return rc;
  }
  if (cudaStreamSynchronize(c->stream) != cudaSuccess) {
    c->last_error = std::string("CUDA error: ") + cudaGetErrorString(cudaGetLastError());
    return -20;
  }
  const int st = c->engine->status();
  if (st != 0) {
    c->last_error = "device status " + std::to_string(st) + " (a bounded wait timed out)";
    return -21;
  }
  return 0;
}

DA3B_API int da3b_ref_views(da_ctx* c, int* out, int n) {
  if (!c || !c->engine || !out) return -1;
  const std::vector<int> v = c->engine->last_ref_views(c->stream);
  for (int i = 0; i < n && i < static_cast<int>(v.size()); ++i) out[i] = v[i];
  return static_cast<int>(v.size());
}

DA3B_API int da3b_launches(da_ctx* c, int n_views, int views_per_scene, int h, int w, int rays) {
  if (!c || !c->engine) return -1;
  return c->engine->launches(n_views, views_per_scene, h, w, rays != 0);
}

DA3B_API int da3b_debug_feature(da_ctx* c, int layer, void* out, size_t capacity, int* rows, int* cols) {
  if (!c || !c->engine || !out) return -1;
  int r = 0, k = 0;
  const __half* p = c->engine->debug_feat(layer, &r, &k);
  if (!p) return -2;
  if (rows) *rows = r;
  if (cols) *cols = k;
  const size_t n = static_cast<size_t>(r) * k;
  if (n > capacity) return -3;
  cudaSetDevice(c->engine->device());
  cudaStreamSynchronize(c->stream);
  return cudaMemcpy(out, p, n * 2, cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -4;
}

DA3B_API int da3b_set_capture_residuals(da_ctx* c, int on) {
  if (!c || !c->engine) return -1;
  c->engine->set_capture_residuals(on != 0);
  return 0;
}

DA3B_API int da3b_debug_residual(da_ctx* c, int layer, float* out, size_t capacity, int* rows, int* cols) {
  if (!c || !c->engine || !out) return -1;
  int r = 0, k = 0;
  const float* p = c->engine->debug_resid(layer, &r, &k);
  if (!p) return -2;
  if (rows) *rows = r;
  if (cols) *cols = k;
  const size_t n = static_cast<size_t>(r) * k;
  if (n > capacity) return -3;
  cudaSetDevice(c->engine->device());
  cudaStreamSynchronize(c->stream);
  return cudaMemcpy(out, p, n * sizeof(float), cudaMemcpyDeviceToHost) == cudaSuccess ? 0 : -4;
}

DA3B_API int da3b_set_graphs(da_ctx* c, int on) {
  if (!c || !c->engine) return -1;
  c->engine->set_use_graph(on != 0);
  return 0;
}

DA3B_API int da3b_set_act_quant(da_ctx* c, int on) {
  if (!c || !c->engine) return -1;
  c->engine->set_act_quant(on != 0);
  return 0;
}

DA3B_API int da3b_set_raw_logits(da_ctx* c, int on) {
  if (!c || !c->engine) return -1;
  c->engine->set_raw_logits(on != 0);
  return 0;
}

DA3B_API int da3b_model_dims(da_ctx* c, int* out) {
  if (!c || !c->engine || !out) return -1;
  const da3b::Config& cfg = c->engine->config();
  out[0] = cfg.embed_dim;
  out[1] = cfg.depth;
  out[2] = cfg.num_heads;
  out[3] = cfg.patch_size;
  out[4] = cfg.cat_token ? 1 : 0;
  out[5] = c->engine->output_dim();
  out[6] = c->engine->has_aux() ? 1 : 0;
  out[7] = cfg.is_da2() ? 1 : 0;
  out[8] = c->engine->has_sky() ? 1 : 0;
  out[9] = c->engine->has_camera() ? 1 : 0;
  return 0;
}

}  // extern "C"
