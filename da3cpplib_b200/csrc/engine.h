// Depth-path engine: one device model, per-shape plans (pre-allocated buffers,
// per-resolution tables, a captured CUDA graph), and the forward launch sequence.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <memory>
#include <string>
#include <tuple>
#include <vector>

#include "model.h"

namespace da3b {

struct Plan;

// Output activation family of the depth head (src/dpt_head.cpp:402-439, src/engine.cpp:218-225).
enum class HeadKind { Da2Relative, Da2Metric, Da3 };

class Engine {
 public:
  ~Engine();
  static std::unique_ptr<Engine> create(const std::string& gguf_path, int device, std::string* err);

  const Config& config() const { return model_->cfg; }
  const DeviceModel& model() const { return *model_; }
  int device() const { return device_; }
  HeadKind head_kind() const;
  bool has_aux() const { return model_->head.aux; }
  int output_dim() const { return model_->head.od; }

  // Depth inference of n_views RGB8 images [n_views][H][W][3] already on the device
  // (H, W multiples of the patch size). Views are grouped into scenes of
  // views_per_scene consecutive images that share global attention (1 = single
  // image). Outputs are f32 planes [n_views][H][W] (conf may be null; for DA2 it is
  // unused); rays (may be null) receives the aux ray head [7][n_views][8*gh][8*gw].
  // Returns 0, or a negative error code with last_error() set. Asynchronous on `s`
  // except on the first call for a shape (plan creation synchronises).
  int run(const uint8_t* rgb_dev, int n_views, int views_per_scene, int H, int W, float* depth_dev,
          float* conf_dev, float* rays_dev, cudaStream_t s);

  // The same forward with the aux ray head, whose output stays on the device:
  // last_rays() then gives its planes [7][n_views][8*gh][8*gw] (null without one).
  int run_with_rays(const uint8_t* rgb, int n_views, int views_per_scene, int H, int W, float* depth, float* conf,
                    cudaStream_t s);
  const float* last_rays(int* n_views, int* ray_h, int* ray_w) const;

  // Prepared-input runs (infer_preprocessed, src/api.cpp:178-193 / src/engine.cpp:230-270;
  // the legacy preprocess): device buffer for V normalised planar f32 images [V][3][H][W]
  // (scenes of S views) of the plan of that shape (allocated on first use; *bytes its
  // size), and the forward reading it.
  float* prepared_input(int V, int S, int H, int W, size_t* bytes);
  int run_prepared(int V, int S, int H, int W, float* depth, float* conf, cudaStream_t s);

  // Sky head (metric / mono DPT) of the last run: relu(sky logits) as f32 [n_views][H][W]
  // into dst (host or device; count must equal n_views * H * W), asynchronous on s.
  int sky(float* dst, size_t count, cudaStream_t s);
  bool has_sky() const { return model_->head.sky; }

  // Camera decoder on the last run's camera tokens: pose encodings [n_views][9]
  // ([t(3), quaternion xyzw (4), fov h/w (2)]) in the original view order.
  int poses(std::vector<float>& pe, cudaStream_t s);
  bool has_camera() const { return model_->camdec.present; }
  // Processed size of the last run (0 x 0 before any).
  void last_size(int* H, int* W) const;

  // Selected reference view per scene of the last run with views_per_scene >= 3 (host copy).
  std::vector<int> last_ref_views(cudaStream_t s);
  // Kernel launches of one forward of the given shape (after a run of that shape).
  int launches(int n_views, int views_per_scene, int H, int W, bool rays) const;
  // Device-side status word (0 = ok), read after a synchronisation.
  int status();
  const std::string& last_error() const { return err_; }
  void set_use_graph(bool on) { use_graph_ = on; }
  // true: the fused out2b epilogue writes raw logits (no output activation); used
  // by parity tests. Changing it drops the cached plans.
  void set_raw_logits(bool on);
  // true: activations entering a Q8_0 linear are rounded through Q8_0 as ggml
  // quantises them before its Q8_0 matmuls; false (default): plain f16 activations,
  // which sit closer to the reference's outputs (two independent Q8_0 roundings
  // disagree by more than one rounding does). Drops the cached plans.
  void set_act_quant(bool on);
  // true: every forward also copies the residual stream x after each ViT block into a
  // per-plan buffer [depth][M][D] f32 (parity tests of every layer). Drops the cached plans.
  void set_capture_residuals(bool on);

  // Debug captures for parity tests: feats of out-layer o ([n_views*Np][C] f16) of
  // the last run; returns nullptr if unavailable.
  const __half* debug_feat(int o, int* rows, int* cols) const;
  const float* debug_x(int* rows, int* cols) const;
  // Residual stream after block `layer` of the last run ([M][D] f32, views in processing
  // order), when residual capture is on; nullptr otherwise.
  const float* debug_resid(int layer, int* rows, int* cols) const;

 private:
  Engine() = default;
  Plan* plan_for(int n_views, int S, int H, int W, bool rays);
  Plan* checked_plan(int V, int S, int H, int W, bool rays, int* code);
  int launch(Plan* p, bool prepared, cudaStream_t s);
  int copy_out(Plan* p, float* depth, float* conf, float* rays, cudaStream_t s);
  int forward(Plan& p, cudaStream_t s);
  int backbone(Plan& p, cudaStream_t s);
  int head(Plan& p, cudaStream_t s);
  int pyramid(Plan& p, const void* fuse_weights, __half* u_out, cudaStream_t s, const cudaEvent_t* lateral_ready);

  std::unique_ptr<DeviceModel> model_;
  // f16 staging buffer of one ViT block's four linears (qkv | proj | fc1 | fc2), filled
  // from the resident Q8_0 bytes ahead of each block when the model keeps them quantised
  __half* wstage_ = nullptr;
  int device_ = 0;
  int* status_ = nullptr;
  bool use_graph_ = true;
  // $DA3B_Q8_TILES=1 at creation: resident Q8_0 block linears whose GEMMs all run on
  // one-CTA tiles are read by GEMMs that dequantise their weight tiles in shared memory
  // instead of through the f16 staging buffer (same bits; measured slower at batch 1)
  bool q8_tiles_ = false;
  // the DPT head's lateral branches 0-2 (projection -> resize -> layer_rn -> first RCU1
  // conv) run on these side streams; ev_[0] forks them from the forward's stream,
  // ev_[1 + r] marks branch r done
  cudaStream_t side_[3] = {nullptr, nullptr, nullptr};
  cudaEvent_t ev_[4] = {nullptr, nullptr, nullptr, nullptr};
  bool raw_logits_ = false;
  bool act_quant_ = false;
  bool capture_resid_ = false;
  std::string err_;
  std::map<std::tuple<int, int, int, int, bool>, std::unique_ptr<Plan>> plans_;
  Plan* last_ = nullptr;
  const float* last_x_ = nullptr;
  const __half* last_feat_[4] = {nullptr, nullptr, nullptr, nullptr};
};

}  // namespace da3b
