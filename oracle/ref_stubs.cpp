// Aborting definitions of the ggml functions and DA3cpplib graph builders that the
// reference's src/dino_backbone.cpp and src/rope2d.cpp refer to, so that those two files
// compile unmodified into oracle/_ref (test infrastructure only, never part of libda3b).
// The checker calls only their host-side functions (build_rope_tables,
// DinoBackbone::interp_pos_embed, DinoBackbone::select_reference_view_saddle), which
// build no ggml graph; reaching any function here is a checker bug, so each one aborts.
#include <cstdio>
#include <cstdlib>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "backend.hpp"
#include "vit_block.hpp"

namespace {
[[noreturn]] void unreachable(const char* what) {
  std::fprintf(stderr, "oracle/_ref: %s is not available in the checker build (no ggml)\n", what);
  std::abort();
}
}  // namespace

ggml_tensor* ggml_cont(ggml_context*, ggml_tensor*) { unreachable("ggml_cont"); }
ggml_tensor* ggml_concat(ggml_context*, ggml_tensor*, ggml_tensor*, int) { unreachable("ggml_concat"); }
ggml_tensor* ggml_add(ggml_context*, ggml_tensor*, ggml_tensor*) { unreachable("ggml_add"); }
ggml_tensor* ggml_mul(ggml_context*, ggml_tensor*, ggml_tensor*) { unreachable("ggml_mul"); }
ggml_tensor* ggml_neg(ggml_context*, ggml_tensor*) { unreachable("ggml_neg"); }
ggml_tensor* ggml_norm(ggml_context*, ggml_tensor*, float) { unreachable("ggml_norm"); }
ggml_tensor* ggml_mul_mat(ggml_context*, ggml_tensor*, ggml_tensor*) { unreachable("ggml_mul_mat"); }
ggml_tensor* ggml_gelu_erf(ggml_context*, ggml_tensor*) { unreachable("ggml_gelu_erf"); }
ggml_tensor* ggml_silu(ggml_context*, ggml_tensor*) { unreachable("ggml_silu"); }
ggml_tensor* ggml_transpose(ggml_context*, ggml_tensor*) { unreachable("ggml_transpose"); }
ggml_tensor* ggml_cpy(ggml_context*, ggml_tensor*, ggml_tensor*) { unreachable("ggml_cpy"); }
ggml_tensor* ggml_reshape_2d(ggml_context*, ggml_tensor*, int64_t, int64_t) { unreachable("ggml_reshape_2d"); }
ggml_tensor* ggml_reshape_3d(ggml_context*, ggml_tensor*, int64_t, int64_t, int64_t) {
  unreachable("ggml_reshape_3d");
}
ggml_tensor* ggml_view_2d(ggml_context*, ggml_tensor*, int64_t, int64_t, size_t, size_t) {
  unreachable("ggml_view_2d");
}
ggml_tensor* ggml_view_3d(ggml_context*, ggml_tensor*, int64_t, int64_t, int64_t, size_t, size_t, size_t) {
  unreachable("ggml_view_3d");
}
ggml_tensor* ggml_conv_2d(ggml_context*, ggml_tensor*, ggml_tensor*, int, int, int, int, int, int) {
  unreachable("ggml_conv_2d");
}
void ggml_build_forward_expand(ggml_cgraph*, ggml_tensor*) { unreachable("ggml_build_forward_expand"); }
bool ggml_backend_buffer_is_host(ggml_backend_buffer_t) { unreachable("ggml_backend_buffer_is_host"); }
void ggml_backend_tensor_set(ggml_tensor*, const void*, size_t, size_t) { unreachable("ggml_backend_tensor_set"); }

namespace da {
// Backend: constructible (the backbone object holds a reference to one), nothing else.
struct Backend::Impl {};
Backend::Backend() {}
Backend::~Backend() {}
ggml_tensor* Backend::add_graph_input_nd(ggml_context*, GraphInputPool&, const float*, const int64_t*, int) {
  unreachable("Backend::add_graph_input_nd");
}
ggml_tensor* Backend::add_graph_input_nd_upload(ggml_context*, const int64_t*, int,
                                                std::function<void(ggml_tensor*)>) {
  unreachable("Backend::add_graph_input_nd_upload");
}
void Backend::capture(ggml_tensor*, std::vector<float>*) { unreachable("Backend::capture"); }
bool Backend::compute(const std::function<ggml_tensor*(ggml_context*)>&, std::vector<float>&) {
  unreachable("Backend::compute");
}
bool Backend::forward_capture(const std::function<ggml_tensor*(ggml_context*)>&, std::vector<float>&) {
  unreachable("Backend::forward_capture");
}
BlockWeights load_block(const ModelLoader&, int) { unreachable("load_block"); }
ggml_tensor* vit_block(ggml_context*, ggml_tensor*, const BlockWeights&, int, int, float, ggml_tensor*, ggml_tensor*) {
  unreachable("vit_block");
}
}  // namespace da
