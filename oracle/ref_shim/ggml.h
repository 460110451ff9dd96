// Declarations of the ggml names that DA3cpplib's sources mention, so that its host-
// only code compiles for the oracle/_ref checker. The reference's ggml submodule is
// absent from its checkout, so no ggml code exists here: every ggml function declared
// below is defined in oracle/ref_stubs.cpp with a body that aborts. The reference
// functions the checker calls (preprocessing, UV embedding, nested alignment, the ray
// solver, RoPE tables, pos-embed interpolation, reference-view selection) never reach
// them. The struct layouts are this checker's own: nothing built here exchanges them
// with a real ggml.
#pragma once
#include <cstddef>
#include <cstdint>

struct ggml_context;
struct ggml_cgraph;
struct ggml_backend_buffer;
typedef struct ggml_backend_buffer* ggml_backend_buffer_t;

enum ggml_type { GGML_TYPE_F32 = 0, GGML_TYPE_F16 = 1, GGML_TYPE_Q8_0 = 8, GGML_TYPE_I32 = 26 };

#define GGML_MAX_DIMS 4

struct ggml_tensor {
  enum ggml_type type;
  struct ggml_backend_buffer* buffer;
  int64_t ne[GGML_MAX_DIMS];
  size_t nb[GGML_MAX_DIMS];
  void* data;
  char name[64];
};

ggml_tensor* ggml_cont(ggml_context* ctx, ggml_tensor* a);
ggml_tensor* ggml_concat(ggml_context* ctx, ggml_tensor* a, ggml_tensor* b, int dim);
ggml_tensor* ggml_add(ggml_context* ctx, ggml_tensor* a, ggml_tensor* b);
ggml_tensor* ggml_mul(ggml_context* ctx, ggml_tensor* a, ggml_tensor* b);
ggml_tensor* ggml_neg(ggml_context* ctx, ggml_tensor* a);
ggml_tensor* ggml_norm(ggml_context* ctx, ggml_tensor* a, float eps);
ggml_tensor* ggml_mul_mat(ggml_context* ctx, ggml_tensor* a, ggml_tensor* b);
ggml_tensor* ggml_gelu_erf(ggml_context* ctx, ggml_tensor* a);
ggml_tensor* ggml_silu(ggml_context* ctx, ggml_tensor* a);
ggml_tensor* ggml_transpose(ggml_context* ctx, ggml_tensor* a);
ggml_tensor* ggml_cpy(ggml_context* ctx, ggml_tensor* a, ggml_tensor* b);
ggml_tensor* ggml_reshape_2d(ggml_context* ctx, ggml_tensor* a, int64_t ne0, int64_t ne1);
ggml_tensor* ggml_reshape_3d(ggml_context* ctx, ggml_tensor* a, int64_t ne0, int64_t ne1, int64_t ne2);
ggml_tensor* ggml_view_2d(ggml_context* ctx, ggml_tensor* a, int64_t ne0, int64_t ne1, size_t nb1, size_t offset);
ggml_tensor* ggml_view_3d(ggml_context* ctx, ggml_tensor* a, int64_t ne0, int64_t ne1, int64_t ne2, size_t nb1,
                          size_t nb2, size_t offset);
ggml_tensor* ggml_conv_2d(ggml_context* ctx, ggml_tensor* a, ggml_tensor* b, int s0, int s1, int p0, int p1, int d0,
                          int d1);
void ggml_build_forward_expand(ggml_cgraph* cgraph, ggml_tensor* tensor);
