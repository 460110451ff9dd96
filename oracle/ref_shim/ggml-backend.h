// Declarations only (see ggml.h in this folder); definitions abort (oracle/ref_stubs.cpp).
#pragma once
#include "ggml.h"
struct ggml_backend;
typedef struct ggml_backend* ggml_backend_t;
bool ggml_backend_buffer_is_host(ggml_backend_buffer_t buffer);
void ggml_backend_tensor_set(ggml_tensor* tensor, const void* data, size_t offset, size_t size);
