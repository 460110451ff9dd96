// Forward declarations only, so that DA3cpplib's model_loader.hpp parses when the
// reference's host-only sources (src/preprocess.cpp, src/uv_posembed.cpp) are compiled
// for the oracle/_ref checker. No ggml code is declared or linked: those two files
// never call ggml. The reference's ggml submodule is absent from its checkout.
#pragma once
#include <cstddef>
#include <cstdint>
struct ggml_tensor;
struct ggml_context;
struct ggml_backend_buffer;
