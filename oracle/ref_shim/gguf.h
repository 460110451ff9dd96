// Forward declaration only (see ggml.h in this folder).
#pragma once
struct gguf_context;
