// GPU preprocessing: the uint8 resizers of preprocess_real (bit-exact with DA3cpplib's
// src/preprocess.cpp:45-197) and their per-axis tap tables.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <map>
#include <tuple>
#include <vector>

namespace da3b {

// Per destination index d: taps [off[d], off[d+1]) of (source index, weight), in the
// order the reference accumulates them.
struct AxisTaps {
  std::vector<int> off, idx;
  std::vector<float> w;
};
AxisTaps cubic_taps(int ssize, int dsize);  // resize_cubic (src/preprocess.cpp:61-99)
AxisTaps area_taps(int ssize, int dsize);   // area_tab (src/preprocess.cpp:103-120)

// Device resizer with cached tap tables and grow-only scratch (allocated on first use
// of a larger size). Not thread-safe; one per device and user.
class Resizer {
 public:
  ~Resizer();
  // HWC RGB8 [B][sh][sw][3] -> [B][dh][dw][3]. mode 0: resize_cubic; 1: resize_area
  // (its bilinear fallback when both axes grow).
  int resize(const uint8_t* src, int B, int sw, int sh, uint8_t* dst, int dw, int dh, int mode, cudaStream_t s);
  // preprocess_real's resizes (src/preprocess.cpp:157-190) into dst at the processed size
  // *out_w x *out_h (dst == nullptr: size query only). src is device memory.
  int preprocess_real(const uint8_t* src, int B, int w, int h, int patch, int target, bool upper, uint8_t* dst,
                      int* out_w, int* out_h, cudaStream_t s);

 private:
  struct DevTaps {
    void* dev = nullptr;
    int* off = nullptr;
    int* idx = nullptr;
    float* w = nullptr;
  };
  const DevTaps* taps(int ssize, int dsize, int mode);
  std::map<std::tuple<int, int, int>, DevTaps> tables_;
  float* tmp_ = nullptr;
  size_t tmp_cap_ = 0;
  uint8_t* mid_ = nullptr;
  size_t mid_cap_ = 0;
};

}  // namespace da3b
