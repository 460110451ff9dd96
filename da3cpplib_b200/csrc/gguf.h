// Minimal GGUF v2/v3 reader: key/value metadata and tensor table over a memory
// mapped file. It serves the same role as ggml's gguf_init_from_file for
// ModelLoader::load (src/model_loader.cpp:73-159) — libda3b reads the reference's
// GGUF files directly without ggml.
#pragma once
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace da3b {

struct GgufValue {
  int type = -1;            // gguf value type id
  uint64_t u = 0;           // unsigned / bool
  int64_t i = 0;            // signed
  double f = 0;             // float
  std::string s;            // string
  std::vector<GgufValue> arr;
};

struct GgufTensor {
  std::string name;
  int type = 0;             // ggml type id (0 f32, 1 f16, 8 q8_0)
  int64_t ne[4] = {1, 1, 1, 1};
  uint64_t offset = 0;      // relative to the data section
  const uint8_t* data = nullptr;
  size_t nbytes = 0;
  int64_t nel() const { return ne[0] * ne[1] * ne[2] * ne[3]; }
};

class GgufFile {
 public:
  ~GgufFile();
  bool open(const std::string& path, std::string* err);
  const GgufValue* kv(const std::string& key) const;
  const GgufTensor* tensor(const std::string& name) const;
  const std::map<std::string, GgufTensor>& tensors() const { return tensors_; }

  uint32_t get_u32(const std::string& k, uint32_t d) const;
  int32_t get_i32(const std::string& k, int32_t d) const;
  float get_f32(const std::string& k, float d) const;
  bool get_bool(const std::string& k, bool d) const;
  std::string get_str(const std::string& k, const std::string& d) const;
  std::vector<int32_t> get_i32_arr(const std::string& k) const;
  std::vector<float> get_f32_arr(const std::string& k) const;

 private:
  std::map<std::string, GgufValue> kv_;
  std::map<std::string, GgufTensor> tensors_;
  void* map_ = nullptr;
  size_t size_ = 0;
};

// Bytes of a tensor with ggml type `type` and `nel` elements (f32, f16, q8_0).
size_t ggml_nbytes(int type, int64_t nel);

}  // namespace da3b
