// GGUF reader (format: magic "GGUF", version, tensor count, kv count, kvs,
// tensor infos, alignment padding, data section). See gguf.h.
#include "gguf.h"

#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

namespace da3b {

namespace {

enum : int {
  kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7, kStr = 8, kArr = 9,
  kU64 = 10, kI64 = 11, kF64 = 12,
};

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  template <typename T>
  T get() {
    T v{};
    if (p + sizeof(T) > end) { ok = false; return v; }
    memcpy(&v, p, sizeof(T));
    p += sizeof(T);
    return v;
  }
  std::string str() {
    const uint64_t n = get<uint64_t>();
    if (!ok || n > static_cast<uint64_t>(end - p)) { ok = false; return {}; }
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
};

bool read_value(Cursor& c, int type, GgufValue& v, int depth) {
  v.type = type;
  switch (type) {
    case kU8: v.u = c.get<uint8_t>(); v.i = static_cast<int64_t>(v.u); v.f = static_cast<double>(v.u); break;
    case kI8: v.i = c.get<int8_t>(); v.u = static_cast<uint64_t>(v.i); v.f = static_cast<double>(v.i); break;
    case kU16: v.u = c.get<uint16_t>(); v.i = static_cast<int64_t>(v.u); v.f = static_cast<double>(v.u); break;
    case kI16: v.i = c.get<int16_t>(); v.u = static_cast<uint64_t>(v.i); v.f = static_cast<double>(v.i); break;
    case kU32: v.u = c.get<uint32_t>(); v.i = static_cast<int64_t>(v.u); v.f = static_cast<double>(v.u); break;
    case kI32: v.i = c.get<int32_t>(); v.u = static_cast<uint64_t>(v.i); v.f = static_cast<double>(v.i); break;
    case kU64: v.u = c.get<uint64_t>(); v.i = static_cast<int64_t>(v.u); v.f = static_cast<double>(v.u); break;
    case kI64: v.i = c.get<int64_t>(); v.u = static_cast<uint64_t>(v.i); v.f = static_cast<double>(v.i); break;
    case kF32: v.f = c.get<float>(); v.i = static_cast<int64_t>(v.f); break;
    case kF64: v.f = c.get<double>(); v.i = static_cast<int64_t>(v.f); break;
    case kBool: v.u = c.get<uint8_t>() != 0; v.i = static_cast<int64_t>(v.u); break;
    case kStr: v.s = c.str(); break;
    case kArr: {
      if (depth > 2) return false;
      const int et = static_cast<int>(c.get<uint32_t>());
      const uint64_t n = c.get<uint64_t>();
      if (!c.ok || n > (1ull << 32)) return false;
      v.arr.resize(n);
      for (uint64_t i = 0; i < n && c.ok; ++i)
        if (!read_value(c, et, v.arr[i], depth + 1)) return false;
      break;
    }
    default: return false;
  }
  return c.ok;
}

}  // namespace

size_t ggml_nbytes(int type, int64_t nel) {
  switch (type) {
    case 0: return static_cast<size_t>(nel) * 4;
    case 1: return static_cast<size_t>(nel) * 2;
    case 8: return static_cast<size_t>(nel) / 32 * 34;
    default: return 0;
  }
}

GgufFile::~GgufFile() {
  if (map_) munmap(map_, size_);
}

bool GgufFile::open(const std::string& path, std::string* err) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) { if (err) *err = "cannot open " + path; return false; }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 32) { ::close(fd); if (err) *err = "bad file " + path; return false; }
  size_ = static_cast<size_t>(st.st_size);
  map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) { map_ = nullptr; if (err) *err = "mmap failed " + path; return false; }
  const uint8_t* base = static_cast<const uint8_t*>(map_);
  Cursor c{base, base + size_};
  if (memcmp(base, "GGUF", 4) != 0) { if (err) *err = "not a GGUF file"; return false; }
  c.p += 4;
  const uint32_t version = c.get<uint32_t>();
  if (version < 2 || version > 3) { if (err) *err = "unsupported GGUF version"; return false; }
  const uint64_t n_tensors = c.get<uint64_t>();
  const uint64_t n_kv = c.get<uint64_t>();
  if (!c.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) { if (err) *err = "corrupt GGUF header"; return false; }
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key = c.str();
    const int type = static_cast<int>(c.get<uint32_t>());
    GgufValue v;
    if (!c.ok || !read_value(c, type, v, 0)) { if (err) *err = "corrupt GGUF kv"; return false; }
    kv_[key] = std::move(v);
  }
  std::vector<GgufTensor> infos(n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    GgufTensor& t = infos[i];
    t.name = c.str();
    const uint32_t nd = c.get<uint32_t>();
    if (!c.ok || nd > 4) { if (err) *err = "corrupt tensor info"; return false; }
    for (uint32_t d = 0; d < nd; ++d) t.ne[d] = static_cast<int64_t>(c.get<uint64_t>());
    t.type = static_cast<int>(c.get<uint32_t>());
    t.offset = c.get<uint64_t>();
    if (!c.ok) { if (err) *err = "corrupt tensor info"; return false; }
  }
  uint64_t align = 32;
  if (auto* a = kv("general.alignment")) align = a->u ? a->u : 32;
  const size_t hdr = static_cast<size_t>(c.p - base);
  const size_t data_off = (hdr + align - 1) / align * align;
  for (auto& t : infos) {
    t.nbytes = ggml_nbytes(t.type, t.nel());
    if (t.nbytes == 0) { if (err) *err = "unsupported tensor type in " + t.name; return false; }
    if (data_off + t.offset + t.nbytes > size_) { if (err) *err = "tensor out of file: " + t.name; return false; }
    t.data = base + data_off + t.offset;
    tensors_[t.name] = t;
  }
  // Nested metric-branch files keep their tensors under m_vit.* / m_head.*; they are
  // also reachable as vit.* / head.* so one loader serves both layouts
  // (src/model_loader.cpp:146-154).
  for (const auto& t : infos) {
    std::string alias;
    if (t.name.rfind("m_vit.", 0) == 0) alias = t.name.substr(2);
    else if (t.name.rfind("m_head.", 0) == 0) alias = t.name.substr(2);
    if (alias.empty()) continue;
    GgufTensor a = tensors_[t.name];
    a.name = alias;
    tensors_[alias] = a;
  }
  return true;
}

const GgufValue* GgufFile::kv(const std::string& key) const {
  auto it = kv_.find(key);
  return it == kv_.end() ? nullptr : &it->second;
}
const GgufTensor* GgufFile::tensor(const std::string& name) const {
  auto it = tensors_.find(name);
  return it == tensors_.end() ? nullptr : &it->second;
}
uint32_t GgufFile::get_u32(const std::string& k, uint32_t d) const {
  auto* v = kv(k);
  return v ? static_cast<uint32_t>(v->u) : d;
}
int32_t GgufFile::get_i32(const std::string& k, int32_t d) const {
  auto* v = kv(k);
  return v ? static_cast<int32_t>(v->i) : d;
}
float GgufFile::get_f32(const std::string& k, float d) const {
  auto* v = kv(k);
  return v ? static_cast<float>(v->f) : d;
}
bool GgufFile::get_bool(const std::string& k, bool d) const {
  auto* v = kv(k);
  return v ? v->u != 0 : d;
}
std::string GgufFile::get_str(const std::string& k, const std::string& d) const {
  auto* v = kv(k);
  return (v && v->type == kStr) ? v->s : d;
}
std::vector<int32_t> GgufFile::get_i32_arr(const std::string& k) const {
  std::vector<int32_t> out;
  auto* v = kv(k);
  if (v && v->type == kArr)
    for (auto& e : v->arr) out.push_back(static_cast<int32_t>(e.i));
  return out;
}
std::vector<float> GgufFile::get_f32_arr(const std::string& k) const {
  std::vector<float> out;
  auto* v = kv(k);
  if (v && v->type == kArr)
    for (auto& e : v->arr) out.push_back(static_cast<float>(e.f));
  return out;
}

}  // namespace da3b
