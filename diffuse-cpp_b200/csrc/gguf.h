// gguf.h — a read-only GGUF (v2 / v3) file reader: header, key-value metadata, tensor table, and
// the tensor data mapped from the file. It serves the model loader (model.cpp), which replaces
// diffuse_model_load_impl (src/diffuse-model.cpp:67-224); the reference reads the same files
// through ggml's gguf_init_from_file.
//
// File layout (little-endian): "GGUF", u32 version, u64 tensor count, u64 key-value count; the
// key-value pairs {string key, u32 value type, value}; the tensor infos {string name, u32 n_dims,
// u64 ne[n_dims], u32 ggml type, u64 data offset}; padding to general.alignment (default 32);
// the tensor data, each offset relative to the start of that section. A string is {u64 length,
// bytes}; an array is {u32 element type, u64 count, elements}.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace dmoe {

enum GgufValueType : uint32_t {
  GGUF_U8 = 0, GGUF_I8 = 1, GGUF_U16 = 2, GGUF_I16 = 3, GGUF_U32 = 4, GGUF_I32 = 5, GGUF_F32 = 6,
  GGUF_BOOL = 7, GGUF_STRING = 8, GGUF_ARRAY = 9, GGUF_U64 = 10, GGUF_I64 = 11, GGUF_F64 = 12
};

struct GgufValue {
  uint32_t type = 0;
  uint64_t u = 0;      // unsigned integer types and bool
  int64_t i = 0;       // signed integer types
  double f = 0.0;      // float types
  std::string s;       // strings
  uint32_t arr_type = 0;
  uint64_t arr_n = 0;  // arrays: element type and count (elements are skipped)
};

struct GgufTensor {
  std::string name;
  int n_dims = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  int32_t type = 0;
  uint64_t offset = 0;
  const uint8_t* data = nullptr;  // inside the mapping
  uint64_t nbytes = 0;            // 0 when the type's block size is unknown
};

// Bytes of `n` elements of ggml type `type` (whole blocks), or 0 for a type this reader does not
// size.
uint64_t ggml_type_nbytes(int32_t type, int64_t n);

class GgufFile {
 public:
  GgufFile() = default;
  GgufFile(const GgufFile&) = delete;
  GgufFile& operator=(const GgufFile&) = delete;
  ~GgufFile();
  // Maps and parses `path`; false with a message in err on any malformed or truncated part.
  bool open(const char* path, std::string& err);
  const GgufValue* find(const std::string& key) const;
  const GgufTensor* tensor(const std::string& name) const;
  uint32_t version() const { return version_; }
  size_t n_tensors() const { return tensors_.size(); }
  size_t n_kv() const { return kv_.size(); }

 private:
  void* map_ = nullptr;
  size_t size_ = 0;
  uint32_t version_ = 0;
  std::unordered_map<std::string, GgufValue> kv_;
  std::vector<GgufTensor> tensors_;
  std::unordered_map<std::string, size_t> by_name_;
};

}  // namespace dmoe
