// GGUF v2/v3 reader and writer (host).  The reader follows the layout the
// engines parse (Singularity/src/core/cortex_a5_engine.cpp:429-659,
// Milda/src/engine.cpp:89-237): header, typed key/value metadata, tensor
// table, data section aligned to general.alignment.
#pragma once

#include <stddef.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace b2 {

enum GgufValueType : uint32_t {
  GGUF_U8 = 0, GGUF_I8 = 1, GGUF_U16 = 2, GGUF_I16 = 3, GGUF_U32 = 4, GGUF_I32 = 5, GGUF_F32 = 6,
  GGUF_BOOL = 7, GGUF_STRING = 8, GGUF_ARRAY = 9, GGUF_U64 = 10, GGUF_I64 = 11, GGUF_F64 = 12,
};

struct GgufValue {
  uint32_t type = 0;
  int64_t i = 0;        // integer / bool value
  double f = 0.0;       // float value
  std::string s;        // string value
  uint32_t arr_type = 0;
  uint64_t arr_n = 0;   // array length (elements are not materialised)
};

struct GgufTensor {
  std::string name;
  uint32_t n_dims = 0;
  int64_t ne[4] = {1, 1, 1, 1};
  int type = 0;
  uint64_t offset = 0;        // relative to the data section
  const uint8_t* data = nullptr;
  size_t bytes = 0;
};

class GgufFile {
 public:
  ~GgufFile();
  // Maps a file read-only; returns false with an error message on failure.
  // The mapping is advised for one sequential pass with read-ahead.
  bool open(const std::string& path, std::string* err);
  // Drops the mapping and asks the kernel to evict the file's pages from the
  // page cache (the weights now live on the device); metadata stays.
  void release_pages();
  // Parses a caller-owned buffer (must outlive this object).
  bool parse(const uint8_t* data, size_t size, std::string* err);

  const GgufValue* get(const std::string& key) const;
  // First key that ends with `suffix` (architecture-prefixed keys).
  const GgufValue* get_suffix(const std::string& suffix) const;
  int64_t get_int(const std::string& suffix, int64_t dflt) const;
  double get_float(const std::string& suffix, double dflt) const;
  std::string get_str(const std::string& key, const std::string& dflt) const;
  const GgufTensor* tensor(const std::string& name) const;

  uint32_t version = 0;
  size_t alignment = 32;
  size_t data_offset = 0;
  std::map<std::string, GgufValue> kv;
  std::vector<GgufTensor> tensors;
  std::map<std::string, size_t> by_name;

 private:
  const uint8_t* base_ = nullptr;
  size_t size_ = 0;
  void* map_ = nullptr;
  size_t map_size_ = 0;
  std::string path_;
};

// Minimal writer: metadata then tensors, data aligned to `alignment`.
class GgufWriter {
 public:
  void add_u32(const std::string& k, uint32_t v);
  void add_f32(const std::string& k, float v);
  void add_str(const std::string& k, const std::string& v);
  // Declares a tensor (ne[0] = row length, ne[1] = rows); data comes later.
  void add_tensor(const std::string& name, int type, int64_t ne0, int64_t ne1, int n_dims);
  // Serialised header size (including padding to the data section).
  size_t header_bytes() const;
  // Byte offset of tensor i inside the file.
  size_t tensor_file_offset(size_t i) const;
  size_t total_bytes() const;
  // Writes the header into out (header_bytes() long).
  void write_header(uint8_t* out) const;
  size_t alignment = 32;

  struct T {
    std::string name;
    int type;
    int64_t ne0, ne1;
    int n_dims;
    size_t bytes;
    size_t offset;
  };
  std::vector<T> tensors;

 private:
  struct KV {
    std::string key;
    uint32_t type;
    uint32_t u;
    float f;
    std::string s;
  };
  std::vector<KV> kvs_;
  void layout() const;
  mutable size_t data_bytes_ = 0;
};

}  // namespace b2
