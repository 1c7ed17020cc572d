// GGUF reader / writer (host).
#include "b2_gguf.hpp"

#include <fcntl.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "b2_internal.hpp"

namespace b2 {

namespace {

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  bool need(size_t n) {
    if ((size_t)(end - p) < n) ok = false;
    return ok;
  }
  uint32_t u32() {
    uint32_t v = 0;
    if (need(4)) memcpy(&v, p, 4), p += 4;
    return v;
  }
  uint64_t u64() {
    uint64_t v = 0;
    if (need(8)) memcpy(&v, p, 8), p += 8;
    return v;
  }
  std::string str() {
    const uint64_t n = u64();
    if (!ok || n > (uint64_t)(end - p)) {
      ok = false;
      return {};
    }
    std::string s(reinterpret_cast<const char*>(p), n);
    p += n;
    return s;
  }
};

size_t scalar_size(uint32_t t) {
  switch (t) {
    case GGUF_U8: case GGUF_I8: case GGUF_BOOL: return 1;
    case GGUF_U16: case GGUF_I16: return 2;
    case GGUF_U32: case GGUF_I32: case GGUF_F32: return 4;
    case GGUF_U64: case GGUF_I64: case GGUF_F64: return 8;
  }
  return 0;
}

// Reads one scalar/string value into v; arrays are skipped after recording
// their element type and length (Milda/src/engine.cpp:89-146 skips likewise).
bool read_value(Cursor& c, uint32_t t, GgufValue& v) {
  v.type = t;
  switch (t) {
    case GGUF_U8: if (c.need(1)) v.i = *c.p, c.p += 1; break;
    case GGUF_I8: if (c.need(1)) v.i = (int8_t)*c.p, c.p += 1; break;
    case GGUF_BOOL: if (c.need(1)) v.i = *c.p != 0, c.p += 1; break;
    case GGUF_U16: { uint16_t x = 0; if (c.need(2)) memcpy(&x, c.p, 2), c.p += 2; v.i = x; break; }
    case GGUF_I16: { int16_t x = 0; if (c.need(2)) memcpy(&x, c.p, 2), c.p += 2; v.i = x; break; }
    case GGUF_U32: v.i = c.u32(); break;
    case GGUF_I32: v.i = (int32_t)c.u32(); break;
    case GGUF_F32: { const uint32_t b = c.u32(); float f; memcpy(&f, &b, 4); v.f = f; break; }
    case GGUF_U64: v.i = (int64_t)c.u64(); break;
    case GGUF_I64: v.i = (int64_t)c.u64(); break;
    case GGUF_F64: { const uint64_t b = c.u64(); double d; memcpy(&d, &b, 8); v.f = d; break; }
    case GGUF_STRING: v.s = c.str(); break;
    case GGUF_ARRAY: {
      v.arr_type = c.u32();
      v.arr_n = c.u64();
      if (!c.ok) return false;
      const size_t es = scalar_size(v.arr_type);
      if (es) {
        if (v.arr_n > (uint64_t)(c.end - c.p) / es) return c.ok = false;
        c.p += es * v.arr_n;
      } else if (v.arr_type == GGUF_STRING) {
        for (uint64_t i = 0; i < v.arr_n && c.ok; ++i) c.str();
      } else {
        return c.ok = false;   // nested arrays are not used by GGUF LLM files
      }
      break;
    }
    default: return c.ok = false;
  }
  return c.ok;
}

}  // namespace

GgufFile::~GgufFile() {
  if (map_) munmap(map_, map_size_);
}

bool GgufFile::open(const std::string& path, std::string* err) {
  const int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) {
    if (err) *err = "cannot open " + path;
    return false;
  }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    ::close(fd);
    if (err) *err = "cannot stat or too small: " + path;
    return false;
  }
  void* p = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_SHARED, fd, 0);
  ::close(fd);
  if (p == MAP_FAILED) {
    if (err) *err = "mmap failed: " + path;
    return false;
  }
  map_ = p;
  map_size_ = (size_t)st.st_size;
  path_ = path;
  // One pass in file order over the tensors: read ahead aggressively and
  // start now (Milda advises MADV_WILLNEED on the large mapped segments,
  // Milda/src/engine.cpp:980-993).
  (void)madvise(map_, map_size_, MADV_SEQUENTIAL);
  (void)madvise(map_, map_size_, MADV_WILLNEED);
  return parse(static_cast<const uint8_t*>(p), map_size_, err);
}

void GgufFile::release_pages() {
  if (!map_) return;
  // Milda evicts the page-cache ranges of the tensors it offloaded to the GPU
  // (POSIX_FADV_DONTNEED, Milda/src/engine.cpp:1018-1041, 1127-1137); here
  // every tensor is on the device, so the whole file goes.  Tensor records
  // keep their metadata; their data pointers are not used after the upload.
  (void)madvise(map_, map_size_, MADV_DONTNEED);
  munmap(map_, map_size_);
  map_ = nullptr;
  const int fd = ::open(path_.c_str(), O_RDONLY);
  if (fd >= 0) {
    (void)posix_fadvise(fd, 0, 0, POSIX_FADV_DONTNEED);
    ::close(fd);
  }
}

bool GgufFile::parse(const uint8_t* data, size_t size, std::string* err) {
  auto fail = [&](const char* m) {
    if (err) *err = m;
    return false;
  };
  base_ = data;
  size_ = size;
  Cursor c{data, data + size};
  if (c.u32() != 0x46554747u) return fail("not a GGUF file (bad magic)");
  version = c.u32();
  if (version != 2 && version != 3) return fail("unsupported GGUF version");
  const uint64_t n_tensors = c.u64(), n_kv = c.u64();
  if (!c.ok || n_tensors > (1u << 20) || n_kv > (1u << 20)) return fail("corrupt GGUF header");
  for (uint64_t i = 0; i < n_kv; ++i) {
    std::string key = c.str();
    const uint32_t t = c.u32();
    GgufValue v;
    if (!c.ok || !read_value(c, t, v)) return fail("corrupt GGUF metadata");
    kv[key] = v;
  }
  const GgufValue* al = get("general.alignment");
  if (al && (al->type == GGUF_U32 || al->type == GGUF_I32)) alignment = (size_t)al->i;
  if (alignment == 0 || (alignment & (alignment - 1))) return fail("general.alignment not a power of two");
  tensors.resize(n_tensors);
  for (uint64_t i = 0; i < n_tensors; ++i) {
    GgufTensor& t = tensors[i];
    t.name = c.str();
    t.n_dims = c.u32();
    if (!c.ok || t.n_dims == 0 || t.n_dims > 4) return fail("corrupt tensor info");
    for (uint32_t d = 0; d < t.n_dims; ++d) t.ne[d] = (int64_t)c.u64();
    t.type = (int)c.u32();
    t.offset = c.u64();
    if (!c.ok) return fail("truncated tensor table");
    by_name[t.name] = i;
  }
  const size_t hdr = (size_t)(c.p - data);
  data_offset = (hdr + alignment - 1) / alignment * alignment;
  for (auto& t : tensors) {
    int64_t rows = 1;
    for (uint32_t d = 1; d < t.n_dims; ++d) rows *= t.ne[d];
    const int be = block_elems(t.type);
    if (t.ne[0] <= 0 || rows <= 0 || t.ne[0] % be) return fail("tensor shape not a multiple of its block");
    t.bytes = row_bytes(t.type, t.ne[0]) * (size_t)rows;
    if (t.bytes == 0) return fail("unsupported tensor type");
    if (data_offset + t.offset + t.bytes > size) return fail("tensor data past end of file (truncated?)");
    t.data = data + data_offset + t.offset;
  }
  return true;
}

const GgufValue* GgufFile::get(const std::string& key) const {
  auto it = kv.find(key);
  return it == kv.end() ? nullptr : &it->second;
}

const GgufValue* GgufFile::get_suffix(const std::string& suffix) const {
  for (const auto& [k, v] : kv)
    if (k.size() >= suffix.size() && k.compare(k.size() - suffix.size(), suffix.size(), suffix) == 0) return &v;
  return nullptr;
}

int64_t GgufFile::get_int(const std::string& suffix, int64_t dflt) const {
  const GgufValue* v = get_suffix(suffix);
  if (!v || v->type == GGUF_STRING || v->type == GGUF_ARRAY || v->type == GGUF_F32 || v->type == GGUF_F64) return dflt;
  return v->i;
}

double GgufFile::get_float(const std::string& suffix, double dflt) const {
  const GgufValue* v = get_suffix(suffix);
  if (!v) return dflt;
  if (v->type == GGUF_F32 || v->type == GGUF_F64) return v->f;
  if (v->type == GGUF_STRING || v->type == GGUF_ARRAY) return dflt;
  return (double)v->i;
}

std::string GgufFile::get_str(const std::string& key, const std::string& dflt) const {
  const GgufValue* v = get(key);
  return (v && v->type == GGUF_STRING) ? v->s : dflt;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
  auto it = by_name.find(name);
  return it == by_name.end() ? nullptr : &tensors[it->second];
}

// ---- writer ----------------------------------------------------------------------------
void GgufWriter::add_u32(const std::string& k, uint32_t v) { kvs_.push_back({k, GGUF_U32, v, 0.0f, {}}); }
void GgufWriter::add_f32(const std::string& k, float v) { kvs_.push_back({k, GGUF_F32, 0, v, {}}); }
void GgufWriter::add_str(const std::string& k, const std::string& v) { kvs_.push_back({k, GGUF_STRING, 0, 0.0f, v}); }

void GgufWriter::add_tensor(const std::string& name, int type, int64_t ne0, int64_t ne1, int n_dims) {
  tensors.push_back({name, type, ne0, ne1, n_dims, row_bytes(type, ne0) * (size_t)ne1, 0});
}

void GgufWriter::layout() const {
  size_t off = 0;
  for (auto& t : const_cast<std::vector<T>&>(tensors)) {
    t.offset = off;
    off = (off + t.bytes + alignment - 1) / alignment * alignment;
  }
  data_bytes_ = off;
}

size_t GgufWriter::header_bytes() const {
  size_t n = 24;
  for (const auto& k : kvs_) {
    n += 8 + k.key.size() + 4;
    n += k.type == GGUF_STRING ? 8 + k.s.size() : 4;
  }
  for (const auto& t : tensors) n += 8 + t.name.size() + 4 + 8 * (size_t)t.n_dims + 4 + 8;
  return (n + alignment - 1) / alignment * alignment;
}

size_t GgufWriter::tensor_file_offset(size_t i) const {
  layout();
  return header_bytes() + tensors[i].offset;
}

size_t GgufWriter::total_bytes() const {
  layout();
  return header_bytes() + data_bytes_;
}

void GgufWriter::write_header(uint8_t* out) const {
  layout();
  uint8_t* p = out;
  auto w32 = [&](uint32_t v) { memcpy(p, &v, 4); p += 4; };
  auto w64 = [&](uint64_t v) { memcpy(p, &v, 8); p += 8; };
  auto wstr = [&](const std::string& s) { w64(s.size()); memcpy(p, s.data(), s.size()); p += s.size(); };
  w32(0x46554747u);
  w32(3);
  w64(tensors.size());
  w64(kvs_.size());
  for (const auto& k : kvs_) {
    wstr(k.key);
    w32(k.type);
    if (k.type == GGUF_STRING) wstr(k.s);
    else if (k.type == GGUF_F32) { memcpy(p, &k.f, 4); p += 4; }
    else w32(k.u);
  }
  for (const auto& t : tensors) {
    wstr(t.name);
    w32((uint32_t)t.n_dims);
    w64((uint64_t)t.ne0);
    if (t.n_dims >= 2) w64((uint64_t)t.ne1);
    w32((uint32_t)t.type);
    w64(t.offset);
  }
  const size_t hb = header_bytes();
  memset(p, 0, hb - (size_t)(p - out));
}

}  // namespace b2
