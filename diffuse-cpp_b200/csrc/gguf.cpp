// gguf.cpp — GGUF reader (format in gguf.h). The file is mapped read-only; every read is bounds
// checked against the mapping, so a truncated or corrupt file gives an error, never a read past
// its end.
#include "gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cerrno>
#include <cstring>

namespace dmoe {

uint64_t ggml_type_nbytes(int32_t type, int64_t n) {
  // {elements per block, bytes per block} of the ggml types (ggml.h enum ggml_type)
  int64_t blk = 0, bytes = 0;
  switch (type) {
    case 0: blk = 1, bytes = 4; break;      // F32
    case 1: blk = 1, bytes = 2; break;      // F16
    case 2: blk = 32, bytes = 18; break;    // Q4_0
    case 3: blk = 32, bytes = 20; break;    // Q4_1
    case 6: blk = 32, bytes = 22; break;    // Q5_0
    case 7: blk = 32, bytes = 24; break;    // Q5_1
    case 8: blk = 32, bytes = 34; break;    // Q8_0
    case 9: blk = 32, bytes = 36; break;    // Q8_1
    case 10: blk = 256, bytes = 84; break;  // Q2_K
    case 11: blk = 256, bytes = 110; break; // Q3_K
    case 12: blk = 256, bytes = 144; break; // Q4_K
    case 13: blk = 256, bytes = 176; break; // Q5_K
    case 14: blk = 256, bytes = 210; break; // Q6_K
    case 15: blk = 256, bytes = 292; break; // Q8_K
    case 24: blk = 1, bytes = 1; break;     // I8
    case 25: blk = 1, bytes = 2; break;     // I16
    case 26: blk = 1, bytes = 4; break;     // I32
    case 27: blk = 1, bytes = 8; break;     // I64
    case 28: blk = 1, bytes = 8; break;     // F64
    case 30: blk = 1, bytes = 2; break;     // BF16
    default: return 0;
  }
  if (n < 0 || n % blk) return 0;
  return (uint64_t)(n / blk) * (uint64_t)bytes;
}

namespace {

struct Cursor {
  const uint8_t* p;
  const uint8_t* end;
  bool ok = true;
  bool take(void* dst, size_t n) {
    if (!ok || (size_t)(end - p) < n) return ok = false;
    std::memcpy(dst, p, n);
    p += n;
    return true;
  }
  bool skip(uint64_t n) {
    if (!ok || (uint64_t)(end - p) < n) return ok = false;
    p += n;
    return true;
  }
  template <class T>
  T get() {
    T v{};
    take(&v, sizeof(T));
    return v;
  }
  bool str(std::string& s) {
    const uint64_t n = get<uint64_t>();
    if (!ok || (uint64_t)(end - p) < n) return ok = false;
    s.assign(reinterpret_cast<const char*>(p), (size_t)n);
    p += n;
    return true;
  }
};

size_t scalar_size(uint32_t t) {
  switch (t) {
    case GGUF_U8: case GGUF_I8: case GGUF_BOOL: return 1;
    case GGUF_U16: case GGUF_I16: return 2;
    case GGUF_U32: case GGUF_I32: case GGUF_F32: return 4;
    case GGUF_U64: case GGUF_I64: case GGUF_F64: return 8;
    default: return 0;
  }
}

bool read_scalar(Cursor& c, uint32_t t, GgufValue& v) {
  switch (t) {
    case GGUF_U8: v.u = c.get<uint8_t>(); v.i = (int64_t)v.u; v.f = (double)v.u; break;
    case GGUF_I8: v.i = c.get<int8_t>(); v.u = (uint64_t)v.i; v.f = (double)v.i; break;
    case GGUF_U16: v.u = c.get<uint16_t>(); v.i = (int64_t)v.u; v.f = (double)v.u; break;
    case GGUF_I16: v.i = c.get<int16_t>(); v.u = (uint64_t)v.i; v.f = (double)v.i; break;
    case GGUF_U32: v.u = c.get<uint32_t>(); v.i = (int64_t)v.u; v.f = (double)v.u; break;
    case GGUF_I32: v.i = c.get<int32_t>(); v.u = (uint64_t)v.i; v.f = (double)v.i; break;
    case GGUF_F32: v.f = c.get<float>(); break;
    case GGUF_BOOL: v.u = c.get<uint8_t>() ? 1 : 0; v.i = (int64_t)v.u; break;
    case GGUF_U64: v.u = c.get<uint64_t>(); v.i = (int64_t)v.u; v.f = (double)v.u; break;
    case GGUF_I64: v.i = c.get<int64_t>(); v.u = (uint64_t)v.i; v.f = (double)v.i; break;
    case GGUF_F64: v.f = c.get<double>(); break;
    default: return c.ok = false;
  }
  return c.ok;
}

}  // namespace

GgufFile::~GgufFile() {
  if (map_) munmap(map_, size_);
}

bool GgufFile::open(const char* path, std::string& err) {
  const int fd = ::open(path, O_RDONLY);
  if (fd < 0) {
    err = std::string("cannot open ") + path + ": " + std::strerror(errno);
    return false;
  }
  struct stat st;
  if (fstat(fd, &st) != 0 || st.st_size < 24) {
    ::close(fd);
    err = std::string(path) + ": not a GGUF file (too short)";
    return false;
  }
  size_ = (size_t)st.st_size;
  map_ = mmap(nullptr, size_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (map_ == MAP_FAILED) {
    map_ = nullptr;
    err = std::string("mmap failed: ") + std::strerror(errno);
    return false;
  }
  const uint8_t* base = static_cast<const uint8_t*>(map_);
  Cursor c{base, base + size_};
  char magic[4];
  c.take(magic, 4);
  if (std::memcmp(magic, "GGUF", 4) != 0) {
    err = std::string(path) + ": bad magic (not a GGUF file)";
    return false;
  }
  version_ = c.get<uint32_t>();
  if (version_ != 2 && version_ != 3) {
    err = "unsupported GGUF version " + std::to_string(version_) + " (2 and 3 are read)";
    return false;
  }
  const uint64_t n_tensors = c.get<uint64_t>(), n_kv = c.get<uint64_t>();
  // every key-value pair and tensor info takes at least 12 / 24 bytes: bound the counts
  if (n_kv > size_ / 12 || n_tensors > size_ / 24) {
    err = "implausible tensor / key counts";
    return false;
  }
  for (uint64_t k = 0; k < n_kv && c.ok; ++k) {
    std::string key;
    GgufValue v;
    c.str(key);
    v.type = c.get<uint32_t>();
    if (!c.ok) break;
    if (v.type == GGUF_STRING) {
      c.str(v.s);
    } else if (v.type == GGUF_ARRAY) {
      v.arr_type = c.get<uint32_t>();
      v.arr_n = c.get<uint64_t>();
      if (v.arr_type == GGUF_STRING) {
        for (uint64_t j = 0; j < v.arr_n && c.ok; ++j) c.skip(c.get<uint64_t>());
      } else if (const size_t es = scalar_size(v.arr_type)) {
        if (v.arr_n > (uint64_t)(c.end - c.p) / es) c.ok = false;
        else c.skip(v.arr_n * es);
      } else {
        err = "key " + key + ": unsupported array element type " + std::to_string(v.arr_type);
        return false;
      }
    } else if (!read_scalar(c, v.type, v)) {
      err = "key " + key + ": unsupported value type " + std::to_string(v.type);
      return false;
    }
    if (c.ok) kv_[key] = std::move(v);
  }
  tensors_.resize((size_t)n_tensors);
  for (uint64_t t = 0; t < n_tensors && c.ok; ++t) {
    GgufTensor& T = tensors_[(size_t)t];
    c.str(T.name);
    const uint32_t nd = c.get<uint32_t>();
    if (!c.ok) break;
    if (nd < 1 || nd > 4) {
      err = "tensor " + T.name + ": " + std::to_string(nd) + " dimensions";
      return false;
    }
    T.n_dims = (int)nd;
    for (uint32_t d = 0; d < nd; ++d) {
      const uint64_t ne = c.get<uint64_t>();
      if (ne > (1ull << 40)) {
        err = "tensor " + T.name + ": dimension too large";
        return false;
      }
      T.ne[d] = (int64_t)ne;
    }
    T.type = (int32_t)c.get<uint32_t>();
    T.offset = c.get<uint64_t>();
  }
  if (!c.ok) {
    err = "truncated GGUF header";
    return false;
  }
  uint64_t align = 32;
  if (const GgufValue* a = find("general.alignment")) {
    if (a->type != GGUF_U32 || a->u == 0 || (a->u & (a->u - 1))) {
      err = "general.alignment must be a power-of-two u32";
      return false;
    }
    align = a->u;
  }
  const uint64_t hdr = (uint64_t)(c.p - base);
  const uint64_t data0 = (hdr + align - 1) / align * align;
  for (GgufTensor& T : tensors_) {
    int64_t n = 1;
    for (int d = 0; d < 4; ++d) {
      if (T.ne[d] != 0 && n > (int64_t(1) << 50) / T.ne[d]) {
        err = "tensor " + T.name + ": too many elements";
        return false;
      }
      n *= T.ne[d];
    }
    T.nbytes = ggml_type_nbytes(T.type, n);
    if (T.offset % align) {
      err = "tensor " + T.name + ": data offset not aligned";
      return false;
    }
    if (data0 + T.offset > size_ || T.nbytes > size_ - data0 - T.offset) {
      err = "tensor " + T.name + ": data past the end of the file";
      return false;
    }
    T.data = base + data0 + T.offset;
    if (!by_name_.emplace(T.name, (size_t)(&T - tensors_.data())).second) {
      err = "duplicate tensor " + T.name;
      return false;
    }
  }
  return true;
}

const GgufValue* GgufFile::find(const std::string& key) const {
  const auto it = kv_.find(key);
  return it == kv_.end() ? nullptr : &it->second;
}

const GgufTensor* GgufFile::tensor(const std::string& name) const {
  const auto it = by_name_.find(name);
  return it == by_name_.end() ? nullptr : &tensors_[it->second];
}

}  // namespace dmoe
