// pk_gguf.cpp -- GGUF container reader (see pk_gguf.h).
#include "pk_gguf.h"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

namespace pk {

namespace {

struct Cursor {
  const uint8_t *b;
  size_t n;
  size_t o = 0;
  bool ok = true;

  bool take(size_t k) {
    if (!ok || k > n - o) {
      ok = false;
      return false;
    }
    return true;
  }
  uint64_t uint(size_t k) {
    if (!take(k)) return 0;
    uint64_t v = 0;
    std::memcpy(&v, b + o, k);  // little-endian host
    o += k;
    return v;
  }
  std::string str() {
    const uint64_t len = uint(8);
    if (!take(len)) return std::string();
    std::string s(reinterpret_cast<const char *>(b + o), (size_t)len);
    o += len;
    return s;
  }
};

// gguf.rs:345-375 skip_array (with string capture for tokenizer arrays).
bool skip_array(Cursor &c, uint32_t et, uint64_t count, std::vector<std::string> *strs, int depth,
                std::vector<int32_t> *i32s = nullptr) {
  if (depth > 4) return false;
  for (uint64_t i = 0; i < count && c.ok; i++) {
    switch (et) {
      case 0: case 1: case 7: c.uint(1); break;
      case 2: case 3: c.uint(2); break;
      case 4: case 6: c.uint(4); break;
      case 5: {
        const uint32_t v = (uint32_t)c.uint(4);
        if (i32s) i32s->push_back((int32_t)v);
      } break;
      case 10: case 11: case 12: c.uint(8); break;
      case 8: {
        std::string s = c.str();
        if (strs) strs->push_back(std::move(s));
      } break;
      case 9: {
        const uint32_t e2 = (uint32_t)c.uint(4);
        const uint64_t c2 = c.uint(8);
        if (!skip_array(c, e2, c2, nullptr, depth + 1)) return false;
      } break;
      default: return false;
    }
  }
  return c.ok;
}

}  // namespace

Gguf::~Gguf() {
  if (map_) munmap(map_, len_);
}

bool Gguf::open(const char *path, std::string &err) {
  const int fd = ::open(path, O_RDONLY);
  if (fd < 0) {
    err = std::string("cannot open ") + path;
    return false;
  }
  struct stat st;
  if (fstat(fd, &st) != 0) {
    ::close(fd);
    err = std::string("cannot stat ") + path;
    return false;
  }
  if (st.st_size == 0) {
    ::close(fd);
    err = std::string("empty file ") + path;
    return false;
  }
  len_ = (size_t)st.st_size;
  void *p = mmap(nullptr, len_, PROT_READ, MAP_PRIVATE, fd, 0);
  ::close(fd);
  if (p == MAP_FAILED) {
    err = std::string("mmap failed for ") + path;
    len_ = 0;
    return false;
  }
  map_ = static_cast<uint8_t *>(p);

  Cursor c{map_, len_};
  if (c.uint(4) != 0x46554747u) {
    err = "not a GGUF file";
    return false;
  }
  const uint32_t version = (uint32_t)c.uint(4);
  if (version < 2 || version > 3) {
    err = "unsupported GGUF version " + std::to_string(version);
    return false;
  }
  const uint64_t n_tensors = c.uint(8), n_kv = c.uint(8);
  if (n_tensors > 1000000 || n_kv > 1000000) {
    err = "implausible gguf header";
    return false;
  }
  for (uint64_t i = 0; i < n_kv && c.ok; i++) {
    std::string key = c.str();
    GgufValue v;
    v.type = (uint32_t)c.uint(4);
    switch (v.type) {
      case 0: v.u = c.uint(1); break;
      case 1: v.u = (uint64_t)(int64_t)(int8_t)c.uint(1); break;
      case 2: v.u = c.uint(2); break;
      case 3: v.u = (uint64_t)(int64_t)(int16_t)c.uint(2); break;
      case 4: v.u = c.uint(4); break;
      case 5: v.u = (uint64_t)(int64_t)(int32_t)c.uint(4); break;
      case 6: {
        const uint32_t bits = (uint32_t)c.uint(4);
        float f;
        std::memcpy(&f, &bits, 4);
        v.f = f;
      } break;
      case 7: v.u = c.uint(1) != 0; break;
      case 8: v.s = c.str(); break;
      case 9:
        v.arr_type = (uint32_t)c.uint(4);
        v.arr_count = c.uint(8);
        if (!skip_array(c, v.arr_type, v.arr_count, v.arr_type == 8 ? &v.arr_str : nullptr, 0,
                        v.arr_type == 5 ? &v.arr_i32 : nullptr)) {
          err = "bad metadata array for key " + key;
          return false;
        }
        break;
      case 10: case 11: v.u = c.uint(8); break;
      case 12: {
        const uint64_t bits = c.uint(8);
        double f;
        std::memcpy(&f, &bits, 8);
        v.f = f;
      } break;
      default:
        err = "unknown gguf metadata type " + std::to_string(v.type) + " for key " + key;
        return false;
    }
    kv_[key] = std::move(v);
  }
  for (uint64_t i = 0; i < n_tensors && c.ok; i++) {
    GgufTensor t;
    t.name = c.str();
    const uint32_t nd = (uint32_t)c.uint(4);
    if (nd > 4) {
      err = "tensor " + t.name + " has " + std::to_string(nd) + " dims";
      return false;
    }
    for (uint32_t j = 0; j < nd; j++) t.ne.push_back(c.uint(8));
    t.type = (uint32_t)c.uint(4);
    t.offset = c.uint(8);
    tensors_.push_back(std::move(t));
  }
  if (!c.ok) {
    err = "gguf truncated at offset " + std::to_string(c.o);
    return false;
  }
  size_t align = 32;
  auto it = kv_.find("general.alignment");
  if (it != kv_.end() && (it->second.type == 4 || it->second.type == 5 || it->second.type == 10)) {
    align = (size_t)it->second.u;
  }
  if (align == 0) align = 1;
  data_offset_ = (c.o + align - 1) / align * align;
  if (data_offset_ > len_) {
    err = "GGUF tensor data begins past the end of the file";
    return false;
  }
  return true;
}

const GgufTensor *Gguf::tensor(const std::string &name) const {
  for (const auto &t : tensors_)
    if (t.name == name) return &t;
  return nullptr;
}

const GgufValue *Gguf::get(const std::string &key) const {
  auto it = kv_.find(key);
  return it == kv_.end() ? nullptr : &it->second;
}

bool Gguf::get_u64(const std::string &key, uint64_t *out) const {  // gguf.rs:206-218
  const GgufValue *v = get(key);
  if (!v) return false;
  if (v->type <= 5 || v->type == 10 || v->type == 11) {
    *out = v->u;
    return true;
  }
  return false;
}

bool Gguf::get_f32(const std::string &key, float *out) const {  // gguf.rs:228-234
  const GgufValue *v = get(key);
  if (!v) return false;
  if (v->type == 6 || v->type == 12) {
    *out = (float)v->f;
    return true;
  }
  uint64_t u;
  if (get_u64(key, &u)) {
    *out = (float)u;
    return true;
  }
  return false;
}

std::string Gguf::get_str(const std::string &key) const {
  const GgufValue *v = get(key);
  return (v && v->type == 8) ? v->s : std::string();
}

}  // namespace pk
