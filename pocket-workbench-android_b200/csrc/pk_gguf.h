// pk_gguf.h -- read-only GGUF v2/v3 view over an mmap'd file.
//
// Follows rust/pocketinfer/src/gguf.rs:107-192 (header, metadata, tensor
// table, alignment -> data_offset) and util.rs:154-217 (zero-copy mmap).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <map>
#include <string>
#include <vector>

namespace pk {

struct GgufTensor {
  std::string name;
  std::vector<uint64_t> ne;
  uint32_t type = 0;
  uint64_t offset = 0;  // relative to data_offset
};

struct GgufValue {
  uint32_t type = 0;      // gguf metadata type id
  uint64_t u = 0;         // integer types (sign-extended for signed ones)
  double f = 0.0;         // f32 / f64
  std::string s;          // string
  uint32_t arr_type = 0;  // array element type
  uint64_t arr_count = 0;
  std::vector<std::string> arr_str;
  std::vector<int32_t> arr_i32;  // elements of an i32 array (tokenizer.ggml.token_type)
};

class Gguf {
 public:
  Gguf() = default;
  ~Gguf();
  Gguf(const Gguf &) = delete;
  Gguf &operator=(const Gguf &) = delete;

  // Returns false and fills err on any parse or IO failure.
  bool open(const char *path, std::string &err);

  const uint8_t *data() const { return map_; }
  size_t size() const { return len_; }
  size_t data_offset() const { return data_offset_; }
  const std::vector<GgufTensor> &tensors() const { return tensors_; }
  const GgufTensor *tensor(const std::string &name) const;

  bool get_u64(const std::string &key, uint64_t *out) const;
  bool get_f32(const std::string &key, float *out) const;
  std::string get_str(const std::string &key) const;
  const GgufValue *get(const std::string &key) const;

 private:
  uint8_t *map_ = nullptr;
  size_t len_ = 0;
  size_t data_offset_ = 0;
  std::map<std::string, GgufValue> kv_;
  std::vector<GgufTensor> tensors_;
};

}  // namespace pk
