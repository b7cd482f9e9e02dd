// GGUF v1-v3 container reader (host).  Follows the reference's GGUFFile
// (src/gguf.rs:438-689): mmap, little-endian header, typed metadata, tensor
// table, data section aligned to general.alignment (default 32), tensor
// byte size by the next-larger-offset rule.
#pragma once
#include <cstdint>
#include <string>
#include <unordered_map>
#include <vector>

namespace fa {

struct GgufMeta {
  uint32_t type = 0;  // GGUF value type id (0..12)
  uint64_t u = 0;
  int64_t i = 0;
  double f64 = 0;
  float f32 = 0;
  bool b = false;
  std::string s;
  uint32_t arr_type = 0;
  uint64_t arr_len = 0;
  std::vector<std::string> arr_str;  // string arrays (e.g. tokenizer.ggml.tokens / merges)
  std::vector<double> arr_num;       // numeric arrays, each element widened exactly
};

struct GgufTensor {
  std::string name;
  uint32_t n_dims = 0;
  uint64_t dims[4] = {0, 0, 0, 0};
  uint32_t ggml_type = 0;
  uint64_t offset = 0;
  uint64_t nelement() const {
    uint64_t n = 1;
    for (uint32_t d = 0; d < n_dims; ++d) n *= dims[d];
    return n;
  }
};

class Gguf {
 public:
  ~Gguf();
  // returns nullptr and sets the thread's error on failure
  static Gguf *open(const std::string &path, int *code);

  uint32_t version = 0;
  uint64_t alignment = 32;
  std::vector<GgufTensor> tensors;

  const GgufMeta *meta(const std::string &key) const;
  bool meta_u64(const std::string &key, uint64_t *v) const;
  bool meta_i64(const std::string &key, int64_t *v) const;
  bool meta_f32(const std::string &key, float *v) const;
  bool meta_bool(const std::string &key, bool *v) const;
  bool meta_string(const std::string &key, std::string *v) const;
  bool vocab_size(uint64_t *v) const;
  // array values: false when the key is absent or not an array of that kind
  const std::vector<std::string> *meta_str_array(const std::string &key) const;
  const std::vector<double> *meta_num_array(const std::string &key) const;
  const GgufTensor *tensor(const std::string &name) const;
  // bytes of a tensor by the next-offset rule; nullptr/0 when empty
  const uint8_t *tensor_data(const GgufTensor &t, size_t *nbytes) const;
  size_t file_size() const { return map_len_; }

 private:
  std::unordered_map<std::string, GgufMeta> meta_;
  std::unordered_map<std::string, size_t> tindex_;
  const uint8_t *map_ = nullptr;
  size_t map_len_ = 0;
  size_t data_offset_ = 0;
};

}  // namespace fa
