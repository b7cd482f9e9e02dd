#include "gguf.hpp"

#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cstring>

#include "fa_host.hpp"

namespace fa {

namespace {

struct Reader {
  const uint8_t *p;
  size_t len, pos = 0;
  bool get(void *dst, size_t n) {
    if (pos + n > len) return false;
    std::memcpy(dst, p + pos, n);
    pos += n;
    return true;
  }
  template <class T>
  bool get(T *v) {
    return get((void *)v, sizeof(T));
  }
  bool str(std::string *out, std::string *err) {
    uint64_t n;
    if (!get(&n)) return *err = "failed to read string length", false;
    if (n > 256ull * 1024 * 1024) return *err = "string length too large: " + std::to_string(n), false;
    if (pos + n > len) return *err = "failed to read string data (want " + std::to_string(n) + " bytes)", false;
    out->assign((const char *)p + pos, n);
    pos += n;
    return true;
  }
};

const size_t kScalarSize[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};

bool read_value(Reader &r, uint32_t t, GgufMeta *m, int depth, std::string *err) {
  m->type = t;
  switch (t) {
    case 0: { uint8_t v; if (!r.get(&v)) break; m->u = v; return true; }
    case 1: { int8_t v; if (!r.get(&v)) break; m->i = v; return true; }
    case 2: { uint16_t v; if (!r.get(&v)) break; m->u = v; return true; }
    case 3: { int16_t v; if (!r.get(&v)) break; m->i = v; return true; }
    case 4: { uint32_t v; if (!r.get(&v)) break; m->u = v; return true; }
    case 5: { int32_t v; if (!r.get(&v)) break; m->i = v; return true; }
    case 6: { float v; if (!r.get(&v)) break; m->f32 = v; return true; }
    case 7: { uint8_t v; if (!r.get(&v)) break; m->b = v != 0; return true; }
    case 8: return r.str(&m->s, err);
    case 10: { uint64_t v; if (!r.get(&v)) break; m->u = v; return true; }
    case 11: { int64_t v; if (!r.get(&v)) break; m->i = v; return true; }
    case 12: { double v; if (!r.get(&v)) break; m->f64 = v; return true; }
    case 9: {
      uint32_t it;
      uint64_t n;
      if (!r.get(&it)) break;
      if (it > 12) return *err = "unknown array item type: " + std::to_string(it), false;
      if (!r.get(&n)) break;
      if (n > 10000000ull) return *err = "array too large: " + std::to_string(n), false;
      m->arr_type = it;
      m->arr_len = n;
      for (uint64_t k = 0; k < n; ++k) {
        if (it == 8) {
          std::string s;
          if (!r.str(&s, err)) return false;
          m->arr_str.push_back(std::move(s));
        } else if (it == 9) {
          GgufMeta tmp;
          if (depth > 8 || !read_value(r, it, &tmp, depth + 1, err)) return false;
        } else {
          GgufMeta e;
          if (!read_value(r, it, &e, depth + 1, err)) return *err = "truncated array", false;
          const double v = it == 6 ? (double)e.f32 : it == 12 ? e.f64 : it == 7 ? (e.b ? 1.0 : 0.0)
                         : (it == 1 || it == 3 || it == 5 || it == 11) ? (double)e.i : (double)e.u;
          m->arr_num.push_back(v);
        }
      }
      return true;
    }
    default: return *err = "unknown value type: " + std::to_string(t), false;
  }
  *err = "truncated metadata value";
  return false;
}

}  // namespace

Gguf::~Gguf() {
  if (map_ && map_len_) munmap((void *)map_, map_len_);
}

Gguf *Gguf::open(const std::string &path, int *code) {
  *code = FA_ERR_GGUF;
  int fd = ::open(path.c_str(), O_RDONLY);
  if (fd < 0) return set_error("cannot open file '" + path + "'"), nullptr;
  struct stat st;
  if (fstat(fd, &st)) {
    ::close(fd);
    return set_error("cannot stat '" + path + "'"), nullptr;
  }
  Gguf *g = new Gguf();
  g->map_len_ = (size_t)st.st_size;
  if (g->map_len_) {
    void *p = mmap(nullptr, g->map_len_, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p == MAP_FAILED) {
      ::close(fd);
      delete g;
      return set_error("cannot map '" + path + "'"), nullptr;
    }
    g->map_ = (const uint8_t *)p;
  }
  ::close(fd);
  Reader r{g->map_, g->map_len_};
  std::string err;
  uint32_t magic, version;
  uint64_t n_t, n_kv;
  auto bad = [&](const std::string &m) {
    set_error(m);
    delete g;
    return (Gguf *)nullptr;
  };
  if (!r.get(&magic)) return bad("failed to read magic");
  // The reference's GGUF_MAGIC (src/gguf.rs:36) is 0x46465547, i.e. the
  // bytes "GUFF"; files from llama.cpp / gguf-py start with "GGUF"
  // (0x46554747).  Both are accepted here.
  if (magic != 0x46465547u && magic != 0x46554747u) {
    char b[96];
    snprintf(b, sizeof b, "invalid GGUF magic: expected 0x46465547, got 0x%08X", magic);
    return bad(b);
  }
  if (!r.get(&version)) return bad("failed to read version");
  if (version > 3) return bad("unsupported GGUF version: " + std::to_string(version) + " (max 3)");
  if (!r.get(&n_t) || !r.get(&n_kv)) return bad("failed to read tensor/metadata counts");
  if (n_t > 1000000ull) return bad("tensor count out of range: " + std::to_string(n_t));
  if (n_kv > 10000000ull) return bad("metadata count out of range: " + std::to_string(n_kv));
  g->version = version;
  for (uint64_t k = 0; k < n_kv; ++k) {
    std::string key;
    if (!r.str(&key, &err)) return bad(err);
    uint32_t vt;
    if (!r.get(&vt)) return bad("failed to read value type");
    if (vt > 12) return bad("unknown value type: " + std::to_string(vt));
    GgufMeta m;
    if (!read_value(r, vt, &m, 0, &err)) return bad(err);
    g->meta_[key] = std::move(m);  // HashMap::insert: the last value wins
  }
  g->alignment = 32;
  if (const GgufMeta *am = g->meta("general.alignment"))
    if (am->type == 10 || am->type == 4) g->alignment = am->u;
  if (g->alignment == 0 || (g->alignment & (g->alignment - 1)))
    return bad("invalid alignment: " + std::to_string(g->alignment) + " (must be a power of two)");
  g->tensors.reserve(n_t);
  for (uint64_t k = 0; k < n_t; ++k) {
    GgufTensor t;
    if (!r.str(&t.name, &err)) return bad(err);
    if (!r.get(&t.n_dims)) return bad("failed to read tensor n_dims");
    if (t.n_dims > 4) return bad("tensor n_dims " + std::to_string(t.n_dims) + " exceeds 4");
    for (uint32_t d = 0; d < t.n_dims; ++d)
      if (!r.get(&t.dims[d])) return bad("failed to read tensor dim");
    if (!r.get(&t.ggml_type) || !r.get(&t.offset)) return bad("failed to read tensor type/offset");
    g->tindex_.emplace(t.name, g->tensors.size());  // first match wins, as tensor_info's find
    g->tensors.push_back(std::move(t));
  }
  g->data_offset_ = (r.pos + g->alignment - 1) & ~(size_t)(g->alignment - 1);
  *code = FA_OK;
  return g;
}

const GgufMeta *Gguf::meta(const std::string &key) const {
  auto it = meta_.find(key);
  return it == meta_.end() ? nullptr : &it->second;
}
bool Gguf::meta_u64(const std::string &key, uint64_t *v) const {
  const GgufMeta *m = meta(key);
  if (!m || (m->type != 10 && m->type != 4)) return false;
  return *v = m->u, true;
}
bool Gguf::meta_i64(const std::string &key, int64_t *v) const {
  const GgufMeta *m = meta(key);
  if (!m || (m->type != 11 && m->type != 5)) return false;
  return *v = m->i, true;
}
bool Gguf::meta_f32(const std::string &key, float *v) const {
  const GgufMeta *m = meta(key);
  if (!m || m->type != 6) return false;
  return *v = m->f32, true;
}
bool Gguf::meta_bool(const std::string &key, bool *v) const {
  const GgufMeta *m = meta(key);
  if (!m || m->type != 7) return false;
  return *v = m->b, true;
}
const std::vector<std::string> *Gguf::meta_str_array(const std::string &key) const {
  const GgufMeta *m = meta(key);
  return (m && m->type == 9 && m->arr_type == 8) ? &m->arr_str : nullptr;
}
const std::vector<double> *Gguf::meta_num_array(const std::string &key) const {
  const GgufMeta *m = meta(key);
  return (m && m->type == 9 && m->arr_type != 8 && m->arr_type != 9) ? &m->arr_num : nullptr;
}

bool Gguf::meta_string(const std::string &key, std::string *v) const {
  const GgufMeta *m = meta(key);
  if (!m || m->type != 8) return false;
  return *v = m->s, true;
}
bool Gguf::vocab_size(uint64_t *v) const {
  if (meta_u64("general.tokenizer.ggml.vocab_size", v)) return true;
  const GgufMeta *m = meta("general.tokenizer.ggml.tokens");
  if (m && m->type == 9) return *v = m->arr_len, true;
  return false;
}
const GgufTensor *Gguf::tensor(const std::string &name) const {
  auto it = tindex_.find(name);
  return it == tindex_.end() ? nullptr : &tensors[it->second];
}

const uint8_t *Gguf::tensor_data(const GgufTensor &t, size_t *nbytes) const {
  size_t data_end = map_len_ > data_offset_ ? map_len_ - data_offset_ : 0;
  uint64_t next = data_end;
  for (const auto &o : tensors)
    if (o.offset > t.offset && o.offset < next) next = o.offset;
  *nbytes = 0;
  if (next <= t.offset) return nullptr;
  size_t sz = (size_t)(next - t.offset), start = data_offset_ + (size_t)t.offset;
  if (start + sz > map_len_) return nullptr;
  *nbytes = sz;
  return map_ + start;
}

}  // namespace fa
