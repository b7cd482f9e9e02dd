// Synthetic llama GGUF writer (fa_synth_write).  Weights are N(0, sigma):
// Philox4x32-10 (Salmon et al., SC'11) keyed by (seed, tensor index) with
// the element's group-of-4 index as counter, turned into normals by the
// Box-Muller transform, then quantised row by row.  Tensor order and names
// follow ModelWeights::load_from_gguf (src/model.rs:252-298); projection
// dims are written (N, K) so the flat data reads as [K][N] the way
// tensor::matmul indexes it (src/tensor.rs:244-258).
#include <fcntl.h>
#include <sys/mman.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "fa_host.hpp"
#include "quant_encode.hpp"

namespace fa {

namespace {

void philox(uint32_t c[4], uint32_t k0, uint32_t k1) {
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c[0], p1 = (uint64_t)0xCD9E8D57u * c[2];
    uint32_t n0 = (uint32_t)(p1 >> 32) ^ c[1] ^ k0, n2 = (uint32_t)(p0 >> 32) ^ c[3] ^ k1;
    c[1] = (uint32_t)p1;
    c[3] = (uint32_t)p0;
    c[0] = n0;
    c[2] = n2;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
}

// four normals for elements 4g..4g+3 of tensor `tid`
void normals4(uint64_t seed, uint32_t tid, uint64_t g, float out[4]) {
  uint32_t c[4] = {(uint32_t)g, (uint32_t)(g >> 32), 0x5EEDu, 0};
  philox(c, (uint32_t)seed ^ (uint32_t)(seed >> 32), tid);
  const float kTwoPi = 6.28318530717958647692f;
  for (int h = 0; h < 2; ++h) {
    float u1 = ((float)(c[2 * h] >> 8) + 0.5f) * (1.0f / 16777216.0f);
    float u2 = (float)(c[2 * h + 1] >> 8) * (1.0f / 16777216.0f);
    float r = std::sqrt(-2.0f * std::log(u1));
    out[2 * h] = r * std::cos(kTwoPi * u2);
    out[2 * h + 1] = r * std::sin(kTwoPi * u2);
  }
}

struct TensorSpec {
  std::string name;
  std::vector<uint64_t> dims;  // ggml order: dims[0] fastest
  int type;
  bool ones;  // norm weights = 1.0
  uint64_t rows, cols;  // flat data = rows x cols, cols contiguous
  uint64_t offset = 0, nbytes = 0;
};

void put(std::vector<uint8_t> &b, const void *p, size_t n) {
  const uint8_t *q = (const uint8_t *)p;
  b.insert(b.end(), q, q + n);
}
void put_str(std::vector<uint8_t> &b, const std::string &s) {
  uint64_t n = s.size();
  put(b, &n, 8);
  put(b, s.data(), n);
}
void kv_u32(std::vector<uint8_t> &b, const std::string &k, uint32_t v) {
  put_str(b, k);
  uint32_t t = 4;
  put(b, &t, 4);
  put(b, &v, 4);
}
void kv_f32(std::vector<uint8_t> &b, const std::string &k, float v) {
  put_str(b, k);
  uint32_t t = 6;
  put(b, &t, 4);
  put(b, &v, 4);
}
void kv_str(std::vector<uint8_t> &b, const std::string &k, const std::string &v) {
  put_str(b, k);
  uint32_t t = 8;
  put(b, &t, 4);
  put_str(b, v);
}

}  // namespace

int synth_write(const char *path, const fa_synth_spec *s, uint64_t seed) {
  if (!path || !s) return fail(FA_ERR_INVALID, "fa_synth_write: null argument");
  if (!s->n_layers || !s->n_embd || !s->n_heads || !s->n_kv_heads || !s->n_ff || !s->vocab)
    return fail(FA_ERR_INVALID, "fa_synth_write: zero dimension");
  if (s->n_embd % s->n_heads || s->n_heads % s->n_kv_heads)
    return fail(FA_ERR_INVALID, "fa_synth_write: heads do not divide");
  const uint32_t d = s->n_embd, hd = d / s->n_heads, kvd = s->n_kv_heads * hd, F = s->n_ff, V = s->vocab;
  std::vector<TensorSpec> ts;
  auto add = [&](const std::string &name, int type, uint64_t rows, uint64_t cols, bool ones) {
    TensorSpec t;
    t.name = name;
    t.type = type;
    t.rows = rows;
    t.cols = cols;
    t.ones = ones;
    t.dims = rows == 1 ? std::vector<uint64_t>{cols} : std::vector<uint64_t>{cols, rows};
    ts.push_back(t);
  };
  add("token_embd.weight", s->type_embd, V, d, false);  // [V][d]: row = token
  for (uint32_t l = 0; l < s->n_layers; ++l) {
    std::string p = "blk." + std::to_string(l) + ".";
    add(p + "attn_norm.weight", FA_GGML_F32, 1, d, true);
    add(p + "attn_q.weight", s->type_q, d, d, false);  // [K=d][N=d]
    add(p + "attn_k.weight", s->type_k, d, kvd, false);
    add(p + "attn_v.weight", s->type_v, d, kvd, false);
    add(p + "attn_output.weight", s->type_o, d, d, false);
    add(p + "ffn_norm.weight", FA_GGML_F32, 1, d, true);
    add(p + "ffn_gate.weight", s->type_gate, d, F, false);
    add(p + "ffn_up.weight", s->type_up, d, F, false);
    add(p + "ffn_down.weight", s->type_down, F, d, false);
  }
  add("output_norm.weight", FA_GGML_F32, 1, d, true);
  if (s->type_out >= 0) add("output.weight", s->type_out, d, V, false);  // [K=d][N=V]
  for (auto &t : ts) {
    if (!type_known(t.type)) return fail(FA_ERR_UNSUPPORTED, "fa_synth_write: unsupported type for " + t.name);
    if (t.cols % block_elems(t.type))
      return fail(FA_ERR_INVALID, "fa_synth_write: " + t.name + " width not a multiple of its block size");
  }
  // header + metadata + tensor infos
  std::vector<uint8_t> hdr;
  uint32_t magic = 0x46465547u, version = 3;
  uint64_t n_t = ts.size(), n_kv = 10;
  put(hdr, &magic, 4);
  put(hdr, &version, 4);
  put(hdr, &n_t, 8);
  put(hdr, &n_kv, 8);
  kv_str(hdr, "general.architecture", "llama");
  kv_u32(hdr, "general.tokenizer.ggml.vocab_size", V);
  kv_u32(hdr, "llama.block_count", s->n_layers);
  kv_u32(hdr, "llama.attention.head_count", s->n_heads);
  kv_u32(hdr, "llama.attention.head_count_kv", s->n_kv_heads);
  kv_u32(hdr, "llama.embedding_length", d);
  kv_u32(hdr, "llama.context_length", s->context_len);
  kv_f32(hdr, "llama.feed_forward_length", (float)F);  // FLOAT32: what metadata_f32 reads
  kv_f32(hdr, "llama.rope.freq_base", s->rope_base);
  kv_f32(hdr, "llama.attention.layer_norm_rms_epsilon", s->norm_eps);
  const uint64_t align = 32;
  uint64_t off = 0;
  for (auto &t : ts) {
    t.offset = off;
    t.nbytes = t.rows * type_nbytes(t.type, t.cols);
    off = (off + t.nbytes + align - 1) & ~(align - 1);
    put_str(hdr, t.name);
    uint32_t nd = (uint32_t)t.dims.size();
    put(hdr, &nd, 4);
    for (uint64_t dd : t.dims) put(hdr, &dd, 8);
    uint32_t ty = (uint32_t)t.type;
    put(hdr, &ty, 4);
    put(hdr, &t.offset, 8);
  }
  uint64_t data_start = (hdr.size() + align - 1) & ~(align - 1);
  uint64_t total = data_start + off;
  int fd = ::open(path, O_RDWR | O_CREAT | O_TRUNC, 0644);
  if (fd < 0) return fail(FA_ERR_INVALID, std::string("fa_synth_write: cannot create ") + path);
  if (ftruncate(fd, (off_t)total)) {
    ::close(fd);
    return fail(FA_ERR_OOM, "fa_synth_write: ftruncate failed");
  }
  uint8_t *map = (uint8_t *)mmap(nullptr, total, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
  ::close(fd);
  if (map == MAP_FAILED) return fail(FA_ERR_OOM, "fa_synth_write: mmap failed");
  std::memcpy(map, hdr.data(), hdr.size());
  // work items: row ranges of every tensor
  struct Item { uint32_t tid; uint64_t r0, r1; };
  std::vector<Item> items;
  for (uint32_t i = 0; i < ts.size(); ++i) {
    uint64_t rows_per = std::max<uint64_t>(1, (1u << 20) / ts[i].cols);
    for (uint64_t r = 0; r < ts[i].rows; r += rows_per) items.push_back({i, r, std::min(ts[i].rows, r + rows_per)});
  }
  unsigned nth = s->threads ? s->threads : std::max(1u, std::thread::hardware_concurrency());
  std::atomic<size_t> next{0};
  auto worker = [&]() {
    std::vector<float> row;
    for (;;) {
      size_t it = next.fetch_add(1);
      if (it >= items.size()) break;
      const Item &w = items[it];
      const TensorSpec &t = ts[w.tid];
      row.resize(t.cols + 4);
      uint8_t *dst = map + data_start + t.offset;
      size_t rb = type_nbytes(t.type, t.cols);
      for (uint64_t r = w.r0; r < w.r1; ++r) {
        if (t.ones) {
          std::fill(row.begin(), row.begin() + t.cols, 1.0f);
        } else {
          uint64_t e0 = r * t.cols;
          // element e uses normals4 group e/4; rows are multiples of 32 wide
          for (uint64_t c = 0; c < t.cols; c += 4) {
            float z[4];
            normals4(seed, w.tid, (e0 + c) / 4, z);
            for (int q = 0; q < 4; ++q) row[c + q] = s->sigma * z[q];
          }
        }
        quantize_row(t.type, row.data(), t.cols, dst + r * rb);
      }
    }
  };
  std::vector<std::thread> pool;
  for (unsigned i = 0; i < nth; ++i) pool.emplace_back(worker);
  for (auto &th : pool) th.join();
  msync(map, total, MS_SYNC);
  munmap(map, total);
  return FA_OK;
}

}  // namespace fa
