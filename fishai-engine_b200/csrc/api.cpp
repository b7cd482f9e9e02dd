// extern "C" entry points declared in include/fishai_cuda.h.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <mutex>
#include <memory>
#include <new>
#include <string>
#include <vector>

#include "../../include/fishai_cuda.h"
#include "fa_host.hpp"
#include "fa_kernels.hpp"
#include "gguf.hpp"
#include "model.hpp"
#include "sdpa.hpp"
#include "tp.hpp"

namespace fa {
int synth_write(const char *path, const fa_synth_spec *s, uint64_t seed);
int tokenizer_from_gguf(const Gguf &g, fa_tokenizer **out);
uint32_t n_ff_of(uint32_t n_embd, float mult);
}  // namespace fa

using namespace fa;

struct fa_gguf {
  std::unique_ptr<Gguf> g;
};
struct fa_model {
  Model m;
  std::vector<Workspace> compat;  // per-token workspaces for multi-token forward
};
struct fa_kv {
  KvCache kv;
};

namespace {

#define API_CUDA(expr)                                                                     \
  do {                                                                                     \
    cudaError_t e_ = (expr);                                                               \
    if (e_ != cudaSuccess) return fail(FA_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)

#define API_NULL(p) \
  if (!(p)) return fail(FA_ERR_INVALID, std::string(__func__) + ": null argument " #p)

void copy_str(const std::string &s, char *buf, size_t cap) {
  if (!buf || !cap) return;
  size_t n = std::min(cap - 1, s.size());
  std::memcpy(buf, s.data(), n);
  buf[n] = 0;
}

int check_err_flags(Model &m, const SeqState *st_dev) {
  SeqState st;
  API_CUDA(cudaMemcpyAsync(&st, st_dev, sizeof st, cudaMemcpyDeviceToHost, m.stream));
  { const int sync_rc = m.sync(); if (sync_rc) return sync_rc; }
  if (st.err & kErrWaitTimeout) {
    m.step_kv = nullptr;  // the step kernel's phase counters are void: upload a fresh plan next time
    return fail(FA_ERR_TIMEOUT, "a bounded device wait gave up");
  }
  if (st.err & kErrBadToken) return fail(FA_ERR_INVALID, "token id out of range");
  if (st.err & kErrContext) return fail(FA_ERR_CONTEXT, "position or KV capacity exceeded");
  return FA_OK;
}

int set_state(Model &m, SeqState *dst, uint32_t token, uint32_t pos, uint32_t len, uint32_t n_feed) {
  SeqState st{};
  st.pos = pos;
  st.len = len;
  st.token = token;
  st.n_feed = n_feed;
  API_CUDA(cudaMemcpyAsync(dst, &st, sizeof st, cudaMemcpyHostToDevice, m.stream));
  return FA_OK;
}

// captured graphs and the uploaded step plan hold workspace pointers
void drop_graph(Model &m) {
  if (m.graph) {
    cudaGraphExecDestroy(m.graph);
    m.graph = nullptr;
  }
  m.step_kv = nullptr;
}

int ensure_ids(Model &m, uint32_t n) {
  if (n <= m.ws.max_ids) return FA_OK;
  uint32_t cap = std::max<uint32_t>(n, 4096);
  void *p = m.dmalloc((size_t)cap * 4);
  if (!p) return fail(FA_ERR_OOM, "ids allocation failed");
  m.ws.ids = (uint32_t *)p;
  m.ws.max_ids = cap;
  drop_graph(m);
  return FA_OK;
}

int ensure_feed(Model &m, uint32_t n) {
  if (n <= m.ws.max_feed) return FA_OK;
  uint32_t cap = std::max<uint32_t>(n, 4096);
  void *p = m.dmalloc((size_t)cap * 4);
  if (!p) return fail(FA_ERR_OOM, "feed allocation failed");
  m.ws.feed = (uint32_t *)p;
  m.ws.max_feed = cap;
  drop_graph(m);
  return FA_OK;
}

int check_seq(const fa_kv *kv, uint32_t seq, uint64_t n_more) {
  if (seq >= kv->kv.n_seq) return fail(FA_ERR_INVALID, "sequence index out of range");
  if ((uint64_t)kv->kv.len[seq] + n_more > kv->kv.max_ctx) return fail(FA_ERR_CONTEXT, "KV cache capacity exceeded");
  return FA_OK;
}

int create_kv(Model &m, uint32_t n_seq, uint32_t max_ctx, int dtype, KvCache *kv) {
  if (!n_seq || !max_ctx) return fail(FA_ERR_INVALID, "fa_kv_create: zero size");
  if (dtype != FA_KV_F32 && dtype != FA_KV_F16) return fail(FA_ERR_INVALID, "fa_kv_create: bad dtype");
  API_CUDA(cudaSetDevice(m.device));
  kv->m = &m;
  m.live_kv.insert(kv);
  kv->n_seq = n_seq;
  kv->max_ctx = max_ctx;
  kv->max_pages = (max_ctx + 15) / 16;
  kv->f16 = dtype == FA_KV_F16;
  kv->len.assign(n_seq, 0);
  const uint64_t pages = (uint64_t)n_seq * kv->max_pages;
  kv->layer_stride = pages * 2 * m.cfg.n_kv_heads * 16 * m.cfg.head_dim;
  const uint64_t bytes = kv->layer_stride * m.cfg.n_layers * (kv->f16 ? 2 : 4);
  if (cudaMalloc(&kv->base, bytes) != cudaSuccess) {
    cudaGetLastError();  // not sticky: later launch checks must not see it
    kv->base = nullptr;
    return fail(FA_ERR_OOM, "KV cache allocation of " + std::to_string(bytes) + " bytes failed");
  }
  API_CUDA(cudaMemset(kv->base, 0, bytes));
  std::vector<uint32_t> pt(pages);
  for (uint64_t i = 0; i < pages; ++i) pt[i] = (uint32_t)i;  // static page assignment per sequence
  if (cudaMalloc(&kv->page_table, pages * 4) != cudaSuccess) {
    cudaGetLastError();
    kv->page_table = nullptr;
    return fail(FA_ERR_OOM, "page table allocation failed");
  }
  API_CUDA(cudaMemcpy(kv->page_table, pt.data(), pages * 4, cudaMemcpyHostToDevice));
  return m.ensure_rope(max_ctx + 1);
}

// reference multi-token forward: every token at `pos`, all n tokens' K/V
// appended before attention, no mask (src/model.rs:316-455)
int forward_compat(fa_model *fm, fa_kv *kv, uint32_t seq, const uint32_t *tokens, uint32_t n, uint32_t pos,
                   float *logits, uint32_t *argmax, float *hidden) {
  Model &m = fm->m;
  int rc;
  while (fm->compat.size() < n) {
    Workspace w;
    if ((rc = m.alloc_workspace(w))) return rc;
    fm->compat.push_back(w);
  }
  const uint32_t len0 = kv->kv.len[seq], d = m.cfg.n_embd, V = m.cfg.vocab_size;
  for (uint32_t t = 0; t < n; ++t)
    if ((rc = set_state(m, fm->compat[t].state, tokens[t], pos, len0 + t, 0))) return rc;
  // attention of every token sees len0 + n entries: a state with len = len0+n-1
  Workspace &w0 = fm->compat[0];
  SeqState *attn_state = nullptr;
  API_CUDA(cudaMalloc(&attn_state, sizeof(SeqState)));
  struct F {
    void *p;
    ~F() { cudaFree(p); }
  } free_attn{attn_state};
  if ((rc = set_state(m, attn_state, 0, pos, len0 + n - 1, 0))) return rc;
  float *hid_dev = nullptr;
  if (hidden) API_CUDA(cudaMalloc(&hid_dev, (size_t)m.cfg.n_layers * n * d * 4));
  struct F2 {
    void *p;
    ~F2() { cudaFree(p); }
  } free_hid{hid_dev};
  for (uint32_t t = 0; t < n; ++t)
    if ((rc = m.enqueue_embed(fm->compat[t], fm->compat[t].state))) return rc;
  for (uint32_t l = 0; l < m.cfg.n_layers; ++l) {
    for (uint32_t t = 0; t < n; ++t)
      if ((rc = m.enqueue_qkv(l, fm->compat[t], kv->kv, seq, fm->compat[t].state))) return rc;
    for (uint32_t t = 0; t < n; ++t) {
      if ((rc = m.enqueue_attn(l, fm->compat[t], kv->kv, seq, attn_state))) return rc;
      float *dump = hid_dev ? hid_dev + ((size_t)l * n + t) * d : nullptr;
      if ((rc = m.enqueue_post_attn(l, fm->compat[t], fm->compat[t].state, dump))) return rc;
    }
  }
  for (uint32_t t = 0; t < n; ++t) {
    if ((rc = m.enqueue_head(fm->compat[t], fm->compat[t].state))) return rc;
    if (logits) API_CUDA(cudaMemcpyAsync(logits + (size_t)t * V, fm->compat[t].logits, (size_t)V * 4,
                                         cudaMemcpyDeviceToHost, m.stream));
  }
  if (hidden) API_CUDA(cudaMemcpyAsync(hidden, hid_dev, (size_t)m.cfg.n_layers * n * d * 4, cudaMemcpyDeviceToHost, m.stream));
  { const int sync_rc = m.sync(); if (sync_rc) return sync_rc; }
  for (uint32_t t = 0; t < n; ++t) {
    if ((rc = check_err_flags(m, fm->compat[t].state))) return rc;
    if (argmax) {
      SeqState st;
      API_CUDA(cudaMemcpy(&st, fm->compat[t].state, sizeof st, cudaMemcpyDeviceToHost));
      argmax[t] = ~(uint32_t)(st.argmax_key & 0xFFFFFFFFull);
    }
  }
  (void)w0;
  kv->kv.len[seq] = len0 + n;
  return FA_OK;
}

}  // namespace

struct fa_sampler {
  fa_sampler_config cfg{};
  uint32_t n_seq = 0, vocab = 0, pow2 = 0;
  int device = 0;
  cudaStream_t stream = nullptr;
  uint32_t *freq = nullptr, *ids = nullptr;
  uint64_t *seeds = nullptr, *counters = nullptr;
  float *probs = nullptr, *in = nullptr;
  unsigned long long *keys = nullptr;
  ~fa_sampler() {
    cudaSetDevice(device);
    if (stream) cudaStreamSynchronize(stream);
    for (void *q : {(void *)freq, (void *)ids, (void *)seeds, (void *)counters, (void *)probs, (void *)in, (void *)keys})
      if (q) cudaFree(q);
    if (stream) cudaStreamDestroy(stream);
  }
  SamplerParams params(uint32_t n) const {
    SamplerParams p{};
    p.temperature = cfg.temperature;
    p.top_p = cfg.top_p;
    p.rep = cfg.repetition_penalty;
    p.freq_pen = cfg.frequency_penalty;
    p.pres_pen = cfg.presence_penalty;
    p.top_k = cfg.top_k;
    p.n = n;
    p.ld = n;
    p.vocab = vocab;
    p.freq = freq;
    p.seeds = seeds;
    p.counters = counters;
    p.probs = probs;
    p.keys = keys;
    p.pow2 = pow2;
    p.ids = ids;
    return p;
  }
};

namespace {
// the whole-row sort scratch, allocated on first use
int sampler_keys(fa_sampler *s, SamplerParams &p) {
  if (!sample_needs_sort(p) || s->keys) return FA_OK;
  uint32_t p2 = 2;
  while (p2 < s->vocab) p2 <<= 1;
  if (cudaMalloc(&s->keys, (size_t)s->n_seq * p2 * sizeof(unsigned long long)) != cudaSuccess)
    return fail(FA_ERR_OOM, "sampler sort scratch allocation failed");
  s->pow2 = p2;
  p.keys = s->keys;
  p.pow2 = p2;
  return FA_OK;
}

int sampler_new(const fa_sampler_config &cfg, uint32_t n_seq, uint32_t vocab, const uint64_t *seeds,
                std::unique_ptr<fa_sampler> *out) {
  if (!n_seq || !vocab) return fail(FA_ERR_INVALID, "fa_sampler_create: zero size");
  std::unique_ptr<fa_sampler> s(new (std::nothrow) fa_sampler());
  if (!s) return fail(FA_ERR_OOM, "sampler allocation failed");
  s->cfg = cfg;
  s->n_seq = n_seq;
  s->vocab = vocab;
  API_CUDA(cudaGetDevice(&s->device));
  if (sampler_init()) return fail(FA_ERR_CUDA, "sampler kernel setup failed");
  API_CUDA(cudaStreamCreateWithFlags(&s->stream, cudaStreamNonBlocking));
  const size_t rows = (size_t)n_seq * vocab;
  API_CUDA(cudaMalloc(&s->freq, rows * 4));
  API_CUDA(cudaMalloc(&s->probs, rows * 4));
  API_CUDA(cudaMalloc(&s->in, (size_t)vocab * 4));
  API_CUDA(cudaMalloc(&s->ids, (size_t)n_seq * 4));
  API_CUDA(cudaMalloc(&s->seeds, (size_t)n_seq * 8));
  API_CUDA(cudaMalloc(&s->counters, (size_t)n_seq * 8));
  API_CUDA(cudaMemset(s->freq, 0, rows * 4));
  API_CUDA(cudaMemset(s->counters, 0, (size_t)n_seq * 8));
  std::vector<uint64_t> sd(n_seq);
  for (uint32_t i = 0; i < n_seq; ++i) sd[i] = seeds ? seeds[i] : i;
  API_CUDA(cudaMemcpy(s->seeds, sd.data(), (size_t)n_seq * 8, cudaMemcpyHostToDevice));
  *out = std::move(s);
  return FA_OK;
}
}  // namespace

extern "C" {

size_t fa_last_error(char *buf, size_t cap) {
  copy_str(last_error(), buf, cap);
  return last_error().size();
}

const char *fa_version(void) { return "fishai-b200 0.1.0 (sm_100a)"; }

// ------------------------------------------------------------------ GGUF
int fa_gguf_open(const char *path, fa_gguf **out) {
  API_NULL(path);
  API_NULL(out);
  int code = FA_OK;
  Gguf *g = Gguf::open(path, &code);
  if (!g) return code;
  *out = new (std::nothrow) fa_gguf();
  if (!*out) {
    delete g;
    return fail(FA_ERR_OOM, "out of memory");
  }
  (*out)->g.reset(g);
  return FA_OK;
}
void fa_gguf_close(fa_gguf *g) { delete g; }
int fa_gguf_version(const fa_gguf *g, uint32_t *v) {
  API_NULL(g);
  API_NULL(v);
  *v = g->g->version;
  return FA_OK;
}
int fa_gguf_alignment(const fa_gguf *g, uint64_t *a) {
  API_NULL(g);
  API_NULL(a);
  *a = g->g->alignment;
  return FA_OK;
}
int fa_gguf_tensor_count(const fa_gguf *g, size_t *n) {
  API_NULL(g);
  API_NULL(n);
  *n = g->g->tensors.size();
  return FA_OK;
}
static void fill_tinfo(const GgufTensor &t, uint32_t *n_dims, uint64_t dims[4], uint32_t *type, uint64_t *offset) {
  if (n_dims) *n_dims = t.n_dims;
  if (dims)
    for (int i = 0; i < 4; ++i) dims[i] = t.dims[i];
  if (type) *type = t.ggml_type;
  if (offset) *offset = t.offset;
}
int fa_gguf_tensor_at(const fa_gguf *g, size_t i, char *name, size_t cap, uint32_t *n_dims, uint64_t dims[4],
                      uint32_t *type, uint64_t *offset) {
  API_NULL(g);
  if (i >= g->g->tensors.size()) return fail(FA_ERR_INVALID, "tensor index out of range");
  const GgufTensor &t = g->g->tensors[i];
  copy_str(t.name, name, cap);
  fill_tinfo(t, n_dims, dims, type, offset);
  return FA_OK;
}
int fa_gguf_tensor_info(const fa_gguf *g, const char *name, uint32_t *n_dims, uint64_t dims[4], uint32_t *type,
                        uint64_t *offset) {
  API_NULL(g);
  API_NULL(name);
  const GgufTensor *t = g->g->tensor(name);
  if (!t) return fail(FA_ERR_INVALID, std::string("tensor not found: ") + name);
  fill_tinfo(*t, n_dims, dims, type, offset);
  return FA_OK;
}
int fa_gguf_read_tensor_data(const fa_gguf *g, const char *name, void *out, size_t cap, size_t *size) {
  API_NULL(g);
  API_NULL(name);
  API_NULL(size);
  *size = 0;
  const GgufTensor *t = g->g->tensor(name);
  if (!t) return fail(FA_ERR_INVALID, std::string("tensor not found: ") + name);
  size_t n = 0;
  const uint8_t *p = g->g->tensor_data(*t, &n);
  if (!p) return FA_OK;
  *size = n;
  if (out) std::memcpy(out, p, std::min(n, cap));
  return FA_OK;
}
int fa_gguf_meta_u64(const fa_gguf *g, const char *key, uint64_t *v, int *found) {
  API_NULL(g);
  API_NULL(key);
  API_NULL(found);
  uint64_t x = 0;
  *found = g->g->meta_u64(key, &x);
  if (v && *found) *v = x;
  return FA_OK;
}
int fa_gguf_meta_i64(const fa_gguf *g, const char *key, int64_t *v, int *found) {
  API_NULL(g);
  API_NULL(key);
  API_NULL(found);
  int64_t x = 0;
  *found = g->g->meta_i64(key, &x);
  if (v && *found) *v = x;
  return FA_OK;
}
int fa_gguf_meta_f32(const fa_gguf *g, const char *key, float *v, int *found) {
  API_NULL(g);
  API_NULL(key);
  API_NULL(found);
  float x = 0;
  *found = g->g->meta_f32(key, &x);
  if (v && *found) *v = x;
  return FA_OK;
}
int fa_gguf_meta_bool(const fa_gguf *g, const char *key, int *v, int *found) {
  API_NULL(g);
  API_NULL(key);
  API_NULL(found);
  bool x = false;
  *found = g->g->meta_bool(key, &x);
  if (v && *found) *v = x;
  return FA_OK;
}
int fa_gguf_meta_string(const fa_gguf *g, const char *key, char *buf, size_t cap, int *found) {
  API_NULL(g);
  API_NULL(key);
  API_NULL(found);
  std::string s;
  *found = g->g->meta_string(key, &s);
  if (*found) copy_str(s, buf, cap);
  return FA_OK;
}
int fa_gguf_vocab_size(const fa_gguf *g, uint64_t *v, int *found) {
  API_NULL(g);
  API_NULL(found);
  uint64_t x = 0;
  *found = g->g->vocab_size(&x);
  if (v && *found) *v = x;
  return FA_OK;
}

// ------------------------------------------------------------ config
int fa_tokenizer_from_gguf(const fa_gguf *g, fa_tokenizer **out) {
  API_NULL(g);
  API_NULL(out);
  return tokenizer_from_gguf(*g->g, out);
}

int fa_config_from_gguf(const fa_gguf *g, fa_config *cfg) {
  API_NULL(g);
  API_NULL(cfg);
  return config_from_gguf(*g->g, cfg);
}
uint32_t fa_config_n_ff(uint32_t n_embd, float mult) { return n_ff_of(n_embd, mult); }

// ------------------------------------------------------------ dequant
int fa_dequantize_device(int type, const void *bytes_dev, size_t nbytes, size_t count, float *out_dev, void *stream) {
  API_NULL(out_dev);
  if (!type_known(type)) return fail(FA_ERR_UNSUPPORTED, "Unsupported ggml type for dequantization: " + std::to_string(type));
  const size_t be = block_elems(type), bb = block_bytes(type);
  const size_t whole = nbytes / bb * be;  // elements backed by complete blocks
  const size_t n = std::min(count, whole);
  if (type == FA_GGML_F32 && nbytes < count * 4) return fail(FA_ERR_INVALID, "Not enough data for F32");
  if (n && launch_dequant_native(type, bytes_dev, n, out_dev, (cudaStream_t)stream))
    return fail(FA_ERR_CUDA, "dequant launch failed");
  return FA_OK;
}

int fa_dequantize(int type, const void *bytes, size_t nbytes, size_t count, float *out, size_t *n_out) {
  API_NULL(out);
  if (!type_known(type)) return fail(FA_ERR_UNSUPPORTED, "Unsupported ggml type for dequantization: " + std::to_string(type));
  if (type == FA_GGML_F32 && nbytes < count * 4) return fail(FA_ERR_INVALID, "Not enough data for F32");
  const size_t be = block_elems(type), bb = block_bytes(type);
  // the reference stops at the first incomplete block (src/quant.rs:130)
  const size_t n = std::min(count, nbytes / bb * be);
  if (n_out) *n_out = n;
  if (!n) return FA_OK;
  void *d_in = nullptr;
  float *d_out = nullptr;
  API_CUDA(cudaMalloc(&d_in, nbytes));
  if (cudaMalloc(&d_out, n * 4) != cudaSuccess) {
    cudaFree(d_in);
    return fail(FA_ERR_OOM, "device allocation failed");
  }
  int rc = FA_OK;
  if (cudaMemcpy(d_in, bytes, nbytes, cudaMemcpyHostToDevice) != cudaSuccess ||
      launch_dequant_native(type, d_in, n, d_out, nullptr) ||
      cudaMemcpy(out, d_out, n * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = fail(FA_ERR_CUDA, std::string("dequantize failed: ") + cudaGetErrorString(cudaGetLastError()));
  cudaFree(d_in);
  cudaFree(d_out);
  return rc;
}

// ------------------------------------------------------------ model
void fa_model_opts_default(fa_model_opts *o) {
  if (!o) return;
  std::memset(o, 0, sizeof *o);
  o->use_graphs = 1;
  o->use_pdl = 1;
  o->tp_world = 1;
}

int fa_model_load(const char *path, const fa_model_opts *opts, fa_model **out) {
  API_NULL(path);
  API_NULL(out);
  fa_model_opts o;
  if (opts) o = *opts;
  else fa_model_opts_default(&o);
  fa_model *m = new (std::nothrow) fa_model();
  if (!m) return fail(FA_ERR_OOM, "out of memory");
  int rc = m->m.load(path, o);
  if (rc) {
    std::string e = last_error();
    delete m;
    return fail(rc, e);
  }
  *out = m;
  return FA_OK;
}
void fa_model_free(fa_model *m) { delete m; }
int fa_model_config(const fa_model *m, fa_config *cfg) {
  API_NULL(m);
  API_NULL(cfg);
  *cfg = m->m.gcfg;
  return FA_OK;
}
int fa_model_tp(const fa_model *m, int32_t *rank, int32_t *world, uint32_t *local_heads, uint32_t *local_kv_heads,
                uint32_t *local_ff) {
  API_NULL(m);
  if (rank) *rank = m->m.tp.rank;
  if (world) *world = m->m.tp.world;
  if (local_heads) *local_heads = m->m.cfg.n_heads;
  if (local_kv_heads) *local_kv_heads = m->m.cfg.n_kv_heads;
  if (local_ff) *local_ff = m->m.cfg.n_ff_used;
  return FA_OK;
}
int fa_tp_unique_id(void *out128) {
  API_NULL(out128);
  std::string msg;
  if (tp_unique_id(out128, &msg)) return fail(FA_ERR_NCCL, "ncclGetUniqueId: " + msg);
  return FA_OK;
}
int fa_tp_shard(int32_t ggml_type, const void *bytes_host, uint32_t K, uint32_t N, int32_t axis, uint32_t rank,
                uint32_t world, void *out_host, size_t cap, size_t *out_bytes, uint32_t *row_bytes) {
  API_NULL(bytes_host);
  API_NULL(out_bytes);
  if (!world || rank >= world) return fail(FA_ERR_INVALID, "fa_tp_shard: rank out of range");
  const uint32_t rb = native_row_bytes(ggml_type, N);
  if (!type_known(ggml_type) || !rb) return fail(FA_ERR_UNSUPPORTED, "fa_tp_shard: unsupported type");
  const uint8_t *src = (const uint8_t *)bytes_host;
  if (axis == 0) {  // rows
    if (K % world) return fail(FA_ERR_INVALID, "fa_tp_shard: rows do not divide by world");
    const uint32_t nr = K / world;
    *out_bytes = (size_t)nr * rb;
    if (row_bytes) *row_bytes = rb;
    if (out_host) std::memcpy(out_host, tp_rows(src, rb, rank * nr), std::min(cap, *out_bytes));
    return FA_OK;
  }
  if (N % world) return fail(FA_ERR_INVALID, "fa_tp_shard: columns do not divide by world");
  const uint32_t nc = N / world;
  std::vector<uint8_t> buf;
  uint32_t srb = 0;
  if (tp_shard_columns(ggml_type, src, K, N, rank * nc, (rank + 1) * nc, buf, &srb))
    return fail(FA_ERR_UNSUPPORTED, "fa_tp_shard: column shard does not fall on block boundaries");
  *out_bytes = buf.size();
  if (row_bytes) *row_bytes = srb;
  if (out_host) std::memcpy(out_host, buf.data(), std::min(cap, buf.size()));
  return FA_OK;
}
int fa_model_weight_bytes(const fa_model *m, uint64_t *device_bytes, uint64_t *step_bytes) {
  API_NULL(m);
  if (device_bytes) *device_bytes = m->m.device_bytes;
  if (step_bytes) *step_bytes = m->m.step_bytes;
  return FA_OK;
}
void *fa_model_stream(fa_model *m) { return m ? (void *)m->m.stream : nullptr; }
int fa_model_step_kernel_active(const fa_model *m) { return m && m->m.step_ok ? 1 : 0; }
int fa_model_set_tc_prefill(fa_model *m, int32_t on) {
  API_NULL(m);
  if (on && !m->m.tc_ok) return fail(FA_ERR_UNSUPPORTED, "tensor-core prefill needs every projection in the MMA layout");
  m->m.want_tc_prefill = on != 0;
  return FA_OK;
}
int fa_debug_set(fa_model *fm, int32_t key, uint64_t value) {
  API_NULL(fm);
  Model &m = fm->m;
  if (key == FA_DEBUG_WAIT_LIMIT_NS) m.dbg_wait_ns = value;
  else if (key == FA_DEBUG_WITHHOLD_WEIGHTS) m.dbg_withhold = value ? 1u : 0u;
  else if (key == FA_DEBUG_FIXED_ORDER_SUMS) m.dbg_fixed_order = value != 0;
  else return fail(FA_ERR_INVALID, "fa_debug_set: unknown key");
  drop_graph(m);  // captured launches hold the old parameters
  return FA_OK;
}
int fa_model_step_launches(const fa_model *m, uint32_t *n) {
  API_NULL(m);
  API_NULL(n);
  *n = m->m.graph ? m->m.graph_kernels : 0;
  return FA_OK;
}

// ------------------------------------------------------------ KV cache
int fa_kv_create(fa_model *m, uint32_t n_seq, uint32_t max_ctx, int32_t dtype, fa_kv **out) {
  API_NULL(m);
  API_NULL(out);
  fa_kv *kv = new (std::nothrow) fa_kv();
  if (!kv) return fail(FA_ERR_OOM, "out of memory");
  int rc = create_kv(m->m, n_seq, max_ctx, dtype, &kv->kv);
  if (rc) {
    std::string e = last_error();
    delete kv;
    return fail(rc, e);
  }
  *out = kv;
  return FA_OK;
}
void fa_kv_free(fa_kv *kv) { delete kv; }
int fa_kv_clear(fa_kv *kv, int32_t seq) {
  API_NULL(kv);
  if (seq < 0) {
    std::fill(kv->kv.len.begin(), kv->kv.len.end(), 0u);
    return FA_OK;
  }
  if ((uint32_t)seq >= kv->kv.n_seq) return fail(FA_ERR_INVALID, "sequence index out of range");
  kv->kv.len[seq] = 0;
  return FA_OK;
}
int fa_kv_seq_len(const fa_kv *kv, uint32_t seq, uint32_t *len) {
  API_NULL(kv);
  API_NULL(len);
  if (seq >= kv->kv.n_seq) return fail(FA_ERR_INVALID, "sequence index out of range");
  *len = kv->kv.len[seq];
  return FA_OK;
}
int fa_kv_get(const fa_kv *kv, uint32_t seq, uint32_t layer, float *k_host, float *v_host) {
  API_NULL(kv);
  const KvCache &c = kv->kv;
  if (seq >= c.n_seq) return fail(FA_ERR_INVALID, "sequence index out of range");
  if (layer >= c.m->cfg.n_layers)
    return fail(FA_ERR_INVALID, "KV cache layer index out of range: " + std::to_string(layer));
  const uint32_t KVH = c.m->cfg.n_kv_heads, hd = c.m->cfg.head_dim, len = c.len[seq];
  const uint32_t pages = (len + 15) / 16;
  const size_t page_elems = (size_t)2 * KVH * 16 * hd, esz = c.f16 ? 2 : 4;
  std::vector<uint8_t> buf(page_elems * esz);
  std::vector<uint32_t> pt(c.max_pages);
  API_CUDA(cudaMemcpy(pt.data(), c.page_table + (size_t)seq * c.max_pages, c.max_pages * 4, cudaMemcpyDeviceToHost));
  for (uint32_t p = 0; p < pages; ++p) {
    const uint8_t *src = (const uint8_t *)c.base + ((size_t)layer * c.layer_stride + (size_t)pt[p] * page_elems) * esz;
    API_CUDA(cudaMemcpy(buf.data(), src, buf.size(), cudaMemcpyDeviceToHost));
    for (uint32_t s = 0; s < 16 && p * 16 + s < len; ++s)
      for (uint32_t h = 0; h < KVH; ++h)
        for (uint32_t dd = 0; dd < hd; ++dd)
          for (int isv = 0; isv < 2; ++isv) {
            const size_t idx = kv_index(0, isv, h, s, dd, KVH, hd);
            float v;
            if (c.f16) v = f16_to_f32(((const uint16_t *)buf.data())[idx]);
            else v = ((const float *)buf.data())[idx];
            float *dst = isv ? v_host : k_host;
            if (dst) dst[((size_t)(p * 16 + s) * KVH + h) * hd + dd] = v;
          }
  }
  return FA_OK;
}

// ------------------------------------------------------------ forward
int fa_forward(fa_model *fm, fa_kv *kv, uint32_t seq, const uint32_t *tokens, uint32_t n, uint32_t pos, float *logits,
               uint32_t *argmax, float *hidden) {
  API_NULL(fm);
  API_NULL(kv);
  API_NULL(tokens);
  if (!n) return fail(FA_ERR_INVALID, "fa_forward: empty token list");
  Model &m = fm->m;
  int rc;
  if ((rc = check_seq(kv, seq, n))) return rc;
  for (uint32_t i = 0; i < n; ++i)
    if (tokens[i] >= m.cfg.vocab_size) return fail(FA_ERR_INVALID, "token id out of range");
  if ((rc = m.ensure_rope(pos + 1))) return rc;
  API_CUDA(cudaSetDevice(m.device));
  if (n > 1) return forward_compat(fm, kv, seq, tokens, n, pos, logits, argmax, hidden);
  float *hid_dev = nullptr;
  if (hidden) API_CUDA(cudaMalloc(&hid_dev, (size_t)m.cfg.n_layers * m.cfg.n_embd * 4));
  struct F {
    void *p;
    ~F() { cudaFree(p); }
  } free_hid{hid_dev};
  // the step's state crosses PCIe through the model's pinned staging
  // buffer: one 40-byte upload, one 40-byte read-back (plus the logits row
  // when asked for)
  *m.h_state = SeqState{};
  m.h_state->pos = pos;
  m.h_state->len = kv->kv.len[seq];
  m.h_state->token = tokens[0];
  API_CUDA(cudaMemcpyAsync(m.ws.state, m.h_state, sizeof(SeqState), cudaMemcpyHostToDevice, m.stream));
  if (hidden) {
    if ((rc = m.enqueue_step(kv->kv, seq, m.ws, hid_dev))) return rc;
  } else {
    if ((rc = m.run_steps(kv->kv, seq, 1))) return rc;
  }
  if (logits)
    API_CUDA(cudaMemcpyAsync(logits, m.ws.logits, (size_t)m.cfg.vocab_size * 4, cudaMemcpyDeviceToHost, m.stream));
  if (hidden)
    API_CUDA(cudaMemcpyAsync(hidden, hid_dev, (size_t)m.cfg.n_layers * m.cfg.n_embd * 4, cudaMemcpyDeviceToHost, m.stream));
  API_CUDA(cudaMemcpyAsync(m.h_state, m.ws.state, sizeof(SeqState), cudaMemcpyDeviceToHost, m.stream));
  { const int sync_rc = m.sync(); if (sync_rc) return sync_rc; }
  const SeqState st = *m.h_state;
  if (st.err) return check_err_flags(m, m.ws.state);
  if (argmax) argmax[0] = st.token;
  kv->kv.len[seq] += 1;
  return FA_OK;
}

int fa_prefill(fa_model *fm, fa_kv *kv, uint32_t seq, const uint32_t *tokens, uint32_t n, uint32_t start_pos,
               float *last_logits, uint32_t *last_argmax) {
  API_NULL(fm);
  API_NULL(kv);
  API_NULL(tokens);
  if (!n) return fail(FA_ERR_INVALID, "fa_prefill: empty token list");
  Model &m = fm->m;
  int rc;
  if ((rc = check_seq(kv, seq, n))) return rc;
  for (uint32_t i = 0; i < n; ++i)
    if (tokens[i] >= m.cfg.vocab_size) return fail(FA_ERR_INVALID, "token id out of range");
  if ((rc = m.ensure_rope(start_pos + n))) return rc;
  API_CUDA(cudaSetDevice(m.device));
  if (m.want_tc_prefill && m.tc_ok) {  // bf16 tensor-core path
    if ((rc = m.prefill_tc(kv->kv, seq, tokens, n, start_pos))) return rc;
    if (last_logits)
      API_CUDA(cudaMemcpyAsync(last_logits, m.ws.logits, (size_t)m.cfg.vocab_size * 4, cudaMemcpyDeviceToHost, m.stream));
    SeqState st;
    API_CUDA(cudaMemcpyAsync(&st, m.ws.state, sizeof st, cudaMemcpyDeviceToHost, m.stream));
    { const int sync_rc = m.sync(); if (sync_rc) return sync_rc; }
    if (last_argmax) *last_argmax = ~(uint32_t)(st.argmax_key & 0xFFFFFFFFull);
    kv->kv.len[seq] += n;
    return FA_OK;
  }
  if ((rc = ensure_feed(m, n)) || (rc = ensure_ids(m, n))) return rc;
  API_CUDA(cudaMemcpyAsync(m.ws.feed, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, m.stream));
  if ((rc = set_state(m, m.ws.state, 0, start_pos, kv->kv.len[seq], n))) return rc;
  if ((rc = m.run_steps(kv->kv, seq, n))) return rc;
  if (last_logits)
    API_CUDA(cudaMemcpyAsync(last_logits, m.ws.logits, (size_t)m.cfg.vocab_size * 4, cudaMemcpyDeviceToHost, m.stream));
  SeqState st;
  API_CUDA(cudaMemcpyAsync(&st, m.ws.state, sizeof st, cudaMemcpyDeviceToHost, m.stream));
  { const int sync_rc = m.sync(); if (sync_rc) return sync_rc; }
  if (st.err) return check_err_flags(m, m.ws.state);
  if (last_argmax) *last_argmax = st.token;
  kv->kv.len[seq] += n;
  return FA_OK;
}

int fa_decode_greedy(fa_model *fm, fa_kv *kv, uint32_t seq, uint32_t first_token, uint32_t pos, uint32_t steps,
                     uint32_t *ids_host) {
  API_NULL(fm);
  API_NULL(kv);
  Model &m = fm->m;
  int rc;
  if ((rc = check_seq(kv, seq, steps))) return rc;
  if (first_token >= m.cfg.vocab_size) return fail(FA_ERR_INVALID, "token id out of range");
  if ((rc = m.ensure_rope(pos + steps))) return rc;
  API_CUDA(cudaSetDevice(m.device));
  if ((rc = ensure_ids(m, steps))) return rc;
  if ((rc = set_state(m, m.ws.state, first_token, pos, kv->kv.len[seq], 0))) return rc;
  if ((rc = m.run_steps(kv->kv, seq, steps))) return rc;
  if (ids_host) API_CUDA(cudaMemcpyAsync(ids_host, m.ws.ids, (size_t)steps * 4, cudaMemcpyDeviceToHost, m.stream));
  { const int sync_rc = m.sync(); if (sync_rc) return sync_rc; }
  if ((rc = check_err_flags(m, m.ws.state))) return rc;
  kv->kv.len[seq] += steps;
  return FA_OK;
}

// ------------------------------------------------------------ generation
int fa_generate(fa_model *fm, const fa_gen_config *cfg, const uint32_t *prompt, uint32_t n_prompt, uint32_t *out,
                uint32_t cap, uint32_t *n_out) {
  API_NULL(fm);
  API_NULL(cfg);
  API_NULL(prompt);
  API_NULL(n_out);
  *n_out = 0;
  // token_ids.last().unwrap() panics on an empty prompt in the reference
  if (!n_prompt) return fail(FA_ERR_INVALID, "fa_generate: empty prompt");
  Model &m = fm->m;
  const uint32_t P = n_prompt, steps = std::max(P, cfg->max_tokens), G = steps - P;
  for (uint32_t i = 0; i < P; ++i)
    if (prompt[i] >= m.cfg.vocab_size) return fail(FA_ERR_INVALID, "token id out of range");
  int rc;
  fa_kv kvh;
  if ((rc = create_kv(m, 1, steps + 1, cfg->kv_dtype, &kvh.kv))) return rc;
  if ((rc = ensure_feed(m, P + 1)) || (rc = ensure_ids(m, steps))) return rc;
  // Sampler::sample after every generated step on the device: its id is the
  // next input and is observed; Sampler::reset per call (src/model.rs:645)
  std::unique_ptr<fa_sampler> smp;
  const uint64_t seed = cfg->seed;
  if ((rc = sampler_new(cfg->sampler, 1, m.cfg.vocab_size, &seed, &smp))) return rc;
  SamplerParams sp = smp->params(m.cfg.vocab_size);
  if ((rc = sampler_keys(smp.get(), sp))) return rc;
  sp.logits = m.ws.logits;
  sp.state = m.ws.state;
  sp.gen_ids = m.ws.ids;
  sp.max_ids = m.ws.max_ids;
  sp.sample_from = P;
  sp.observe = 1;
  drop_graph(m);
  m.gen_sample = &sp;
  struct Unhook {
    Model &m;
    ~Unhook() {
      m.gen_sample = nullptr;
      drop_graph(m);
    }
  } unhook{m};
  std::vector<uint32_t> feed(prompt, prompt + P);
  feed.push_back(prompt[P - 1]);  // generate_step re-feeds the last prompt token (src/model.rs:656-657)
  API_CUDA(cudaMemcpyAsync(m.ws.feed, feed.data(), feed.size() * 4, cudaMemcpyHostToDevice, m.stream));
  if ((rc = set_state(m, m.ws.state, 0, 0, 0, G ? P + 1 : P))) return rc;
  std::vector<uint32_t> ids(steps);
  uint32_t done = 0;
  bool stopped = false;
  uint32_t n_gen = 0;
  while (done < steps && !stopped) {
    const uint32_t chunk = std::min<uint32_t>(steps - done, cfg->n_stop ? 32 : steps);
    if ((rc = m.run_steps(kvh.kv, 0, chunk))) return rc;
    API_CUDA(cudaMemcpyAsync(ids.data() + done, m.ws.ids + done, (size_t)chunk * 4, cudaMemcpyDeviceToHost, m.stream));
    { const int sync_rc = m.sync(); if (sync_rc) return sync_rc; }
    for (uint32_t s = done; s < done + chunk; ++s) {
      if (s < P) continue;  // prefill logits are discarded
      const uint32_t t = ids[s];
      for (uint32_t j = 0; j < cfg->n_stop; ++j)
        if (cfg->stop_ids[j] == t) stopped = true;
      if (stopped) break;
      if (out && n_gen < cap) out[n_gen] = t;
      ++n_gen;
    }
    done += chunk;
  }
  if ((rc = check_err_flags(m, m.ws.state))) return rc;
  *n_out = n_gen;
  return FA_OK;
}

// ------------------------------------------------------------ sampler
int fa_sampler_create(const fa_sampler_config *cfg, uint32_t n_seq, uint32_t vocab, const uint64_t *seeds,
                      fa_sampler **out) {
  API_NULL(cfg);
  API_NULL(out);
  *out = nullptr;
  std::unique_ptr<fa_sampler> s;
  const int rc = sampler_new(*cfg, n_seq, vocab, seeds, &s);
  if (rc) return rc;
  *out = s.release();
  return FA_OK;
}

void fa_sampler_free(fa_sampler *s) { delete s; }

int fa_sample_device(fa_sampler *s, const float *logits_dev, uint32_t n, uint32_t *ids_dev, uint32_t *ids_host,
                     void *stream) {
  API_NULL(s);
  API_NULL(logits_dev);
  if (!n || n > s->n_seq) return fail(FA_ERR_INVALID, "fa_sample_device: row count out of range");
  API_CUDA(cudaSetDevice(s->device));
  cudaStream_t st = stream ? (cudaStream_t)stream : s->stream;
  SamplerParams p = s->params(s->vocab);
  p.logits = logits_dev;
  if (ids_dev) p.ids = ids_dev;
  int rc;
  if ((rc = sampler_keys(s, p))) return rc;
  if (launch_sample(p, n, st)) return fail(FA_ERR_CUDA, "sampler launch failed");
  if (ids_host) {
    API_CUDA(cudaMemcpyAsync(ids_host, p.ids, (size_t)n * 4, cudaMemcpyDeviceToHost, st));
    API_CUDA(cudaStreamSynchronize(st));
  }
  return FA_OK;
}

int fa_sample(fa_sampler *s, uint32_t seq, const float *logits_host, uint32_t vocab, uint32_t *id_host) {
  API_NULL(s);
  API_NULL(id_host);
  if (seq >= s->n_seq) return fail(FA_ERR_INVALID, "fa_sample: sequence index out of range");
  if (vocab > s->vocab) return fail(FA_ERR_INVALID, "fa_sample: more logits than the sampler's vocabulary");
  if (!vocab) {  // argmax of an empty vector is 0 (src/sampling.rs:297-310)
    *id_host = 0;
    return FA_OK;
  }
  API_NULL(logits_host);
  API_CUDA(cudaSetDevice(s->device));
  SamplerParams p = s->params(vocab);
  p.row0 = seq;
  p.logits = s->in;
  int rc;
  if ((rc = sampler_keys(s, p))) return rc;
  API_CUDA(cudaMemcpyAsync(s->in, logits_host, (size_t)vocab * 4, cudaMemcpyHostToDevice, s->stream));
  if (launch_sample(p, 1, s->stream)) return fail(FA_ERR_CUDA, "sampler launch failed");
  API_CUDA(cudaMemcpyAsync(id_host, s->ids + seq, 4, cudaMemcpyDeviceToHost, s->stream));
  API_CUDA(cudaStreamSynchronize(s->stream));
  return FA_OK;
}

int fa_sampler_observe(fa_sampler *s, uint32_t seq, uint32_t token) {
  API_NULL(s);
  if (seq >= s->n_seq) return fail(FA_ERR_INVALID, "fa_sampler_observe: sequence index out of range");
  // ids at or beyond the vocabulary cannot change a sample of <= vocab logits
  if (token >= s->vocab) return FA_OK;
  API_CUDA(cudaSetDevice(s->device));
  if (launch_sampler_observe(s->freq, s->vocab, seq, token, s->stream)) return fail(FA_ERR_CUDA, "observe launch failed");
  API_CUDA(cudaStreamSynchronize(s->stream));
  return FA_OK;
}

int fa_sampler_reset(fa_sampler *s, int32_t seq) {
  API_NULL(s);
  if (seq >= (int32_t)s->n_seq) return fail(FA_ERR_INVALID, "fa_sampler_reset: sequence index out of range");
  API_CUDA(cudaSetDevice(s->device));
  const size_t row = (size_t)s->vocab * 4;
  if (seq < 0) API_CUDA(cudaMemsetAsync(s->freq, 0, row * s->n_seq, s->stream));
  else API_CUDA(cudaMemsetAsync((uint8_t *)s->freq + row * seq, 0, row, s->stream));
  API_CUDA(cudaStreamSynchronize(s->stream));
  return FA_OK;
}

int fa_sampler_freq(fa_sampler *s, uint32_t seq, uint32_t token, uint32_t *count) {
  API_NULL(s);
  API_NULL(count);
  if (seq >= s->n_seq) return fail(FA_ERR_INVALID, "fa_sampler_freq: sequence index out of range");
  *count = 0;
  if (token >= s->vocab) return FA_OK;
  API_CUDA(cudaSetDevice(s->device));
  API_CUDA(cudaStreamSynchronize(s->stream));
  API_CUDA(cudaMemcpy(count, s->freq + (size_t)seq * s->vocab + token, 4, cudaMemcpyDeviceToHost));
  return FA_OK;
}

// ------------------------------------------------------------ attention
}  // extern "C"
namespace fa {
int sdpa_check(const char *who, const float *q, const float *k, const float *v, uint32_t q_len, uint32_t kv_len,
               uint32_t H, uint32_t KVH, uint32_t hd, const float *out) {
  const std::string w(who);
  if (!q || !k || !v || !out) return fail(FA_ERR_INVALID, w + ": null buffer");
  if (!q_len || !kv_len || !H || !KVH || !hd) return fail(FA_ERR_INVALID, w + ": zero size");
  if (hd > 128 || H % KVH || (H / KVH != 1 && H / KVH != 2 && H / KVH != 4 && H / KVH != 8))
    return fail(FA_ERR_UNSUPPORTED, w + ": head_dim <= 128 and n_heads/n_kv_heads in {1,2,4,8}");
  return FA_OK;
}

AttnParams sdpa_params(const float *q, const float *k, const float *v, uint32_t q_len, uint32_t kv_len, uint32_t H,
                       uint32_t KVH, uint32_t hd, float *out, float *part, uint32_t *counters) {
  AttnParams ap{};
  ap.q = q;
  ap.kc = k;
  ap.vc = v;
  ap.t_fixed = kv_len;
  ap.q_rows = q_len;
  ap.kv.n_kv = KVH;
  ap.kv.head_dim = hd;
  ap.kv.f16 = 0;
  ap.n_heads = H;
  ap.splits = kSdpaSplits;
  ap.scale = 1.0f / std::sqrt((float)hd);  // src/tensor.rs:486
  ap.part = part;
  ap.counters = counters;
  ap.out = out;
  return ap;
}
}  // namespace fa

namespace {
std::mutex g_sdpa_mu;
struct SdpaScratch {
  void *buf = nullptr;
  size_t bytes = 0;
};
SdpaScratch g_sdpa[64];  // per device
}  // namespace
extern "C" {

int fa_sdpa(const float *q, const float *k, const float *v, uint32_t q_len, uint32_t kv_len, uint32_t H, uint32_t KVH,
            uint32_t hd, float *out, void *stream) {
  int rc = sdpa_check("fa_sdpa", q, k, v, q_len, kv_len, H, KVH, hd, out);
  if (rc) return rc;
  int dev = 0;
  API_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return fail(FA_ERR_INVALID, "fa_sdpa: device ordinal out of range");
  const size_t part_floats = sdpa_part_floats(q_len, H, hd);
  const size_t need = part_floats * 4 + sdpa_counters(q_len, KVH) * 4;
  std::lock_guard<std::mutex> lock(g_sdpa_mu);
  SdpaScratch &s = g_sdpa[dev];
  if (s.bytes < need) {
    if (s.buf) cudaFree(s.buf);
    s.buf = nullptr;
    s.bytes = 0;
    if (cudaMalloc(&s.buf, need) != cudaSuccess) return fail(FA_ERR_OOM, "fa_sdpa: scratch allocation failed");
    s.bytes = need;
  }
  float *part = (float *)s.buf;
  uint32_t *counters = (uint32_t *)(part + part_floats);
  API_CUDA(cudaMemsetAsync(counters, 0, sdpa_counters(q_len, KVH) * 4, (cudaStream_t)stream));
  AttnParams ap = sdpa_params(q, k, v, q_len, kv_len, H, KVH, hd, out, part, counters);
  if (launch_attention(ap, false, (cudaStream_t)stream)) return fail(FA_ERR_CUDA, "fa_sdpa: launch failed");
  return FA_OK;
}

int fa_sdpa_host(const float *q, const float *k, const float *v, uint32_t q_len, uint32_t kv_len, uint32_t H,
                 uint32_t KVH, uint32_t hd, float *out) {
  int rc = sdpa_check("fa_sdpa_host", q, k, v, q_len, kv_len, H, KVH, hd, out);
  if (rc) return rc;
  const size_t nq = (size_t)q_len * H * hd, nkv = (size_t)kv_len * KVH * hd;
  float *buf = nullptr;
  if (cudaMalloc(&buf, (2 * nq + 2 * nkv) * 4) != cudaSuccess) {
    cudaGetLastError();
    return fail(FA_ERR_OOM, "fa_sdpa_host: device buffers");
  }
  struct F {
    void *p;
    ~F() { cudaFree(p); }
  } free_buf{buf};
  float *dq = buf, *dk = dq + nq, *dv = dk + nkv, *dout = dv + nkv;
  API_CUDA(cudaMemcpy(dq, q, nq * 4, cudaMemcpyHostToDevice));
  API_CUDA(cudaMemcpy(dk, k, nkv * 4, cudaMemcpyHostToDevice));
  API_CUDA(cudaMemcpy(dv, v, nkv * 4, cudaMemcpyHostToDevice));
  if ((rc = fa_sdpa(dq, dk, dv, q_len, kv_len, H, KVH, hd, dout, nullptr))) return rc;
  API_CUDA(cudaMemcpy(out, dout, nq * 4, cudaMemcpyDeviceToHost));
  return FA_OK;
}

// ------------------------------------------------------------ profiling
int fa_profile_gemv(fa_model *fm, int32_t kind, uint32_t reps, float *avg_ms, uint64_t *bytes_per_launch) {
  API_NULL(fm);
  API_NULL(avg_ms);
  Model &m = fm->m;
  if (kind < 0 || kind > 4 || !reps) return fail(FA_ERR_INVALID, "fa_profile_gemv: bad kind or reps");
  if (kind == 4 && m.tied) return fail(FA_ERR_INVALID, "fa_profile_gemv: tied head has no GEMV");
  API_CUDA(cudaSetDevice(m.device));
  fa_kv kvh;
  int rc;
  if ((rc = create_kv(m, 1, 16, FA_KV_F32, &kvh.kv))) return rc;
  if ((rc = set_state(m, m.ws.state, 0, 0, 0, 0))) return rc;
  const uint32_t L = m.cfg.n_layers;
  auto launch = [&](uint32_t i) -> int {
    const uint32_t l = i % L;
    switch (kind) {
      case 0: return m.enqueue_qkv(l, m.ws, kvh.kv, 0, m.ws.state, m.raw_qkv_ok());
      case 4: return m.enqueue_head(m.ws, m.ws.state);
      default: {
        const LayerW &lw = m.layers[l];
        const GemvPlan &P = kind == 1 ? lw.o : kind == 2 ? lw.gateup : lw.down;
        GemvParams p = m.gemv_base(P);
        p.pro = kind == 2 ? kProRmsNorm : kProPlain;
        p.in = kind == 1 ? m.ws.attn_out : kind == 2 ? m.ws.x : m.ws.h;
        p.norm_w = lw.ffn_norm;
        p.ssq = m.ws.ssq_o;
        p.n_ssq = lw.o.parts();
        p.eps = m.cfg.norm_eps;
        p.epi = kind == 2 ? kEpiSwiglu : kEpiStore;
        p.out = kind == 2 ? m.ws.h : m.ws.logits;  // scratch destination
        p.state = m.ws.state;
        if (m.use_red()) {  // the launches of the decode step (o and down add into x, gate/up into gu)
          p.epi = kEpiRed;
          p.out = kind == 2 ? m.ws.gu : m.ws.x;
          if (kind == 2) {
            p.ssq = nullptr;
            p.n_ssq = 0;
            p.red_half = m.cfg.n_ff_used;
          } else if (kind == 3) {
            p.pro = kProSwiglu;
            p.in = m.ws.gu;
            p.in2 = m.ws.gu + m.cfg.n_ff_used;
          }
        }
        return launch_gemv(p, m.pdl, m.stream) ? fail(FA_ERR_CUDA, "gemv launch failed") : FA_OK;
      }
    }
  };
  for (uint32_t i = 0; i < std::min<uint32_t>(reps, 8); ++i)
    if ((rc = launch(i))) return rc;  // warm-up
  cudaEvent_t e0, e1;
  API_CUDA(cudaEventCreate(&e0));
  API_CUDA(cudaEventCreate(&e1));
  API_CUDA(cudaEventRecord(e0, m.stream));
  for (uint32_t i = 0; i < reps; ++i)
    if ((rc = launch(i))) return rc;
  API_CUDA(cudaEventRecord(e1, m.stream));
  API_CUDA(cudaEventSynchronize(e1));
  float ms = 0.0f;
  API_CUDA(cudaEventElapsedTime(&ms, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  *avg_ms = ms / reps;
  if (bytes_per_launch) {
    const LayerW &lw = m.layers[0];
    const GemvPlan &P = kind == 0 ? lw.qkv : kind == 1 ? lw.o : kind == 2 ? lw.gateup : kind == 3 ? lw.down : m.head;
    *bytes_per_launch = P.native_bytes;
  }
  return check_err_flags(m, m.ws.state);
}

// ------------------------------------------------------------ synth
int fa_synth_write(const char *path, const fa_synth_spec *spec, uint64_t seed) { return synth_write(path, spec, seed); }

}  // extern "C"

// ------------------------------------------------------------ token-parallel GEMM
namespace {

const GemvPlan *plan_of(Model &m, int32_t proj, uint32_t layer) {
  if (proj == 4) return &m.head;
  if (layer >= m.layers.size()) return nullptr;
  const LayerW &lw = m.layers[layer];
  switch (proj) {
    case 0: return &lw.qkv;
    case 1: return &lw.o;
    case 2: return &lw.gateup;
    case 3: return &lw.down;
    default: return nullptr;
  }
}
struct DevBuf {
  void *p = nullptr;
  ~DevBuf() { if (p) cudaFree(p); }
};
}  // namespace

extern "C" int fa_gemm_tokens(fa_model *fm, int32_t proj, uint32_t layer, const float *x_host, uint32_t T,
                              float *y_host, uint32_t *n_out) {
  API_NULL(fm);
  API_NULL(x_host);
  API_NULL(n_out);
  Model &m = fm->m;
  const GemvPlan *P = plan_of(m, proj, layer);
  if (!P) return fail(FA_ERR_INVALID, "fa_gemm_tokens: projection or layer out of range");
  if (!P->mma || P->qg_tiles.empty()) return fail(FA_ERR_UNSUPPORTED, "fa_gemm_tokens: projection not in the MMA layout");
  if (!T) return fail(FA_ERR_INVALID, "fa_gemm_tokens: zero tokens");
  *n_out = P->n_out;
  if (!y_host) return FA_OK;
  API_CUDA(cudaSetDevice(m.device));
  const uint32_t K = P->K, N = P->n_out;
  std::vector<uint16_t> xb((size_t)T * K);
  for (size_t i = 0; i < xb.size(); ++i) xb[i] = f32_to_f16(x_host[i]);
  DevBuf x, y, err, part;
  const uint64_t part_floats = qgemm_part_floats(512, (uint32_t)m.n_sm);  // stream-K partial tiles
  API_CUDA(cudaMalloc(&part.p, part_floats * 4));
  API_CUDA(cudaMalloc(&x.p, xb.size() * 2));
  API_CUDA(cudaMalloc(&y.p, (size_t)T * N * 4));
  API_CUDA(cudaMalloc(&err.p, 4));
  API_CUDA(cudaMemcpyAsync(x.p, xb.data(), xb.size() * 2, cudaMemcpyHostToDevice, m.stream));
  API_CUDA(cudaMemsetAsync(y.p, 0, (size_t)T * N * 4, m.stream));
  API_CUDA(cudaMemsetAsync(err.p, 0, 4, m.stream));
  QgXMap map;
  const uint32_t bn = T <= 64 ? 64 : T <= 128 ? 128 : 256;
  if (qgemm_make_xmap(&map, x.p, K, T, bn)) return fail(FA_ERR_CUDA, "tensor map encoding failed");
  QgParams p{};
  p.w = P->w;
  p.chunks = P->d_chunks;
  p.tiles = P->d_qg_tiles;
  p.n_tiles = (uint32_t)P->qg_tiles.size();
  p.K = K;
  p.T = T;
  p.out = (float *)y.p;
  p.ldo = N;
  p.epi = kQgStore;
  p.err = (uint32_t *)err.p;
  p.part = (float *)part.p;
  p.part_floats = part_floats;
  p.prefetch = P->qg_prefetch;
  if (launch_qgemm(p, map, (uint32_t)m.n_sm, m.stream)) return fail(FA_ERR_CUDA, "token GEMM launch failed");
  uint32_t e = 0;
  API_CUDA(cudaMemcpyAsync(y_host, y.p, (size_t)T * N * 4, cudaMemcpyDeviceToHost, m.stream));
  API_CUDA(cudaMemcpyAsync(&e, err.p, 4, cudaMemcpyDeviceToHost, m.stream));
  { const int sync_rc = m.sync(); if (sync_rc) return sync_rc; }
  if (e) return fail(FA_ERR_TIMEOUT, "token GEMM: a bounded device wait gave up");
  return FA_OK;
}

// Device time of the token GEMM on device-resident operands (X: T x K bf16
// of a fixed pattern, Y f32): average over `reps` launches after one warm-up.
extern "C" int fa_profile_gemm(fa_model *fm, int32_t proj, uint32_t layer, uint32_t T, uint32_t reps, float *avg_ms,
                               double *flop) {
  API_NULL(fm);
  API_NULL(avg_ms);
  Model &m = fm->m;
  const GemvPlan *P = plan_of(m, proj, layer);
  if (!P || !P->mma || P->qg_tiles.empty() || !T || !reps) return fail(FA_ERR_INVALID, "fa_profile_gemm: bad arguments");
  API_CUDA(cudaSetDevice(m.device));
  const uint32_t K = P->K, N = P->n_out;
  DevBuf x, y, part;
  const uint64_t part_floats = qgemm_part_floats(512, (uint32_t)m.n_sm);  // stream-K partial tiles
  API_CUDA(cudaMalloc(&part.p, part_floats * 4));
  API_CUDA(cudaMalloc(&x.p, (size_t)T * K * 2));
  API_CUDA(cudaMalloc(&y.p, (size_t)T * N * 4));
  API_CUDA(cudaMemsetAsync(x.p, 0x1C, (size_t)T * K * 2, m.stream));  // f16 0x1C1C ~ 0.0041
  QgXMap map;
  if (qgemm_make_xmap(&map, x.p, K, T, T <= 64 ? 64 : T <= 128 ? 128 : 256)) return fail(FA_ERR_CUDA, "tensor map encoding failed");
  QgParams p{};
  p.w = P->w;
  p.chunks = P->d_chunks;
  p.tiles = P->d_qg_tiles;
  p.n_tiles = (uint32_t)P->qg_tiles.size();
  p.K = K;
  p.T = T;
  p.out = (float *)y.p;
  p.ldo = N;
  p.epi = kQgStore;
  p.part = (float *)part.p;
  p.part_floats = part_floats;
  p.prefetch = P->qg_prefetch;
  cudaEvent_t e0, e1;
  API_CUDA(cudaEventCreate(&e0));
  API_CUDA(cudaEventCreate(&e1));
  int rc = FA_OK;
  if (launch_qgemm(p, map, (uint32_t)m.n_sm, m.stream)) rc = fail(FA_ERR_CUDA, "token GEMM launch failed");
  cudaEventRecord(e0, m.stream);
  for (uint32_t r = 0; r < reps && rc == FA_OK; ++r)
    if (launch_qgemm(p, map, (uint32_t)m.n_sm, m.stream)) rc = fail(FA_ERR_CUDA, "token GEMM launch failed");
  cudaEventRecord(e1, m.stream);
  cudaError_t ce = cudaEventSynchronize(e1);
  float ms = 0.0f;
  cudaEventElapsedTime(&ms, e0, e1);
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  if (rc) return rc;
  if (ce != cudaSuccess) return fail(FA_ERR_CUDA, std::string("token GEMM: ") + cudaGetErrorString(ce));
  *avg_ms = ms / (float)reps;
  if (flop) *flop = 2.0 * T * (double)K * N;
  return FA_OK;
}

extern "C" int fa_decode_batch(fa_model *fm, fa_kv *kv, uint32_t b, const uint32_t *tokens, const uint32_t *pos,
                               fa_sampler *s, uint32_t steps, uint32_t *ids_out, float *logits_out) {
  API_NULL(fm);
  API_NULL(kv);
  API_NULL(tokens);
  API_NULL(pos);
  API_NULL(s);
  API_NULL(ids_out);
  if (!steps) return FA_OK;
  Model &m = fm->m;
  if (b > s->n_seq) return fail(FA_ERR_INVALID, "fa_decode_batch: more sequences than sampler rows");
  if (m.cfg.vocab_size > s->vocab) return fail(FA_ERR_INVALID, "fa_decode_batch: sampler vocabulary too small");
  API_CUDA(cudaSetDevice(m.device));
  SamplerParams sp = s->params(m.cfg.vocab_size);
  int rc;
  if ((rc = sampler_keys(s, sp))) return rc;
  API_CUDA(cudaStreamSynchronize(s->stream));  // observes / resets queued on the sampler's stream
  return m.decode_batch(kv->kv, b, tokens, pos, sp, steps, ids_out, logits_out);
}

