// Host runtime: GGUF -> device weights (native blocks re-laid into column
// chunks), workspaces, KV cache, and the per-token kernel sequence of
// ModelWeights::forward (src/model.rs:316-455).
#include "model.hpp"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstring>
#include <thread>

namespace fa {

#define CUDA_TRY(expr)                                                                    \
  do {                                                                                    \
    cudaError_t e_ = (expr);                                                              \
    if (e_ != cudaSuccess) return fail(FA_ERR_CUDA, std::string(#expr) + ": " + cudaGetErrorString(e_)); \
  } while (0)

static const char *kLayerNames[9] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                     "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};

uint32_t n_ff_of(uint32_t n_embd, float mult) {  // src/model.rs:66-70
  float raw = (float)n_embd * mult;
  uint64_t r = (raw != raw || raw <= 0.0f) ? 0 : (uint64_t)raw;
  return (uint32_t)((r + 255) / 256 * 256);
}

// ModelConfig::from_gguf, src/model.rs:92-180
int config_from_gguf(const Gguf &g, fa_config *c) {
  std::memset(c, 0, sizeof *c);
  std::string arch;
  if (!g.meta_string("general.architecture", &arch)) return fail(FA_ERR_GGUF, "missing general.architecture");
  if (arch != "llama" && arch != "qwen2" && arch != "mistral" && arch != "phi")
    return fail(FA_ERR_UNSUPPORTED, "unsupported model architecture: " + arch);
  uint64_t v;
  auto req = [&](const char *suffix, uint32_t *dst) {
    std::string k = arch + "." + suffix;
    if (!g.meta_u64(k, &v)) return fail(FA_ERR_GGUF, "missing " + k);
    *dst = (uint32_t)v;
    return FA_OK;
  };
  int rc;
  if ((rc = req("block_count", &c->n_layers))) return rc;
  if ((rc = req("attention.head_count", &c->n_heads))) return rc;
  c->n_kv_heads = g.meta_u64(arch + ".attention.head_count_kv", &v) ? (uint32_t)v : c->n_heads;
  if ((rc = req("embedding_length", &c->n_embd))) return rc;
  if ((rc = req("context_length", &c->context_len))) return rc;
  if (g.vocab_size(&v)) {
    c->vocab_size = (uint32_t)v;
  } else if (const GgufTensor *t = g.tensor("token_embd.weight")) {
    c->vocab_size = c->n_embd ? (uint32_t)(t->nelement() / c->n_embd) : 0;
  } else {
    return fail(FA_ERR_GGUF, "cannot determine vocab size");
  }
  if (c->n_heads == 0) return fail(FA_ERR_GGUF, "attention.head_count is 0");
  c->head_dim = c->n_embd / c->n_heads;
  if (c->head_dim == 0) return fail(FA_ERR_GGUF, "n_embd not divisible by head count");
  float f;
  c->ffn_dim_multiplier = g.meta_f32(arch + ".feed_forward_length", &f) ? f / (float)c->n_embd : 2.667f;
  c->norm_eps = g.meta_f32(arch + ".attention.layer_norm_rms_epsilon", &f) ? f : 1e-5f;
  c->rope_base = g.meta_f32(arch + ".rope.freq_base", &f) ? f : 10000.0f;
  c->rope_freq_dim = c->head_dim / 2;
  c->n_ff = n_ff_of(c->n_embd, c->ffn_dim_multiplier);
  c->n_ff_used = c->n_ff;
  c->tied_output = g.tensor("output.weight") == nullptr;
  return FA_OK;
}

void *Model::dmalloc(size_t bytes) {
  void *p = nullptr;
  if (cudaMalloc(&p, bytes ? bytes : 16) != cudaSuccess) {
    cudaGetLastError();  // an allocation failure is not sticky: keep it out of later launch checks
    return nullptr;
  }
  allocs.push_back(p);
  device_bytes += bytes;
  return p;
}

Model::~Model() {
  for (KvCache *kv : live_kv) kv->m = nullptr;  // caches may outlive the model
  if (graph) cudaGraphExecDestroy(graph);
  if (device >= 0) cudaSetDevice(device);
  if (h_state) cudaFreeHost(h_state);
  for (void *p : allocs) cudaFree(p);
  if (stream) cudaStreamDestroy(stream);
}

namespace {

struct TensorRef {
  const GgufTensor *t = nullptr;
  const uint8_t *data = nullptr;
  size_t nbytes = 0;
  int type = 0;
  uint64_t nelem = 0;
  uint32_t row_bytes = 0;   // stride of the rows at `data` (0: native_row_bytes of the width)
  uint32_t algo_bytes = 0;  // bytes a row contributes to the algorithmic count (0: row_bytes)
  std::vector<uint8_t> own; // storage of a tensor-parallel column shard
};

int get_tensor(const Gguf &g, const std::string &name, TensorRef *r) {
  r->t = g.tensor(name);
  if (!r->t) return fail(FA_ERR_GGUF, "tensor not found: " + name);
  r->type = (int)r->t->ggml_type;
  r->nelem = r->t->nelement();
  if (!type_known(r->type)) return fail(FA_ERR_UNSUPPORTED, "unsupported ggml type " + std::to_string(r->type) + " for " + name);
  r->data = g.tensor_data(*r->t, &r->nbytes);
  if (!r->data) return fail(FA_ERR_GGUF, "tensor '" + name + "' has no data");
  if (r->nbytes < type_nbytes(r->type, r->nelem / block_elems(r->type) * block_elems(r->type)))
    return fail(FA_ERR_GGUF, "tensor '" + name + "' is truncated");
  return FA_OK;
}

uint32_t pick_cw(int type, uint32_t N, bool paired) {
  uint32_t cw = 256;
  if (N >= 1024 * 37) cw = 1024;
  else if (N >= 512 * 37) cw = 512;
  if (paired && (type == kQ4_K || type == kQ6_K)) cw = std::max(cw, 512u);
  return cw;
}

// columns [c0, c1) of every row of `src` ([K][N]) as a tensor of its own
int shard_cols(const TensorRef &src, const char *what, uint32_t K, uint32_t N, uint32_t c0, uint32_t c1,
               TensorRef *dst) {
  dst->t = src.t;
  dst->type = src.type;
  uint32_t rb = 0;
  if (tp_shard_columns(src.type, src.data, K, N, c0, c1, dst->own, &rb))
    return fail(FA_ERR_UNSUPPORTED, std::string("tensor-parallel shard of ") + what + ": columns [" +
                                        std::to_string(c0) + ", " + std::to_string(c1) +
                                        ") do not fall on the type's block boundaries");
  dst->data = dst->own.data();
  dst->nbytes = dst->own.size();
  dst->nelem = (uint64_t)K * (c1 - c0);
  dst->row_bytes = rb;
  // a half super-block streams its 64 code bytes and the shared 16-byte header
  dst->algo_bytes = (src.type == kQ4_K && c1 - c0 == 128) ? 80 : rb;
  return FA_OK;
}

// rows [r0, r0 + nr) of `src` ([K][N]): a contiguous range of the mapping
void shard_rows(const TensorRef &src, uint32_t N, uint32_t r0, uint32_t nr, TensorRef *dst) {
  const uint32_t rb = native_row_bytes(src.type, N);
  dst->t = src.t;
  dst->type = src.type;
  dst->data = tp_rows(src.data, rb, r0);
  dst->nbytes = (size_t)nr * rb;
  dst->nelem = (uint64_t)nr * N;
}

}  // namespace

// One GEMV launch covering `parts` (tensors sharing K).  paired: parts[0]
// and parts[1] are gate/up interleaved per chunk.  Launches whose tensors are
// all Q4_K / Q6_K / Q8_0 / Q4_0 (K a multiple of 16) use the tensor-core
// kernel and its MMA tile layout with 1024-column chunks; others use the
// 8-row-group layout.  cw_div: chunk width must be a multiple of it
// (RoPE pairs of a head stay in one chunk).
static int build_plan(Model &m, GemvPlan &P, const std::vector<TensorRef> &parts, const std::vector<uint32_t> &out_base,
                      bool paired, uint32_t K, const std::vector<uint32_t> &widths, uint32_t CW, void *staging,
                      void *staging2, uint32_t cw_div = 1) {
  bool mma = K % 16 == 0 && 1024 % cw_div == 0;
  for (size_t i = 0; i < parts.size(); ++i) mma = mma && mma_type(parts[i].type) && widths[paired ? 0 : i] % 32 == 0;
  if (mma) CW = 1024;
  P.mma = mma;
  P.K = K;
  P.K8 = (K + 7) / 8 * 8;
  P.CW = CW;
  P.native_bytes = 0;
  const uint32_t rows = mma ? K / 16 : P.K8 / 8;  // row groups per chunk
  auto gbytes = [&](int type, uint32_t w) { return mma ? mma_group_bytes(type, w) : group_bytes(type, w); };
  // sizes
  std::vector<uint64_t> region;
  uint64_t total = 0;
  const size_t nparts = paired ? 1 : parts.size();
  for (size_t i = 0; i < nparts; ++i) {
    const uint32_t N = paired ? 2 * widths[0] : widths[i];
    region.push_back(total);
    uint64_t b = 0;
    for (uint32_t c0 = 0; c0 < N; c0 += CW) b += (uint64_t)rows * gbytes(parts[i].type, std::min(CW, N - c0));
    total += (b + 255) / 256 * 256;
  }
  uint8_t *buf = (uint8_t *)m.dmalloc(total);
  if (!buf) return fail(FA_ERR_OOM, "device allocation of " + std::to_string(total) + " weight bytes failed");
  P.w = buf;
  uint32_t max_gb = 0;
  for (size_t i = 0; i < nparts; ++i) {
    const TensorRef &a = parts[i];
    const uint32_t N = widths[i];
    const uint32_t rb = a.row_bytes ? a.row_bytes : native_row_bytes(a.type, N);
    const uint64_t nb = (uint64_t)K * rb, ab = (uint64_t)K * (a.algo_bytes ? a.algo_bytes : rb);
    if (!mma && rb != native_row_bytes(a.type, N))
      return fail(FA_ERR_UNSUPPORTED, "a half super-block shard needs the tensor-core layout");
    CUDA_TRY(cudaMemcpyAsync(staging, a.data, nb, cudaMemcpyHostToDevice, m.stream));
    P.native_bytes += ab;
    const void *src_b = nullptr;
    if (paired) {
      const TensorRef &b = parts[1];
      if (b.type != a.type) return fail(FA_ERR_UNSUPPORTED, "ffn_gate and ffn_up must share a ggml type");
      CUDA_TRY(cudaMemcpyAsync(staging2, b.data, nb, cudaMemcpyHostToDevice, m.stream));
      P.native_bytes += ab;
      src_b = staging2;
    }
    const int rc = mma ? launch_repack_mma(a.type, staging, src_b, K, N, CW, buf, region[i], m.stream)
                       : launch_repack(a.type, staging, src_b, K, N, CW, buf, region[i], m.stream);
    if (rc) return fail(FA_ERR_CUDA, "repack launch failed");
    CUDA_TRY(cudaStreamSynchronize(m.stream));
    const uint32_t Nv = paired ? 2 * N : N;
    for (uint32_t c = 0, c0 = 0; c0 < Nv; c0 += CW, ++c) {
      ChunkDesc d{};
      const uint32_t w = std::min(CW, Nv - c0);
      d.offset = region[i] + (uint64_t)c * rows * gbytes(a.type, CW);
      d.gbytes = gbytes(a.type, w);
      d.type = (uint16_t)a.type;
      d.width = (uint16_t)w;
      d.out_col = out_base[i] + c0;
      d.sgroups = mma ? gemv_mma_stage_groups(d.gbytes, a.type) : 0;
      P.chunks.push_back(d);
      max_gb = std::max(max_gb, d.gbytes);
    }
  }
  P.n_out = 0;
  for (const ChunkDesc &d : P.chunks) P.n_out = std::max<uint32_t>(P.n_out, d.out_col + d.width);
  if (mma) {
    P.stage_bytes = 0;  // the largest stage (sgroups whole groups) of any chunk
    for (const ChunkDesc &d : P.chunks) P.stage_bytes = std::max(P.stage_bytes, d.sgroups * d.gbytes);
    P.x_slot = 0;
  } else {
    P.stage_bytes = std::max<uint32_t>(16384, (max_gb + 15) / 16 * 16);
    uint32_t max_ng = 1;
    for (const ChunkDesc &d : P.chunks) max_ng = std::max(max_ng, P.stage_bytes / d.gbytes);
    P.x_slot = 8 * max_ng;
  }
  // stream-K split: CTA i streams bytes [i*B/P, (i+1)*B/P) of the chunk-major
  // (chunk, row group) sequence, rounded to whole groups
  const uint32_t G = rows, nc = (uint32_t)P.chunks.size();
  std::vector<uint64_t> start(nc + 1, 0);
  for (uint32_t c = 0; c < nc; ++c) start[c + 1] = start[c] + (uint64_t)G * P.chunks[c].gbytes;
  const uint64_t B = start[nc];
  uint64_t units = (uint64_t)G * nc;
  P.n_ctas = (uint32_t)std::min<uint64_t>(m.n_sm, units);
  auto unit_at = [&](uint64_t b, uint32_t *c, uint32_t *g) {
    uint32_t k = 0;
    while (k + 1 < nc && start[k + 1] <= b) ++k;
    uint64_t gg = (b - start[k] + P.chunks[k].gbytes / 2) / P.chunks[k].gbytes;
    if (gg >= G) {
      *c = k + 1;
      *g = 0;
    } else {
      *c = k;
      *g = (uint32_t)gg;
    }
  };
  P.ranges.resize(P.n_ctas);
  for (uint32_t i = 0; i < P.n_ctas; ++i) {
    CtaRange &r = P.ranges[i];
    unit_at(B * i / P.n_ctas, &r.c0, &r.g0);
    unit_at(B * (i + 1) / P.n_ctas, &r.c1, &r.g1);
  }
  // contributors of each chunk (CTAs with a non-empty range touching it);
  // rounding can leave some CTAs empty, so the list is explicit
  std::vector<std::vector<uint16_t>> who(nc);
  P.max_chunks_per_cta = 1;
  for (uint32_t i = 0; i < P.n_ctas; ++i) {
    const CtaRange &r = P.ranges[i];
    if (r.c0 > r.c1 || (r.c0 == r.c1 && r.g0 >= r.g1)) continue;  // empty range
    const uint32_t last = r.g1 > 0 ? r.c1 : r.c1 - 1;
    P.max_chunks_per_cta = std::max(P.max_chunks_per_cta, last - r.c0 + 1);
    for (uint32_t c = r.c0; c <= last; ++c) who[c].push_back((uint16_t)i);
  }
  if (mma) {
    P.max_units = 1;
    for (const CtaRange &r : P.ranges) {
      const uint64_t a = (uint64_t)r.c0 * G + r.g0, b = (uint64_t)r.c1 * G + r.g1;
      if (b > a) P.max_units = std::max<uint32_t>(P.max_units, (uint32_t)(b - a));
    }
    P.n_stages = gemv_mma_stages(P.stage_bytes, P.max_units, 227 * 1024);
    if (P.n_stages < 2)
      return fail(FA_ERR_UNSUPPORTED, "GEMV pipeline does not fit in shared memory (" +
                                          std::to_string(P.max_units) + " row groups per CTA)");
  }
  P.contrib.clear();
  for (uint32_t c = 0; c < nc; ++c) {
    if (who[c].empty() || P.n_ctas > 65535) return fail(FA_ERR_INVALID, "GEMV split failed");
    P.chunks[c].contrib_off = (uint32_t)P.contrib.size();
    P.chunks[c].n_contrib = (uint32_t)who[c].size();
    if (mma && who[c].size() > kGemvMaxContrib) return fail(FA_ERR_UNSUPPORTED, "GEMV chunk has too many contributors");
    for (uint16_t i : who[c]) P.contrib.push_back(i * P.max_chunks_per_cta + (c - P.ranges[i].c0));
  }
  P.d_chunks = (ChunkDesc *)m.dmalloc(P.chunks.size() * sizeof(ChunkDesc));
  P.d_ranges = (CtaRange *)m.dmalloc(P.ranges.size() * sizeof(CtaRange));
  P.d_contrib = (uint32_t *)m.dmalloc(P.contrib.size() * sizeof(uint32_t));
  if (!P.d_chunks || !P.d_ranges || !P.d_contrib) return fail(FA_ERR_OOM, "GEMV table allocation failed");
  CUDA_TRY(cudaMemcpy(P.d_contrib, P.contrib.data(), P.contrib.size() * sizeof(uint32_t), cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(P.d_chunks, P.chunks.data(), P.chunks.size() * sizeof(ChunkDesc), cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(P.d_ranges, P.ranges.data(), P.ranges.size() * sizeof(CtaRange), cudaMemcpyHostToDevice));
  if (mma) {  // 128-column output tiles of the token-parallel GEMM
    P.qg_tiles.clear();
    for (uint32_t c = 0; c < nc; ++c)
      for (uint32_t c0 = 0; c0 < P.chunks[c].width; c0 += 128)
        P.qg_tiles.push_back({c, c0, std::min<uint32_t>(128, P.chunks[c].width - c0), 0});
    P.qg_prefetch = nc && (P.chunks[0].type == kQ8_0 || P.chunks[0].type == kQ4_0) ? P.chunks[0].type : 0u;
    for (uint32_t c = 0; c < nc; ++c)
      if (P.chunks[c].type != P.qg_prefetch) P.qg_prefetch = 0;
    if (!P.qg_prefetch) {
      // the mixed-type ring copies whole super-block headers, d and scale
      // vectors with 16-byte cp.async: K-quant chunks of whole super-blocks
      bool any = nc > 0;
      for (const ChunkDesc &d : P.chunks)
        any = any && d.offset % 16 == 0 && d.gbytes % 16 == 0 &&
              ((d.type != kQ4_K && d.type != kQ6_K) || d.width % 256 == 0);
      P.qg_prefetch = any ? kPfAny : 0u;
    }
    P.d_qg_tiles = (QgTile *)m.dmalloc(P.qg_tiles.size() * sizeof(QgTile));
    if (!P.d_qg_tiles) return fail(FA_ERR_OOM, "GEMM tile table allocation failed");
    CUDA_TRY(cudaMemcpy(P.d_qg_tiles, P.qg_tiles.data(), P.qg_tiles.size() * sizeof(QgTile), cudaMemcpyHostToDevice));
  }
  m.part_floats = std::max<size_t>(m.part_floats, (size_t)P.n_ctas * P.max_chunks_per_cta * P.CW);
  m.max_chunks = std::max<uint32_t>(m.max_chunks, nc);
  return FA_OK;
}

int Model::ensure_rope(uint32_t max_pos) {
  if (max_pos <= rope_max) return FA_OK;
  const uint32_t hd = cfg.head_dim, half = hd / 2;
  std::vector<float> tab((size_t)max_pos * hd);
  std::vector<float> freq(half);
  for (uint32_t i = 0; i < half; ++i)  // rope_emb, src/tensor.rs:386-397
    freq[i] = 1.0f / std::pow(cfg.rope_base, (2.0f * (float)i) / (float)hd);
  for (uint32_t p = 0; p < max_pos; ++p)
    for (uint32_t i = 0; i < half; ++i) {
      const float ang = (float)p * freq[i];
      tab[(size_t)p * hd + 2 * i] = std::cos(ang);
      tab[(size_t)p * hd + 2 * i + 1] = std::sin(ang);
    }
  float *d = (float *)dmalloc(tab.size() * sizeof(float));
  if (!d) return fail(FA_ERR_OOM, "rope table allocation failed");
  CUDA_TRY(cudaMemcpy(d, tab.data(), tab.size() * sizeof(float), cudaMemcpyHostToDevice));
  rope_tab = d;
  rope_max = max_pos;
  if (graph) {  // captured graphs hold the old table pointer
    cudaGraphExecDestroy(graph);
    graph = nullptr;
  }
  return FA_OK;
}

int Model::load(const std::string &path, const fa_model_opts &o) {
  device = o.device;
  pdl = o.use_pdl != 0;
  graphs = o.use_graphs != 0;
  want_step = o.use_step_kernel != 0;
  want_tc_prefill = o.use_tc_prefill != 0;
  CUDA_TRY(cudaSetDevice(device));
  CUDA_TRY(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  CUDA_TRY(cudaMallocHost(&h_state, sizeof(SeqState)));
  if (gemv_init() || gemv_mma_init() || attention_init() || step_init() || sampler_init() || qgemm_init() ||
      attn_rows_init())
    return fail(FA_ERR_CUDA, "kernel attribute setup failed");
  CUDA_TRY(cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, device));
  int code = FA_OK;
  gguf.reset(Gguf::open(path, &code));
  if (!gguf) return code;
  const Gguf &g = *gguf;
  int rc = config_from_gguf(g, &cfg);
  if (rc) return rc;
  const uint32_t d = cfg.n_embd, H = cfg.n_heads, KVH = cfg.n_kv_heads, hd = cfg.head_dim;
  if (KVH == 0 || H % KVH) return fail(FA_ERR_UNSUPPORTED, "head_count must be a multiple of head_count_kv");
  if (H * hd != d || hd % 2 || hd > 128 || (H / KVH != 1 && H / KVH != 2 && H / KVH != 4 && H / KVH != 8)) return fail(FA_ERR_UNSUPPORTED, "unsupported head geometry");
  const uint32_t qd = H * hd, kvd = KVH * hd;
  TensorRef gate0;
  if ((rc = get_tensor(g, "blk.0.ffn_gate.weight", &gate0))) return rc;
  cfg.n_ff_used = (uint32_t)(gate0.nelem / d);
  const uint32_t F = cfg.n_ff_used, V = cfg.vocab_size, L = cfg.n_layers;
  // validate every tensor first
  std::vector<std::vector<TensorRef>> lt(L, std::vector<TensorRef>(9));
  size_t max_native = 0;
  for (uint32_t l = 0; l < L; ++l)
    for (int j = 0; j < 9; ++j) {
      if ((rc = get_tensor(g, "blk." + std::to_string(l) + "." + kLayerNames[j] + ".weight", &lt[l][j]))) return rc;
      max_native = std::max(max_native, lt[l][j].nbytes);
    }
  const uint64_t expect[9] = {d, (uint64_t)d * qd, (uint64_t)d * kvd, (uint64_t)d * kvd, (uint64_t)qd * d,
                              d, (uint64_t)d * F, (uint64_t)d * F, (uint64_t)F * d};
  const uint32_t widths[9] = {d, qd, kvd, kvd, d, d, F, F, d};
  for (uint32_t l = 0; l < L; ++l)
    for (int j = 0; j < 9; ++j) {
      const TensorRef &t = lt[l][j];
      if (t.nelem != expect[j])
        return fail(FA_ERR_GGUF, "tensor blk." + std::to_string(l) + "." + kLayerNames[j] + " has " +
                                     std::to_string(t.nelem) + " elements, expected " + std::to_string(expect[j]));
      if (j != 0 && j != 5) {
        if (!gemv_type_supported(t.type))
          return fail(FA_ERR_UNSUPPORTED, std::string("ggml type not supported for projections: ") + std::to_string(t.type));
        if (widths[j] % type_block(t.type)) return fail(FA_ERR_UNSUPPORTED, "projection width not block aligned");
      }
    }
  // tensor parallelism: this rank keeps query heads [R*H/W, (R+1)*H/W), the
  // KV heads they read, FFN columns [R*F/W, (R+1)*F/W) of gate and up, and
  // the matching rows of attn_output and ffn_down (whose partial sums the
  // ranks add up with an all-reduce); embedding, norms and the output head
  // are replicated
  gcfg = cfg;
  const uint32_t W = o.tp_world > 1 ? (uint32_t)o.tp_world : 1u;
  const uint32_t R = W > 1 ? (uint32_t)o.tp_rank : 0u;
  if (W > 1) {
    if (o.tp_rank < 0 || R >= W) return fail(FA_ERR_INVALID, "tp_rank out of range");
    if (H % W || KVH % W || F % W)
      return fail(FA_ERR_UNSUPPORTED, "heads, KV heads and FFN width must divide by the tensor-parallel world");
    if (cfg.tied_output) return fail(FA_ERR_UNSUPPORTED, "tensor parallelism needs an untied output head");
    if (!o.nccl_id) return fail(FA_ERR_INVALID, "tensor parallelism needs the rank-0 NCCL unique id");
    if ((rc = tp.init((int)R, (int)W, o.nccl_id, device))) return rc;
    want_step = false;  // the persistent step kernel is single-GPU
  }
  const uint32_t Hl = H / W, KVHl = KVH / W, Fl = F / W, qdl = Hl * hd, kvdl = KVHl * hd;
  cfg.n_heads = Hl;
  cfg.n_kv_heads = KVHl;
  cfg.n_ff_used = Fl;
  TensorRef temb, onorm, out;
  if ((rc = get_tensor(g, "token_embd.weight", &temb))) return rc;
  if ((rc = get_tensor(g, "output_norm.weight", &onorm))) return rc;
  if (temb.nelem != (uint64_t)V * d) return fail(FA_ERR_GGUF, "token_embd.weight size mismatch");
  if (d % block_elems(temb.type)) return fail(FA_ERR_UNSUPPORTED, "embedding rows not block aligned");
  tied = cfg.tied_output != 0;
  if (!tied) {
    if ((rc = get_tensor(g, "output.weight", &out))) return rc;
    if (out.nelem != (uint64_t)V * d) return fail(FA_ERR_GGUF, "output.weight size mismatch");
    if (!gemv_type_supported(out.type) || V % type_block(out.type))
      return fail(FA_ERR_UNSUPPORTED, "output.weight type/width not supported");
    max_native = std::max(max_native, out.nbytes);
  }
  void *staging = nullptr, *staging2 = nullptr;
  CUDA_TRY(cudaMalloc(&staging, max_native));
  CUDA_TRY(cudaMalloc(&staging2, max_native));
  struct Free {
    void *a, *b;
    ~Free() {
      cudaFree(a);
      cudaFree(b);
    }
  } free_staging{staging, staging2};

  auto upload_f32 = [&](const TensorRef &t, float **dst) -> int {
    *dst = (float *)dmalloc((t.nelem + 8) * sizeof(float));  // read in whole 8-row groups
    if (!*dst) return fail(FA_ERR_OOM, "norm allocation failed");
    CUDA_TRY(cudaMemset(*dst, 0, (t.nelem + 8) * sizeof(float)));
    CUDA_TRY(cudaMemcpyAsync(staging, t.data, type_nbytes(t.type, t.nelem), cudaMemcpyHostToDevice, stream));
    if (launch_dequant_native(t.type, staging, t.nelem, *dst, stream)) return fail(FA_ERR_CUDA, "dequant launch failed");
    CUDA_TRY(cudaStreamSynchronize(stream));
    return FA_OK;
  };

  layers.resize(L);
  step_bytes = 0;
  for (uint32_t l = 0; l < L; ++l) {
    LayerW &lw = layers[l];
    auto &T = lt[l];
    if ((rc = upload_f32(T[0], &lw.attn_norm))) return rc;
    if ((rc = upload_f32(T[5], &lw.ffn_norm))) return rc;
    TensorRef wq, wk, wv, wo, wg, wu, wd;
    if (W > 1) {
      if ((rc = shard_cols(T[1], "attn_q", d, qd, R * qdl, (R + 1) * qdl, &wq)) ||
          (rc = shard_cols(T[2], "attn_k", d, kvd, R * kvdl, (R + 1) * kvdl, &wk)) ||
          (rc = shard_cols(T[3], "attn_v", d, kvd, R * kvdl, (R + 1) * kvdl, &wv)) ||
          (rc = shard_cols(T[6], "ffn_gate", d, F, R * Fl, (R + 1) * Fl, &wg)) ||
          (rc = shard_cols(T[7], "ffn_up", d, F, R * Fl, (R + 1) * Fl, &wu)))
        return rc;
      shard_rows(T[4], d, R * qdl, qdl, &wo);
      shard_rows(T[8], d, R * Fl, Fl, &wd);
    } else {
      wq = T[1], wk = T[2], wv = T[3], wo = T[4], wg = T[6], wu = T[7], wd = T[8];
    }
    if ((rc = build_plan(*this, lw.qkv, {wq, wk, wv}, {0, qdl, qdl + kvdl}, false, d, {qdl, kvdl, kvdl}, 256, staging,
                         staging2, hd)))
      return rc;
    if ((rc = build_plan(*this, lw.o, {wo}, {0}, false, qdl, {d}, pick_cw(wo.type, d, false), staging, staging2)))
      return rc;
    if ((rc = build_plan(*this, lw.gateup, {wg, wu}, {0}, true, d, {Fl}, pick_cw(wg.type, 2 * Fl, true), staging,
                         staging2)))
      return rc;
    if ((rc = build_plan(*this, lw.down, {wd}, {0}, false, Fl, {d}, pick_cw(wd.type, d, false), staging, staging2)))
      return rc;
    step_bytes += lw.qkv.native_bytes + lw.o.native_bytes + lw.gateup.native_bytes + lw.down.native_bytes;
    step_bytes += type_nbytes(T[0].type, d) + type_nbytes(T[5].type, d);
  }
  if ((rc = upload_f32(onorm, &out_norm))) return rc;
  step_bytes += type_nbytes(onorm.type, d);
  emb_type = temb.type;
  emb = dmalloc(type_nbytes(temb.type, temb.nelem));
  if (!emb) return fail(FA_ERR_OOM, "embedding allocation failed");
  CUDA_TRY(cudaMemcpy(emb, temb.data, type_nbytes(temb.type, temb.nelem), cudaMemcpyHostToDevice));
  step_bytes += type_nbytes(temb.type, d);  // one embedding row per token
  if (!tied) {
    if ((rc = build_plan(*this, head, {out}, {0}, false, d, {V}, pick_cw(out.type, V, false), staging, staging2)))
      return rc;
    step_bytes += head.native_bytes;
  } else {
    step_bytes += type_nbytes(temb.type, temb.nelem);
  }
  // numerics constants computed on the host exactly as the reference does
  attn_scale = 1.0f / std::sqrt((float)hd);  // src/tensor.rs:486
  if ((rc = ensure_rope(std::max<uint32_t>(cfg.context_len, 16)))) return rc;
  part = (float *)dmalloc(part_floats * sizeof(float));
  counters = (uint32_t *)dmalloc((size_t)max_chunks * sizeof(uint32_t));
  if (!part || !counters) return fail(FA_ERR_OOM, "GEMV scratch allocation failed");
  CUDA_TRY(cudaMemset(counters, 0, (size_t)max_chunks * sizeof(uint32_t)));
  if ((rc = alloc_workspace(ws))) return rc;
  red_ok = W == 1 && !tied && head.mma && cfg.n_ff_used % 4 == 0;
  for (const LayerW &lw : layers) red_ok = red_ok && lw.qkv.mma && lw.o.mma && lw.gateup.mma && lw.down.mma;
  if (W > 1) {
    // the collective replaces the epilogues' sum-of-squares partials with a
    // prologue that squares x itself: the tensor-core GEMV's mode only
    for (const LayerW &lw : layers)
      if (!lw.qkv.mma || !lw.o.mma || !lw.gateup.mma || !lw.down.mma || !head.mma)
        return fail(FA_ERR_UNSUPPORTED, "tensor parallelism needs Q4_K / Q6_K / Q8_0 / Q4_0 projections");
    if (!(ar_send = (float *)dmalloc(((size_t)d + 8) * 4))) return fail(FA_ERR_OOM, "all-reduce buffer");
    // one all-reduce outside any graph capture: NCCL sets up its peer
    // connections here rather than inside the first captured step
    CUDA_TRY(cudaMemsetAsync(ar_send, 0, ((size_t)d + 8) * 4, stream));
    if ((rc = tp.all_reduce(ar_send, ar_send, d, stream)) || (rc = sync())) return rc;
  }
  if ((rc = setup_step_kernel())) return rc;
  gguf.reset();  // host mapping no longer needed
  return FA_OK;
}

// ---------------------------------------------------------------------------
KvCache::~KvCache() {
  if (m) {
    cudaSetDevice(m->device);
    m->live_kv.erase(this);
    if (m->graph_kv == this) {
      if (m->graph) cudaGraphExecDestroy(m->graph);
      m->graph = nullptr;
      m->graph_kv = nullptr;
    }
    if (m->step_kv == this) m->step_kv = nullptr;
  }
  cudaFree(base);
  cudaFree(page_table);
}

KvView KvCache::view() const {
  KvView v;
  v.base = base;
  v.layer_stride = layer_stride;
  v.page_table = page_table;
  v.max_pages = max_pages;
  v.n_kv = m->cfg.n_kv_heads;
  v.head_dim = m->cfg.head_dim;
  v.f16 = f16;
  return v;
}

GemvParams Model::gemv_base(const GemvPlan &P) const {
  GemvParams p{};
  p.w = P.w;
  p.chunks = P.d_chunks;
  p.n_chunks = (uint32_t)P.chunks.size();
  p.ranges = P.d_ranges;
  p.contrib = P.d_contrib;
  p.n_ctas = P.n_ctas;
  p.max_chunks_per_cta = P.max_chunks_per_cta;
  p.K = P.K;
  p.K8 = P.K8;
  p.mma = P.mma ? 1 : 0;
  p.n_stages = P.n_stages;
  p.max_units = P.max_units;
  p.CW = P.CW;
  p.stage_bytes = P.stage_bytes;
  p.x_slot = P.x_slot;
  p.part = part;
  p.counters = counters;
  p.withhold_weights = dbg_withhold;
  p.wait_limit_ns = dbg_wait_ns;
  return p;
}

int Model::enqueue_embed(Workspace &w, SeqState *st) {
  EmbedParams ep{};
  ep.emb = (const uint8_t *)emb;
  ep.feed = w.feed;
  ep.type = emb_type;
  ep.d = cfg.n_embd;
  ep.vocab = cfg.vocab_size;
  ep.x = w.x;
  ep.ssq_out = w.ssq_e;
  ep.n_ssq = embed_ctas;
  ep.state = st;
  return launch_embed(ep, pdl, stream) ? fail(FA_ERR_CUDA, "embed launch failed") : FA_OK;
}

bool Model::raw_qkv_ok() const {
  // the batch-1 paged attention takes raw q/k/v; its o projection combines the splits
  return use_red() && !layers.empty() && attn_fused(0) && (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim % 4 == 0;
}

int Model::enqueue_qkv(uint32_t l, Workspace &w, const KvCache &kv, uint32_t seq, SeqState *st, bool raw) {
  const LayerW &lw = layers[l];
  GemvParams p = gemv_base(lw.qkv);
  p.pro = kProRmsNorm;
  p.in = w.x;
  p.norm_w = lw.attn_norm;
  p.ssq = l == 0 ? w.ssq_e : w.ssq_d;
  p.n_ssq = l == 0 ? embed_ctas : layers[l - 1].down.parts();
  if (l > 0 && (tp.world > 1 || use_red())) {  // x came from an all-reduce or red.adds: the prologue sums its squares
    p.ssq = nullptr;
    p.n_ssq = 0;
  }
  if (use_red()) {  // the gate/up sums of the previous layer were read by its down launch, which completed
    p.zero = w.gu;
    p.n_zero = 2 * cfg.n_ff_used;
  }
  p.eps = cfg.norm_eps;
  p.epi = kEpiQkv;
  p.out = w.q;
  p.q_dim = cfg.n_heads * cfg.head_dim;
  p.kv_dim = cfg.n_kv_heads * cfg.head_dim;
  p.rope_tab = rope_tab;
  p.rope_max = rope_max;
  p.kv = kv.view();
  p.seq = seq;
  p.layer = l;
  p.state = st;
  if (raw) {  // q | k | v sums by red.add; RoPE and the cache append happen in the attention
    p.epi = kEpiRed;
    p.out = w.qkv_raw;
  }
  return launch_gemv(p, pdl, stream) ? fail(FA_ERR_CUDA, "qkv gemv launch failed") : FA_OK;
}

bool Model::attn_fused(uint32_t l) const {
  AttnParams ap{};
  SeqState dummy{};  // the support test only asks that a state exists
  ap.q_rows = 1;
  ap.state = &dummy;
  ap.kv.head_dim = cfg.head_dim;
  ap.kv.n_kv = cfg.n_kv_heads;
  ap.n_heads = cfg.n_heads;
  ap.splits = attn_splits;
  const GemvPlan &o = layers[l].o;
  return attn_paged_supported(ap) && o.mma && o.K == cfg.n_heads * cfg.head_dim &&
         (uint64_t)cfg.n_heads * (attn_splits + 1) <= gemv_mma_table_words();
}

int Model::enqueue_attn(uint32_t l, Workspace &w, const KvCache &kv, uint32_t seq, SeqState *st, bool raw) {
  AttnParams ap{};
  ap.q = w.q;
  ap.q_rows = 1;
  ap.kv = kv.view();
  ap.seq = seq;
  ap.layer = l;
  ap.n_heads = cfg.n_heads;
  ap.splits = attn_splits;
  ap.scale = attn_scale;
  ap.part = w.attn_part;
  ap.counters = w.attn_cnt;
  ap.out = w.attn_out;
  ap.state = st;
  ap.partials_only = attn_fused(l) ? 1 : 0;
  ap.early_kv = capturing_step && pdl ? 1 : 0;
  if (raw) {
    ap.qkv_raw = w.qkv_raw;
    ap.rope_tab = rope_tab;
    ap.rope_max = rope_max;
  }
  return launch_attention(ap, pdl, stream) ? fail(FA_ERR_CUDA, "attention launch failed") : FA_OK;
}

int Model::enqueue_post_attn(uint32_t l, Workspace &w, SeqState *st, float *hidden_dump, bool raw) {
  const LayerW &lw = layers[l];
  GemvParams p = gemv_base(lw.o);
  p.pro = kProPlain;
  p.in = w.attn_out;
  if (attn_fused(l)) {
    p.pro = kProAttn;
    p.attn_part = w.attn_part;
    p.attn_splits = attn_splits;
    p.attn_hd = cfg.head_dim;
  }
  p.epi = kEpiResid;
  p.resid = w.x;
  p.ssq_out = w.ssq_o;
  p.state = st;
  // tensor parallel: rank 0 adds its partial sums to the residual in place,
  // the others store theirs; the all-reduce then leaves x + sum on every rank
  const bool part = tp.world > 1 && tp.rank > 0, red = use_red();
  if (part) {
    p.epi = kEpiStore;
    p.out = ar_send;
  }
  if (red) {  // x += o: every CTA adds its split-K piece into the residual
    p.epi = kEpiRed;
    p.out = w.x;
  }
  if (raw) {  // the attention, which read the raw q/k/v sums, has completed
    p.zero = w.qkv_raw;
    p.n_zero = (cfg.n_heads + 2 * cfg.n_kv_heads) * cfg.head_dim;
  }
  int rc;
  if (launch_gemv(p, pdl, stream)) return fail(FA_ERR_CUDA, "o gemv launch failed");
  if (tp.world > 1 && (rc = tp_reduce(w.x, ar_send, cfg.n_embd))) return rc;
  p = gemv_base(lw.gateup);
  p.pro = kProRmsNorm;
  p.in = w.x;
  p.norm_w = lw.ffn_norm;
  p.ssq = tp.world > 1 ? nullptr : w.ssq_o;
  p.n_ssq = tp.world > 1 ? 0 : lw.o.parts();
  p.eps = cfg.norm_eps;
  p.epi = kEpiSwiglu;
  p.out = w.h;
  p.state = st;
  if (red) {  // gate and up sums into gu (zeroed by this layer's qkv launch); SwiGLU in down's prologue
    p.ssq = nullptr;
    p.n_ssq = 0;
    p.epi = kEpiRed;
    p.out = w.gu;
    p.red_half = cfg.n_ff_used;
  }
  if (launch_gemv(p, pdl, stream)) return fail(FA_ERR_CUDA, "gate/up gemv launch failed");
  p = gemv_base(lw.down);
  p.pro = kProPlain;
  p.in = w.h;
  p.epi = kEpiResid;
  p.resid = w.x;
  p.ssq_out = w.ssq_d;
  p.state = st;
  if (red) {  // x += down(silu(gate) * up)
    p.pro = kProSwiglu;
    p.in = w.gu;
    p.in2 = w.gu + cfg.n_ff_used;
    p.epi = kEpiRed;
    p.out = w.x;
  }
  if (part) {
    p.epi = kEpiStore;
    p.out = ar_send;
  }
  if (launch_gemv(p, pdl, stream)) return fail(FA_ERR_CUDA, "down gemv launch failed");
  if (tp.world > 1 && (rc = tp_reduce(w.x, ar_send, cfg.n_embd))) return rc;
  if (hidden_dump)
    CUDA_TRY(cudaMemcpyAsync(hidden_dump, w.x, cfg.n_embd * 4, cudaMemcpyDeviceToDevice, stream));
  return FA_OK;
}

int Model::enqueue_head(Workspace &w, SeqState *st) {
  const uint32_t L = cfg.n_layers;
  const float *ssq_in = L ? w.ssq_d : w.ssq_e;
  const uint32_t n_ssq = L ? layers[L - 1].down.parts() : embed_ctas;
  if (!tied) {
    GemvParams p = gemv_base(head);
    p.pro = kProRmsNorm;
    p.in = w.x;
    p.norm_w = out_norm;
    const bool self_ssq = tp.world > 1 || (use_red() && L > 0);
    p.ssq = self_ssq ? nullptr : ssq_in;
    p.n_ssq = self_ssq ? 0 : n_ssq;
    p.eps = cfg.norm_eps;
    p.epi = kEpiLogits;
    p.out = w.logits;
    p.state = st;
    return launch_gemv(p, pdl, stream) ? fail(FA_ERR_CUDA, "head gemv launch failed") : FA_OK;
  }
  TiedHeadParams tp{};
  tp.emb = (const uint8_t *)emb;
  tp.type = emb_type;
  tp.d = cfg.n_embd;
  tp.vocab = cfg.vocab_size;
  tp.x = w.x;
  tp.norm_w = out_norm;
  tp.ssq = ssq_in;
  tp.n_ssq = n_ssq;
  tp.eps = cfg.norm_eps;
  tp.logits = w.logits;
  tp.state = st;
  return launch_tied_head(tp, pdl, stream) ? fail(FA_ERR_CUDA, "tied head launch failed") : FA_OK;
}

int Model::enqueue_step(const KvCache &kv, uint32_t seq, Workspace &w, float *hidden_dump) {
  int rc;
  if ((rc = enqueue_embed(w, w.state))) return rc;
  const bool raw = raw_qkv_ok();
  for (uint32_t l = 0; l < cfg.n_layers; ++l) {
    if ((rc = enqueue_qkv(l, w, kv, seq, w.state, raw))) return rc;
    if ((rc = enqueue_attn(l, w, kv, seq, w.state, raw))) return rc;
    if ((rc = enqueue_post_attn(l, w, w.state, hidden_dump ? hidden_dump + (size_t)l * cfg.n_embd : nullptr, raw)))
      return rc;
  }
  if ((rc = enqueue_head(w, w.state))) return rc;
  if (launch_step_end(w.state, w.ids, w.max_ids, pdl, stream)) return fail(FA_ERR_CUDA, "step_end launch failed");
  return FA_OK;
}

int Model::alloc_workspace(Workspace &w) {
  const uint32_t d = cfg.n_embd, qd = cfg.n_heads * cfg.head_dim;
  w.x = (float *)dmalloc(((size_t)d + 8) * 4);  // +8: inputs are read in whole 8-row groups
  w.q = (float *)dmalloc(qd * 4);
  w.h = (float *)dmalloc(((size_t)cfg.n_ff_used + 8) * 4);
  w.logits = (float *)dmalloc((size_t)cfg.vocab_size * 4);
  w.attn_part = (float *)dmalloc((size_t)cfg.n_heads * attn_splits * (2 + cfg.head_dim) * 4);
  w.attn_out = (float *)dmalloc(((size_t)qd + 8) * 4);
  w.attn_cnt = (uint32_t *)dmalloc(cfg.n_kv_heads * 4);
  w.ssq_e = (float *)dmalloc((size_t)std::max<uint32_t>(embed_ctas, (uint32_t)n_sm) * 4);
  uint32_t n_ssq_o = 1, n_ssq_d = 1;  // sum-of-squares partials of the residual launches
  for (const LayerW &lw : layers) {
    n_ssq_o = std::max(n_ssq_o, lw.o.parts());
    n_ssq_d = std::max(n_ssq_d, lw.down.parts());
  }
  w.ssq_o = (float *)dmalloc((size_t)n_ssq_o * 4);
  w.ssq_d = (float *)dmalloc((size_t)n_ssq_d * 4);
  w.state = (SeqState *)dmalloc(sizeof(SeqState));
  const size_t gu_floats = 2 * (size_t)cfg.n_ff_used + 8, qkv_floats = qd + 2 * (size_t)cfg.n_kv_heads * cfg.head_dim + 8;
  w.gu = (float *)dmalloc(gu_floats * 4);
  w.qkv_raw = (float *)dmalloc(qkv_floats * 4);
  if (!w.x || !w.q || !w.h || !w.logits || !w.attn_part || !w.attn_out || !w.attn_cnt || !w.ssq_e || !w.ssq_o ||
      !w.ssq_d || !w.state || !w.gu || !w.qkv_raw)
    return fail(FA_ERR_OOM, "workspace allocation failed");
  CUDA_TRY(cudaMemset(w.gu, 0, gu_floats * 4));
  CUDA_TRY(cudaMemset(w.qkv_raw, 0, qkv_floats * 4));
  CUDA_TRY(cudaMemset(w.state, 0, sizeof(SeqState)));
  CUDA_TRY(cudaMemset(w.attn_cnt, 0, cfg.n_kv_heads * 4));
  CUDA_TRY(cudaMemset(w.x, 0, ((size_t)d + 8) * 4));
  CUDA_TRY(cudaMemset(w.h, 0, ((size_t)cfg.n_ff_used + 8) * 4));
  CUDA_TRY(cudaMemset(w.attn_out, 0, ((size_t)qd + 8) * 4));
  return FA_OK;
}

int Model::tp_reduce(float *x, const float *partials, size_t count) {
  return tp.all_reduce(tp.rank == 0 ? x : partials, x, count, stream);
}

int Model::sync() {
  if (tp.world <= 1) {
    const cudaError_t e = cudaStreamSynchronize(stream);
    return e == cudaSuccess ? FA_OK : fail(FA_ERR_CUDA, std::string("stream: ") + cudaGetErrorString(e));
  }
  // a peer that died leaves our collectives waiting: poll with a bound
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(stream);
    if (e == cudaSuccess) return FA_OK;
    if (e != cudaErrorNotReady) return fail(FA_ERR_CUDA, std::string("stream: ") + cudaGetErrorString(e));
    std::string msg;
    if (tp.check_async(&msg)) return fail(FA_ERR_NCCL, "collective failed: " + msg);
    if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(60)) {
      tp.abort();
      return fail(FA_ERR_TIMEOUT, "tensor-parallel step did not finish within 60 s (a peer rank stopped?)");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

// kernel launches one replay of a captured graph performs
static uint32_t count_kernel_nodes(cudaGraph_t g) {
  size_t n = 0;
  if (cudaGraphGetNodes(g, nullptr, &n) != cudaSuccess || !n) return 0;
  std::vector<cudaGraphNode_t> nodes(n);
  if (cudaGraphGetNodes(g, nodes.data(), &n) != cudaSuccess) return 0;
  uint32_t k = 0;
  for (size_t i = 0; i < n; ++i) {
    cudaGraphNodeType t;
    if (cudaGraphNodeGetType(nodes[i], &t) == cudaSuccess && t == cudaGraphNodeTypeKernel) ++k;
  }
  return k;
}

int Model::run_steps(const KvCache &kv, uint32_t seq, uint32_t n) {
  int rc;
  if (step_ok && (rc = prepare_step(kv, seq))) return rc;
  auto one_step = [&]() -> int {
    if (step_ok) {
      const int e = launch_step(step, step_smem, stream);
      if (e) return fail(FA_ERR_CUDA, std::string("step kernel launch failed: ") + cudaGetErrorString((cudaError_t)e) +
                                          " (smem " + std::to_string(step_smem) + ", " +
                                          step_occupancy_report(step, step_smem) + ")");
    } else {
      const int rc2 = enqueue_step(kv, seq, ws, nullptr);
      if (rc2) return rc2;
    }
    if (gen_sample && launch_sample(*gen_sample, 1, stream)) return fail(FA_ERR_CUDA, "sampler launch failed");
    return FA_OK;
  };
  if (!graphs) {
    for (uint32_t i = 0; i < n; ++i)
      if ((rc = one_step())) return rc;
    return FA_OK;
  }
  if (!graph || graph_kv != &kv || graph_seq != seq || graph_sample != gen_sample) {
    if (graph) {
      cudaGraphExecDestroy(graph);
      graph = nullptr;
    }
    CUDA_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    capturing_step = true;
    rc = one_step();
    capturing_step = false;
    cudaGraph_t gr = nullptr;
    cudaError_t ce = cudaStreamEndCapture(stream, &gr);
    if (rc) {
      if (gr) cudaGraphDestroy(gr);
      return rc;
    }
    if (ce != cudaSuccess) return fail(FA_ERR_CUDA, std::string("graph capture failed: ") + cudaGetErrorString(ce));
    graph_kernels = count_kernel_nodes(gr);
    ce = cudaGraphInstantiate(&graph, gr, 0);
    cudaGraphDestroy(gr);
    if (ce != cudaSuccess) return fail(FA_ERR_CUDA, std::string("graph instantiate failed: ") + cudaGetErrorString(ce));
    graph_kv = &kv;
    graph_seq = seq;
    graph_sample = gen_sample;
  }
  for (uint32_t i = 0; i < n; ++i) CUDA_TRY(cudaGraphLaunch(graph, stream));
  return FA_OK;
}

// The persistent step kernel serves models whose projections are all in the
// MMA layout with an untied head and head_dim a multiple of 8 (<= 128).
int Model::setup_step_kernel() {
  const uint32_t L = cfg.n_layers, hd = cfg.head_dim, rep = cfg.n_heads / cfg.n_kv_heads;
  bool ok = !tied && L > 0 && head.mma && hd % 8 == 0 && hd <= 128 && cfg.n_heads % cfg.n_kv_heads == 0 &&
            (rep == 1 || rep == 2 || rep == 4 || rep == 8) && attn_splits <= 64;
  for (const LayerW &lw : layers) ok = ok && lw.qkv.mma && lw.o.mma && lw.gateup.mma && lw.down.mma;
  // the tensor-core prefill needs every layer projection in the MMA layout
  tc_ok = L > 0 && (hd == 64 || hd == 128) && cfg.n_heads % cfg.n_kv_heads == 0;
  for (const LayerW &lw : layers) tc_ok = tc_ok && lw.qkv.mma && lw.o.mma && lw.gateup.mma && lw.down.mma;
  if (!ok || !want_step) return FA_OK;
  const uint32_t n_phases = 1 + 5 * L + 1, n_gemv = 4 * L + 1;
  d_phases = (StepPhase *)dmalloc(n_phases * sizeof(StepPhase));
  d_gemv = (GemvParams *)dmalloc(n_gemv * sizeof(GemvParams));
  d_step_done = (uint32_t *)dmalloc(n_phases * sizeof(uint32_t));
  d_step_sync = (uint32_t *)dmalloc(2 * sizeof(uint32_t));
  if (!d_phases || !d_gemv || !d_step_done || !d_step_sync) return fail(FA_ERR_OOM, "step plan allocation failed");
  step_ok = true;
  return FA_OK;
}

int Model::prepare_step(const KvCache &kv, uint32_t seq) {
  if (step_kv == &kv && step_seq == seq) return FA_OK;
  const uint32_t L = cfg.n_layers, KVH = cfg.n_kv_heads, hd = cfg.head_dim, rep = cfg.n_heads / KVH;
  // ring geometry shared by every GEMV phase; the attention groups' scratch
  // overlays the tables and the x slice, which sizes the x slice from below
  uint32_t stage_bytes = head.stage_bytes, max_units = head.max_units;
  for (const LayerW &lw : layers)
    for (const GemvPlan *P : {&lw.qkv, &lw.o, &lw.gateup, &lw.down}) {
      stage_bytes = std::max(stage_bytes, P->stage_bytes);
      max_units = std::max(max_units, P->max_units);
    }
  const uint32_t groups = 2, gbytes = (uint32_t)step_attn_group_bytes(rep, hd);
  // (the ring offset is rounded to 128 bytes, so grow unit by unit until it fits)
  while (gemv_mma_ring_offset(max_units) - gemv_mma_table_offset() < groups * gbytes) ++max_units;
  const uint32_t n_stages = gemv_mma_stages(stage_bytes, max_units, 227 * 1024);
  if (n_stages < 2) return fail(FA_ERR_UNSUPPORTED, "step kernel ring does not fit in shared memory");
  std::vector<StepPhase> ph;
  std::vector<GemvParams> gp;
  auto add_gemv = [&](GemvParams p, uint32_t dep, uint32_t dep_count) {
    p.stage_bytes = stage_bytes;
    p.n_stages = n_stages;
    p.max_units = max_units;
    p.done = d_step_done + ph.size();
    ph.push_back({kPhGemv, (uint32_t)gp.size(), dep, dep_count});
    gp.push_back(p);
  };
  const uint32_t grid = (uint32_t)n_sm;
  ph.push_back({kPhEmbed, 0, ~0u, 0});
  uint32_t prev = 0, prev_count = grid;  // the phase the next RMSNorm input comes from
  for (uint32_t l = 0; l < L; ++l) {
    const LayerW &lw = layers[l];
    GemvParams p = gemv_base(lw.qkv);
    p.pro = kProRmsNorm;
    p.in = ws.x;
    p.norm_w = lw.attn_norm;
    p.ssq = l == 0 ? ws.ssq_e : ws.ssq_d;
    p.n_ssq = l == 0 ? grid : layers[l - 1].down.parts();
    p.eps = cfg.norm_eps;
    p.epi = kEpiQkv;
    p.out = ws.q;
    p.q_dim = cfg.n_heads * hd;
    p.kv_dim = KVH * hd;
    p.rope_tab = rope_tab;
    p.rope_max = rope_max;
    p.kv = kv.view();
    p.seq = seq;
    p.layer = l;
    p.state = ws.state;
    const uint32_t q_qkv = (uint32_t)ph.size();
    add_gemv(p, prev, prev_count);
    const uint32_t q_attn = (uint32_t)ph.size();
    ph.push_back({kPhAttn, l, q_qkv, lw.qkv.parts()});
    p = gemv_base(lw.o);
    p.pro = kProPlain;
    p.in = ws.attn_out;
    p.epi = kEpiResid;
    p.resid = ws.x;
    p.ssq_out = ws.ssq_o;
    p.state = ws.state;
    const uint32_t q_o = (uint32_t)ph.size();
    add_gemv(p, q_attn, KVH);
    p = gemv_base(lw.gateup);
    p.pro = kProRmsNorm;
    p.in = ws.x;
    p.norm_w = lw.ffn_norm;
    p.ssq = ws.ssq_o;
    p.n_ssq = lw.o.parts();
    p.eps = cfg.norm_eps;
    p.epi = kEpiSwiglu;
    p.out = ws.h;
    p.state = ws.state;
    const uint32_t q_gu = (uint32_t)ph.size();
    add_gemv(p, q_o, lw.o.parts());
    p = gemv_base(lw.down);
    p.pro = kProPlain;
    p.in = ws.h;
    p.epi = kEpiResid;
    p.resid = ws.x;
    p.ssq_out = ws.ssq_d;
    p.state = ws.state;
    prev = (uint32_t)ph.size();
    prev_count = lw.down.parts();
    add_gemv(p, q_gu, lw.gateup.parts());
  }
  GemvParams p = gemv_base(head);
  p.pro = kProRmsNorm;
  p.in = ws.x;
  p.norm_w = out_norm;
  p.ssq = ws.ssq_d;
  p.n_ssq = layers[L - 1].down.parts();
  p.eps = cfg.norm_eps;
  p.epi = kEpiLogits;
  p.out = ws.logits;
  p.state = ws.state;
  add_gemv(p, prev, prev_count);
  CUDA_TRY(cudaMemcpy(d_phases, ph.data(), ph.size() * sizeof(StepPhase), cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemcpy(d_gemv, gp.data(), gp.size() * sizeof(GemvParams), cudaMemcpyHostToDevice));
  CUDA_TRY(cudaMemset(d_step_done, 0, ph.size() * sizeof(uint32_t)));
  CUDA_TRY(cudaMemset(d_step_sync, 0, 2 * sizeof(uint32_t)));
  StepParams sp{};
  sp.phases = d_phases;
  sp.n_phases = (uint32_t)ph.size();
  sp.gemv = d_gemv;
  AttnParams &ap = sp.attn;
  ap.q = ws.q;
  ap.q_rows = 1;
  ap.kv = kv.view();
  ap.seq = seq;
  ap.n_heads = cfg.n_heads;
  ap.splits = attn_splits;
  ap.scale = attn_scale;
  ap.part = ws.attn_part;
  ap.counters = ws.attn_cnt;
  ap.out = ws.attn_out;
  ap.state = ws.state;
  EmbedParams &ep = sp.embed;
  ep.emb = (const uint8_t *)emb;
  ep.feed = ws.feed;
  ep.type = emb_type;
  ep.d = cfg.n_embd;
  ep.vocab = cfg.vocab_size;
  ep.x = ws.x;
  ep.ssq_out = ws.ssq_e;
  ep.n_ssq = grid;
  ep.state = ws.state;
  sp.done = d_step_done;
  sp.sync = d_step_sync;
  sp.ids = ws.ids;
  sp.max_ids = ws.max_ids;
  sp.n_stages = n_stages;
  sp.stage_bytes = stage_bytes;
  sp.max_units = max_units;
  sp.attn_groups = groups;
  sp.n_ctas = grid;
  step = sp;
  step_smem = gemv_mma_ring_offset(max_units) + (size_t)n_stages * stage_bytes;
  step_kv = &kv;
  step_seq = seq;
  return FA_OK;
}

// ---------------------------------------------------------------------------
// Token-parallel prefill: per layer RMSNorm rows -> qkv GEMM -> RoPE + KV
// append -> causal attention -> o GEMM (+residual) -> RMSNorm rows -> gate/up
// GEMM -> SwiGLU -> down GEMM (+residual), in chunks of up to 2048 tokens.
// ---------------------------------------------------------------------------
constexpr uint32_t kPrefillChunk = 2048;

int Model::ensure_prefill_ws(uint32_t cap) {
  if (cap <= pws.cap) return FA_OK;
  const uint32_t d = cfg.n_embd, qd = cfg.n_heads * cfg.head_dim, F = layers[0].down.K;
  const uint32_t qkv_n = layers[0].qkv.n_out, gu_n = layers[0].gateup.n_out;
  PrefillWs w;
  w.cap = cap;
  w.tok = (uint32_t *)dmalloc((size_t)cap * 4);
  w.err = (uint32_t *)dmalloc(4);
  w.X = (float *)dmalloc((size_t)cap * d * 4);
  w.QKV = (float *)dmalloc((size_t)cap * qkv_n * 4);
  w.GU = (float *)dmalloc((size_t)cap * gu_n * 4);
  w.Xn = dmalloc((size_t)cap * d * 2);
  w.Qh = dmalloc((size_t)cap * qd * 2);
  w.Ob = dmalloc((size_t)cap * qd * 2);
  w.Hb = dmalloc((size_t)cap * F * 2);
  if (tp.rank > 0) w.Y = (float *)dmalloc((size_t)cap * d * 4);
  if (!w.tok || !w.err || !w.X || !w.QKV || !w.GU || !w.Xn || !w.Qh || !w.Ob || !w.Hb || (tp.rank > 0 && !w.Y))
    return fail(FA_ERR_OOM, "prefill workspace allocation failed");
  const uint32_t bns[3] = {64, 128, 256};
  for (int b = 0; b < 3; ++b)
    if (qgemm_make_xmap(&w.mxn[b], w.Xn, d, cap, bns[b]) || qgemm_make_xmap(&w.mob[b], w.Ob, qd, cap, bns[b]) ||
        qgemm_make_xmap(&w.mhb[b], w.Hb, F, cap, bns[b]))
      return fail(FA_ERR_CUDA, "tensor map encoding failed");
  pws = w;  // the previous buffers stay owned by `allocs` until teardown
  return ensure_qg_part((uint64_t)8 * std::min<uint32_t>(cap, 512) * std::max(d, qkv_n));
}

int Model::ensure_qg_part(uint64_t floats) {
  floats = std::max<uint64_t>(floats, qgemm_part_floats(512, (uint32_t)n_sm));
  if (floats <= qg_part_floats) return FA_OK;
  float *q = (float *)dmalloc(floats * 4);
  if (!q) return fail(FA_ERR_OOM, "GEMM split-K workspace allocation failed");
  qg_part = q;
  qg_part_floats = floats;
  return FA_OK;
}

int Model::run_qgemm(const GemvPlan &P, const QgXMap &map, uint32_t T, float *out, uint32_t ldo, int epi, bool red,
                     float *zero, uint64_t n_zero) {
  QgParams p{};
  p.part = qg_part;
  p.part_floats = qg_part_floats;
  p.w = P.w;
  p.chunks = P.d_chunks;
  p.tiles = P.d_qg_tiles;
  p.n_tiles = (uint32_t)P.qg_tiles.size();
  p.K = P.K;
  p.T = T;
  p.out = out;
  p.ldo = ldo;
  p.epi = epi;
  p.err = pws.err;
  p.prefetch = P.qg_prefetch;
  // split tiles by red.add into a destination that is zero (store: a later
  // batched-decode GEMM clears it, see `zero`) or the residual; one
  // rank only (the partial-sum buffers of tensor-parallel ranks are not kept
  // zero); the launcher keeps it to 64-token tiles
  p.red = red && tp.world == 1 && !dbg_fixed_order ? 1u : 0u;
  p.zero = zero;
  p.n_zero = n_zero;
  return launch_qgemm(p, map, (uint32_t)n_sm, stream) ? fail(FA_ERR_CUDA, "token GEMM launch failed") : FA_OK;
}

int Model::prefill_tc(KvCache &kv, uint32_t seq, const uint32_t *toks, uint32_t n, uint32_t start_pos) {
  if (!tc_ok) return fail(FA_ERR_UNSUPPORTED, "tensor-core prefill needs every projection in the MMA layout");
  const uint32_t d = cfg.n_embd, hd = cfg.head_dim, Hq = cfg.n_heads, Hkv = cfg.n_kv_heads;
  const uint32_t F = layers[0].down.K, qkv_n = layers[0].qkv.n_out, gu_n = layers[0].gateup.n_out;
  int rc;
  if ((rc = ensure_rope(start_pos + n + 1)) || (rc = ensure_prefill_ws(std::min(n, kPrefillChunk)))) return rc;
  CUDA_TRY(cudaMemsetAsync(pws.err, 0, 4, stream));
  const KvView kvv = kv.view();
  const float scale_log2 = (1.0f / std::sqrt((float)hd)) * 1.4426950408889634f;
  uint32_t T = 0;
  for (uint32_t i0 = 0; i0 < n; i0 += pws.cap) {
    T = std::min(pws.cap, n - i0);
    const uint32_t len0 = kv.len[seq] + i0, pos0 = start_pos + i0;
    const int b = T <= 64 ? 0 : T <= 128 ? 1 : 2;
    CUDA_TRY(cudaMemcpyAsync(pws.tok, toks + i0, (size_t)T * 4, cudaMemcpyHostToDevice, stream));
    if (launch_embed_rows(emb, emb_type, pws.tok, T, d, cfg.vocab_size, pws.X, pws.err, stream))
      return fail(FA_ERR_CUDA, "embed launch failed");
    for (uint32_t l = 0; l < cfg.n_layers; ++l) {
      const LayerW &lw = layers[l];
      if (launch_norm_rows_h(pws.X, lw.attn_norm, cfg.norm_eps, T, d, pws.Xn, pws.err, stream))
        return fail(FA_ERR_CUDA, "norm launch failed");
      if ((rc = run_qgemm(lw.qkv, pws.mxn[b], T, pws.QKV, qkv_n, kQgStore))) return rc;
      if (launch_rope_kv_rows(pws.QKV, T, Hq, Hkv, hd, rope_tab, rope_max, pos0, len0, kvv, seq, l, pws.Qh, pws.err,
                              stream))
        return fail(FA_ERR_CUDA, "rope launch failed");
      AttnRowsParams ap{};
      ap.qh = pws.Qh;
      ap.T = T;
      ap.Hq = Hq;
      ap.Hkv = Hkv;
      ap.hd = hd;
      ap.len0 = len0;
      ap.kv = kvv;
      ap.seq = seq;
      ap.layer = l;
      ap.scale_log2 = scale_log2;
      ap.out = pws.Ob;
      if (launch_attn_rows(ap, stream)) return fail(FA_ERR_CUDA, "prefill attention launch failed");
      // tensor parallel: rank 0 adds its partial sums to X, the others store
      // theirs in Y; the all-reduce leaves X + sum on every rank
      float *o_dst = tp.rank > 0 ? pws.Y : pws.X;
      const int o_epi = tp.rank > 0 ? kQgStore : kQgResid;
      if ((rc = run_qgemm(lw.o, pws.mob[b], T, o_dst, d, o_epi))) return rc;
      if (tp.world > 1 && (rc = tp_reduce(pws.X, pws.Y, (size_t)T * d))) return rc;
      if (launch_norm_rows_h(pws.X, lw.ffn_norm, cfg.norm_eps, T, d, pws.Xn, pws.err, stream))
        return fail(FA_ERR_CUDA, "norm launch failed");
      if ((rc = run_qgemm(lw.gateup, pws.mxn[b], T, pws.GU, gu_n, kQgStore))) return rc;
      if (launch_swiglu_rows(pws.GU, T, F, lw.gateup.CW, pws.Hb, pws.err, stream))
        return fail(FA_ERR_CUDA, "swiglu launch failed");
      if ((rc = run_qgemm(lw.down, pws.mhb[b], T, o_dst, d, o_epi))) return rc;
      if (tp.world > 1 && (rc = tp_reduce(pws.X, pws.Y, (size_t)T * d))) return rc;
    }
  }
  // the last token through the decode head: logits + argmax
  const uint32_t n_ssq = layers[cfg.n_layers - 1].down.parts();
  if (launch_last_row(pws.X, T - 1, d, ws.x, ws.ssq_d, n_ssq, stream)) return fail(FA_ERR_CUDA, "last row launch failed");
  SeqState st{};
  st.pos = start_pos + n - 1;
  st.len = kv.len[seq] + n - 1;
  CUDA_TRY(cudaMemcpyAsync(ws.state, &st, sizeof st, cudaMemcpyHostToDevice, stream));
  if ((rc = enqueue_head(ws, ws.state))) return rc;
  uint32_t e = 0;
  CUDA_TRY(cudaMemcpyAsync(&e, pws.err, 4, cudaMemcpyDeviceToHost, stream));
  if ((rc = sync())) return rc;
  if (e & kErrWaitTimeout) return fail(FA_ERR_TIMEOUT, "prefill: a bounded device wait gave up");
  if (e & kErrBadToken) return fail(FA_ERR_INVALID, "token id out of range");
  if (e & kErrContext) return fail(FA_ERR_CONTEXT, "position or KV capacity exceeded");
  if (e & kErrRange) return fail(FA_ERR_UNSUPPORTED, "an activation exceeds the f16 range of the tensor-core prefill");
  return FA_OK;
}

// ---------------------------------------------------------------------------
// Batched decode: b sequences advance one token per step; the projections run
// as f16 tcgen05 GEMMs with T = b, attention per row over the row's own cache
// sequence, then Sampler::sample per row.  One step is a captured CUDA graph.
// ---------------------------------------------------------------------------
int Model::ensure_batch_ws(uint32_t b) {
  if (b <= bws.cap) return FA_OK;
  const uint32_t d = cfg.n_embd, qd = cfg.n_heads * cfg.head_dim, F = layers[0].down.K, V = cfg.vocab_size;
  const uint32_t qkv_n = layers[0].qkv.n_out, gu_n = layers[0].gateup.n_out, KVH = cfg.n_kv_heads;
  BatchWs w;
  w.cap = b;
  w.splits = std::max<uint32_t>(1, std::min<uint32_t>(32, (8 * (uint32_t)n_sm + b * KVH - 1) / (b * KVH)));
  w.X = (float *)dmalloc((size_t)b * d * 4);
  w.QKV = (float *)dmalloc((size_t)b * qkv_n * 4);
  w.Qf = (float *)dmalloc((size_t)b * qd * 4);
  w.Of = (float *)dmalloc((size_t)b * qd * 4);
  w.GU = (float *)dmalloc((size_t)b * gu_n * 4);
  w.logits = (float *)dmalloc((size_t)b * V * 4);
  w.part = (float *)dmalloc((size_t)b * cfg.n_heads * w.splits * (2 + cfg.head_dim) * 4);
  w.Xn = dmalloc((size_t)b * d * 2);
  w.Oh = dmalloc((size_t)b * qd * 2);
  w.Hb = dmalloc((size_t)b * F * 2);
  w.counters = (uint32_t *)dmalloc((size_t)b * KVH * 4);
  w.err = (uint32_t *)dmalloc(4);
  w.step = (uint32_t *)dmalloc(4);
  w.states = (SeqState *)dmalloc((size_t)b * sizeof(SeqState));
  if (tp.rank > 0 && !(w.Y = (float *)dmalloc((size_t)b * d * 4)))
    return fail(FA_ERR_OOM, "batched decode workspace allocation failed");
  if (!w.X || !w.QKV || !w.Qf || !w.Of || !w.GU || !w.logits || !w.part || !w.Xn || !w.Oh || !w.Hb || !w.counters ||
      !w.err || !w.step || !w.states)
    return fail(FA_ERR_OOM, "batched decode workspace allocation failed");
  CUDA_TRY(cudaMemset(w.counters, 0, (size_t)b * KVH * 4));
  // the token GEMMs add split tiles into these; the o / down GEMMs clear them
  CUDA_TRY(cudaMemset(w.QKV, 0, (size_t)b * qkv_n * 4));
  CUDA_TRY(cudaMemset(w.GU, 0, (size_t)b * gu_n * 4));
  const uint32_t bn = b <= 64 ? 64 : b <= 128 ? 128 : 256;
  if (qgemm_make_xmap(&w.mxn, w.Xn, d, b, bn) || qgemm_make_xmap(&w.moh, w.Oh, qd, b, bn) ||
      qgemm_make_xmap(&w.mhb, w.Hb, F, b, bn))
    return fail(FA_ERR_CUDA, "tensor map encoding failed");
  bws = w;
  return ensure_qg_part((uint64_t)8 * b * std::max(d, qkv_n));
}

int Model::enqueue_batch_step(const KvCache &kv, uint32_t b, const SamplerParams &sp, uint32_t *hist,
                              uint32_t max_steps) {
  const uint32_t d = cfg.n_embd, hd = cfg.head_dim, Hq = cfg.n_heads, Hkv = cfg.n_kv_heads;
  const uint32_t F = layers[0].down.K, qkv_n = layers[0].qkv.n_out, gu_n = layers[0].gateup.n_out;
  const KvView kvv = kv.view();
  int rc;
  uint32_t *tok = sp.ids;  // the sampler's ids are the next step's input tokens
  if (launch_embed_rows(emb, emb_type, tok, b, d, cfg.vocab_size, bws.X, bws.err, stream))
    return fail(FA_ERR_CUDA, "embed launch failed");
  for (uint32_t l = 0; l < cfg.n_layers; ++l) {
    const LayerW &lw = layers[l];
    if (launch_norm_rows_h(bws.X, lw.attn_norm, cfg.norm_eps, b, d, bws.Xn, bws.err, stream))
      return fail(FA_ERR_CUDA, "norm launch failed");
    if ((rc = run_qgemm(lw.qkv, bws.mxn, b, bws.QKV, qkv_n, kQgStore, true))) return rc;
    if (launch_rope_kv_batch(bws.QKV, b, Hq, Hkv, hd, rope_tab, rope_max, bws.states, kvv, 0, l, bws.Qf, bws.err,
                             stream))
      return fail(FA_ERR_CUDA, "rope launch failed");
    AttnParams ap{};
    ap.q = bws.Qf;
    ap.q_rows = b;
    ap.kv = kvv;
    ap.layer = l;
    ap.n_heads = Hq;
    ap.splits = bws.splits;
    ap.scale = attn_scale;
    ap.part = bws.part;
    ap.counters = bws.counters;
    ap.out = bws.Of;
    ap.out_h = bws.Oh;  // the combine writes the o GEMM's f16 operand directly
    ap.err = bws.err;
    ap.state = bws.states;
    ap.row_states = bws.states;
    ap.row_seq0 = 0;
    if (launch_attn_decode_rows(ap, stream)) return fail(FA_ERR_CUDA, "batched attention launch failed");
    float *o_dst = tp.rank > 0 ? bws.Y : bws.X;  // as in prefill_tc
    const int o_epi = tp.rank > 0 ? kQgStore : kQgResid;
    // o clears q|k|v (read by the RoPE kernel before it) for the next layer's
    // qkv red.adds; down clears gate/up (read by SwiGLU) likewise
    if ((rc = run_qgemm(lw.o, bws.moh, b, o_dst, d, o_epi, true, bws.QKV, (uint64_t)b * qkv_n))) return rc;
    if (tp.world > 1 && (rc = tp_reduce(bws.X, bws.Y, (size_t)b * d))) return rc;
    if (launch_norm_rows_h(bws.X, lw.ffn_norm, cfg.norm_eps, b, d, bws.Xn, bws.err, stream))
      return fail(FA_ERR_CUDA, "norm launch failed");
    if ((rc = run_qgemm(lw.gateup, bws.mxn, b, bws.GU, gu_n, kQgStore, true))) return rc;
    if (launch_swiglu_rows(bws.GU, b, F, lw.gateup.CW, bws.Hb, bws.err, stream))
      return fail(FA_ERR_CUDA, "swiglu launch failed");
    if ((rc = run_qgemm(lw.down, bws.mhb, b, o_dst, d, o_epi, true, bws.GU, (uint64_t)b * gu_n))) return rc;
    if (tp.world > 1 && (rc = tp_reduce(bws.X, bws.Y, (size_t)b * d))) return rc;
  }
  if (launch_norm_rows_h(bws.X, out_norm, cfg.norm_eps, b, d, bws.Xn, bws.err, stream))
    return fail(FA_ERR_CUDA, "norm launch failed");
  if ((rc = run_qgemm(head, bws.mxn, b, bws.logits, cfg.vocab_size, kQgStore))) return rc;
  if (launch_sample(sp, b, stream)) return fail(FA_ERR_CUDA, "sampler launch failed");
  if (launch_batch_step_end(bws.states, b, tok, hist, max_steps, bws.step, stream))
    return fail(FA_ERR_CUDA, "step end launch failed");
  return FA_OK;
}

int Model::decode_batch(KvCache &kv, uint32_t b, const uint32_t *tok, const uint32_t *pos, SamplerParams sp,
                        uint32_t steps, uint32_t *ids_host, float *logits_host) {
  if (!tc_ok || tied || !head.mma)
    return fail(FA_ERR_UNSUPPORTED, "batched decode needs every projection and the output head in the MMA layout");
  if (!b || b > kv.n_seq) return fail(FA_ERR_INVALID, "batched decode: sequence count out of range");
  uint32_t max_pos = 0;
  for (uint32_t r = 0; r < b; ++r) {
    if (tok[r] >= cfg.vocab_size) return fail(FA_ERR_INVALID, "token id out of range");
    if ((uint64_t)kv.len[r] + steps > kv.max_ctx) return fail(FA_ERR_CONTEXT, "KV cache capacity exceeded");
    max_pos = std::max(max_pos, pos[r] + steps);
  }
  int rc;
  if ((rc = ensure_rope(max_pos + 1)) || (rc = ensure_batch_ws(b))) return rc;
  std::vector<SeqState> st(b);
  for (uint32_t r = 0; r < b; ++r) {
    st[r] = SeqState{};
    st[r].pos = pos[r];
    st[r].len = kv.len[r];
    st[r].token = tok[r];
  }
  uint32_t *hist = nullptr;
  CUDA_TRY(cudaMalloc(&hist, (size_t)steps * b * 4));
  struct Free {
    void *p;
    ~Free() { cudaFree(p); }
  } free_hist{hist};
  CUDA_TRY(cudaMemcpyAsync(bws.states, st.data(), b * sizeof(SeqState), cudaMemcpyHostToDevice, stream));
  CUDA_TRY(cudaMemcpyAsync(sp.ids, tok, (size_t)b * 4, cudaMemcpyHostToDevice, stream));
  CUDA_TRY(cudaMemsetAsync(bws.step, 0, 4, stream));
  CUDA_TRY(cudaMemsetAsync(bws.err, 0, 4, stream));
  sp.logits = bws.logits;
  sp.ld = cfg.vocab_size;
  sp.n = cfg.vocab_size;
  sp.row0 = 0;
  sp.state = nullptr;
  sp.observe = 1;
  if (logits_host) {  // per-step logits requested: plain launches, a copy after each step
    for (uint32_t s = 0; s < steps; ++s) {
      if ((rc = enqueue_batch_step(kv, b, sp, hist, steps))) return rc;
      CUDA_TRY(cudaMemcpyAsync(logits_host + (size_t)s * b * cfg.vocab_size, bws.logits,
                               (size_t)b * cfg.vocab_size * 4, cudaMemcpyDeviceToHost, stream));
    }
  } else {
    cudaGraph_t gr = nullptr;
    cudaGraphExec_t ge = nullptr;
    CUDA_TRY(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal));
    rc = enqueue_batch_step(kv, b, sp, hist, steps);
    const cudaError_t ce = cudaStreamEndCapture(stream, &gr);
    if (rc) {
      if (gr) cudaGraphDestroy(gr);
      return rc;
    }
    if (ce != cudaSuccess) return fail(FA_ERR_CUDA, std::string("graph capture failed: ") + cudaGetErrorString(ce));
    const cudaError_t ie = cudaGraphInstantiate(&ge, gr, 0);
    cudaGraphDestroy(gr);
    if (ie != cudaSuccess) return fail(FA_ERR_CUDA, std::string("graph instantiate failed: ") + cudaGetErrorString(ie));
    cudaError_t le = cudaSuccess;
    for (uint32_t s = 0; s < steps && le == cudaSuccess; ++s) le = cudaGraphLaunch(ge, stream);
    cudaGraphExecDestroy(ge);
    if (le != cudaSuccess) return fail(FA_ERR_CUDA, std::string("graph launch failed: ") + cudaGetErrorString(le));
  }
  uint32_t e = 0;
  CUDA_TRY(cudaMemcpyAsync(ids_host, hist, (size_t)steps * b * 4, cudaMemcpyDeviceToHost, stream));
  CUDA_TRY(cudaMemcpyAsync(&e, bws.err, 4, cudaMemcpyDeviceToHost, stream));
  if ((rc = sync())) return rc;
  if (e & kErrWaitTimeout) return fail(FA_ERR_TIMEOUT, "batched decode: a bounded device wait gave up");
  if (e & kErrBadToken) return fail(FA_ERR_INVALID, "token id out of range");
  if (e & kErrContext) return fail(FA_ERR_CONTEXT, "position or KV capacity exceeded");
  if (e & kErrRange) return fail(FA_ERR_UNSUPPORTED, "an activation exceeds the f16 range of the tensor-core path");
  for (uint32_t r = 0; r < b; ++r) kv.len[r] += steps;
  return FA_OK;
}

}  // namespace fa

