// Host runtime of the device token loop: model weights in device memory,
// KV cache, per-sequence workspaces and the enqueue of one decode step.
#pragma once
#include <cuda_runtime.h>

#include <memory>
#include <set>
#include <string>
#include <vector>

#include "fa_host.hpp"
#include "fa_kernels.hpp"
#include "gguf.hpp"
#include "tp.hpp"

namespace fa {

struct GemvPlan {
  std::vector<ChunkDesc> chunks;
  std::vector<CtaRange> ranges;
  std::vector<uint32_t> contrib;  // per chunk: partial slot of each contributing CTA
  ChunkDesc *d_chunks = nullptr;
  CtaRange *d_ranges = nullptr;
  uint32_t *d_contrib = nullptr;
  const uint8_t *w = nullptr;
  bool mma = false;           // MMA tile layout (k_gemv_mma)
  uint32_t K = 0, K8 = 0, CW = 256, stage_bytes = 16384, x_slot = 64, n_stages = 0, max_units = 0;
  uint32_t n_ctas = 0, max_chunks_per_cta = 1;
  uint64_t native_bytes = 0;  // algorithmic bytes (native GGML blocks)
  std::vector<QgTile> qg_tiles;  // token-parallel GEMM output tiles (MMA layout only)
  QgTile *d_qg_tiles = nullptr;
  uint32_t qg_prefetch = 0;      // kQ8_0 / kQ4_0 when every chunk has that type (the GEMM's prefetch ring), else 0
  uint32_t n_out = 0;            // width of the launch output space
  // epilogue completions of one launch: one per chunk (its last arriving
  // CTA), each leaving one sum-of-squares partial (residual launches) and
  // one `done` count
  uint32_t parts() const { return (uint32_t)chunks.size(); }
};

struct LayerW {
  GemvPlan qkv, o, gateup, down;
  float *attn_norm = nullptr, *ffn_norm = nullptr;
};

struct Workspace {
  float *x = nullptr, *q = nullptr, *h = nullptr, *logits = nullptr, *attn_part = nullptr, *attn_out = nullptr;
  uint32_t *attn_cnt = nullptr;
  float *ssq_e = nullptr, *ssq_o = nullptr, *ssq_d = nullptr;
  float *gu = nullptr;         // red.add mode: gate sums [F] then up sums [F] (zero outside gate/up..down)
  float *qkv_raw = nullptr;    // raw-qkv mode: q | k | v sums of the qkv launch (zero outside qkv..attention)
  float *hidden = nullptr;     // optional per-layer dump target
  SeqState *state = nullptr;
  uint32_t *ids = nullptr;     // generated ids (device)
  uint32_t max_ids = 0;
  uint32_t *feed = nullptr;    // tokens fed before argmax continuation (device)
  uint32_t max_feed = 0;
};

struct KvCache;

// buffers of the token-parallel (tensor-core) prefill, `cap` tokens per chunk
struct PrefillWs {
  uint32_t cap = 0;
  uint32_t *tok = nullptr, *err = nullptr;
  float *X = nullptr, *QKV = nullptr, *GU = nullptr;
  float *Y = nullptr;  // tensor parallel, ranks > 0: this rank's o / down partial sums [cap][d]
  void *Xn = nullptr, *Qh = nullptr, *Ob = nullptr, *Hb = nullptr;
  QgXMap mxn[3], mob[3], mhb[3];  // TMA maps of Xn, Ob, Hb for 64, 128, 256 tokens per tile
};

// buffers of the batched decode step, `cap` sequences
struct BatchWs {
  uint32_t cap = 0, splits = 1;
  float *X = nullptr, *QKV = nullptr, *Qf = nullptr, *Of = nullptr, *GU = nullptr, *logits = nullptr, *part = nullptr;
  float *Y = nullptr;  // tensor parallel, ranks > 0: o / down partial sums [cap][d]
  void *Xn = nullptr, *Oh = nullptr, *Hb = nullptr;
  uint32_t *counters = nullptr, *err = nullptr, *step = nullptr;
  SeqState *states = nullptr;
  QgXMap mxn, moh, mhb;
};

struct Model {
  // this rank's configuration: with tensor parallelism n_heads, n_kv_heads and
  // n_ff_used are the rank's shares (the attention heads, KV heads and FFN
  // columns it holds); gcfg is the model's own configuration
  fa_config cfg{};
  fa_config gcfg{};
  TpComm tp;                     // world 1: no communicator
  float *ar_send = nullptr;      // decode step, ranks > 0: o / down partial sums [d]
  int device = 0;
  bool pdl = true, graphs = true;
  bool capturing_step = false;  // the per-step graph is being captured
  cudaStream_t stream = nullptr;
  std::unique_ptr<Gguf> gguf;
  std::vector<LayerW> layers;
  GemvPlan head;
  bool tied = false;
  void *emb = nullptr;
  int emb_type = 0;
  float *out_norm = nullptr;
  float *rope_tab = nullptr;
  uint32_t rope_max = 0;
  uint32_t attn_splits = 24;
  int n_sm = 148;
  float *part = nullptr;         // GEMV chunk partials, shared by every launch
  uint32_t *counters = nullptr;  // GEMV chunk arrival counters
  size_t part_floats = 0;
  uint32_t max_chunks = 0;
  uint32_t embed_ctas = 16;
  float attn_scale = 1.0f;
  Workspace ws;                 // single-sequence decode workspace
  std::vector<void *> allocs;   // every device allocation, freed at teardown
  std::set<KvCache *> live_kv;  // caches created on this model (detached at teardown)
  SeqState *h_state = nullptr;  // pinned host staging of the single-token forward's state
  // failure-path testing (fa_debug_set): GEMV launches withhold their weight
  // copies / use a shorter wait limit
  uint32_t dbg_withhold = 0;
  uint64_t dbg_wait_ns = 0;
  // batch-1 projections o, gate/up and down reduce their split-K pieces by
  // red.add into the destination (kEpiRed; SwiGLU and the RMSNorm sums move
  // to the next launch's prologue).  Needs every GEMV on the tensor-core
  // path, an untied head and one rank.  dbg_fixed_order: the fixed-order
  // last-arriver reduction instead (bit-reproducible run to run).
  bool red_ok = false, dbg_fixed_order = false;
  bool use_red() const { return red_ok && !dbg_fixed_order; }
  uint64_t device_bytes = 0, step_bytes = 0;
  // persistent decode-step kernel (all GEMVs in the MMA layout, untied head)
  bool want_step = false;            // requested by the load options
  bool step_ok = false;
  const KvCache *step_kv = nullptr;   // (kv, seq) the uploaded plan is for
  uint32_t step_seq = 0;
  StepParams step{};
  size_t step_smem = 0;
  StepPhase *d_phases = nullptr;
  GemvParams *d_gemv = nullptr;
  uint32_t *d_step_done = nullptr, *d_step_sync = nullptr;
  // token-parallel prefill (bf16 tensor cores)
  bool want_tc_prefill = false, tc_ok = false;
  PrefillWs pws;
  int ensure_prefill_ws(uint32_t cap);
  // red: split tiles by red.add (into a zeroed out, or the residual); zero:
  // a buffer the launch clears after its wait for the previous kernel
  int run_qgemm(const GemvPlan &P, const QgXMap &map, uint32_t T, float *out, uint32_t ldo, int epi, bool red = false,
                float *zero = nullptr, uint64_t n_zero = 0);
  // prompt tokens [0, n) at positions start_pos.., appended after the cache's
  // current length; leaves the last token's logits in ws.logits and the
  // argmax in ws.state->argmax_key
  int prefill_tc(KvCache &kv, uint32_t seq, const uint32_t *tokens_host, uint32_t n, uint32_t start_pos);
  // split-K partials of the token GEMMs (shared by prefill and batched decode)
  float *qg_part = nullptr;
  uint64_t qg_part_floats = 0;
  int ensure_qg_part(uint64_t floats);
  // batched decode (f16 tensor-core GEMMs at T = b)
  BatchWs bws;
  int ensure_batch_ws(uint32_t b);
  int enqueue_batch_step(const KvCache &kv, uint32_t b, const SamplerParams &sp, uint32_t *hist, uint32_t max_steps);
  // `steps` decode steps of sequences 0..b-1 of kv: row r starts from token
  // tok[r] at RoPE position pos[r] after its cached positions; every step
  // samples each row with sp (row r = sampler row r) and observes the id.
  // ids_host [steps][b]; logits_host (optional) [steps][b][vocab]
  int decode_batch(KvCache &kv, uint32_t b, const uint32_t *tok, const uint32_t *pos, SamplerParams sp, uint32_t steps,
                   uint32_t *ids_host, float *logits_host);
  // decode-step graph cache
  cudaGraphExec_t graph = nullptr;
  uint32_t graph_kernels = 0;   // kernel nodes of the captured step graph
  const KvCache *graph_kv = nullptr;
  uint32_t graph_seq = 0;
  // device sampler run after every step of a generation (null: argmax only)
  const SamplerParams *gen_sample = nullptr, *graph_sample = nullptr;

  ~Model();
  int load(const std::string &path, const fa_model_opts &o);
  int ensure_rope(uint32_t max_pos);
  // pieces of one token step (embed -> layers -> head -> step_end)
  int enqueue_embed(Workspace &w, SeqState *st);
  // raw: the single-token step's form — qkv adds its sums into w.qkv_raw
  // (red.add) and the attention applies RoPE and appends the new K/V itself;
  // the o launch then clears qkv_raw.  Multi-token calls (all tokens' K/V
  // appended before any attention) use the qkv epilogue instead.
  bool raw_qkv_ok() const;
  int enqueue_qkv(uint32_t l, Workspace &w, const KvCache &kv, uint32_t seq, SeqState *st, bool raw = false);
  int enqueue_attn(uint32_t l, Workspace &w, const KvCache &kv, uint32_t seq, SeqState *st, bool raw = false);
  // layer l's o projection combines the batch-1 attention's split partials
  // in its prologue (the attention then leaves them uncombined)
  bool attn_fused(uint32_t l) const;
  int enqueue_post_attn(uint32_t l, Workspace &w, SeqState *st, float *hidden_dump, bool raw = false);
  int enqueue_head(Workspace &w, SeqState *st);
  int enqueue_step(const KvCache &kv, uint32_t seq, Workspace &w, float *hidden_dump);
  int setup_step_kernel();                               // eligibility + device tables (at load)
  int prepare_step(const KvCache &kv, uint32_t seq);     // upload the step plan for (kv, seq)
  int alloc_workspace(Workspace &w);
  // run `n` steps (graph replays when enabled)
  int run_steps(const KvCache &kv, uint32_t seq, uint32_t n);
  // tensor parallel: the all-reduce that completes a row-sharded projection
  // (rank 0 added the residual itself): send = x on rank 0, own partials
  // elsewhere; recv = x on every rank
  int tp_reduce(float *x, const float *partials, size_t count);
  // wait for the model stream; under tensor parallelism bounded (60 s) and
  // watching the communicator's asynchronous error
  int sync();
  void *dmalloc(size_t bytes);
  GemvParams gemv_base(const GemvPlan &P) const;
};

struct KvCache {
  Model *m = nullptr;
  void *base = nullptr;
  uint32_t *page_table = nullptr;
  uint32_t n_seq = 0, max_ctx = 0, max_pages = 0;
  int f16 = 0;
  uint64_t layer_stride = 0;  // elements
  std::vector<uint32_t> len;  // positions stored per sequence
  ~KvCache();
  KvView view() const;
};

int config_from_gguf(const Gguf &g, fa_config *cfg);

}  // namespace fa
