// Kernel parameter blocks and launchers (host-callable, defined in *.cu).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "fa_layout.hpp"

namespace fa {

// Error flags written by device code (host reads them after a step).
enum : uint32_t {
  kErrNone = 0,
  kErrWaitTimeout = 1u << 0,  // a bounded mbarrier wait gave up
  kErrBadToken = 1u << 1,     // token id >= vocab
  kErrContext = 1u << 2,      // position beyond the KV capacity / RoPE table
  kErrRange = 1u << 3,        // an activation outside the f16 range of the tensor-core path
};

// Per-sequence decode state kept in device memory so a captured CUDA graph
// can be replayed step after step without host updates.
// The reference keeps RoPE position and cache length apart: forward(pos)
// rotates with `pos` but always appends to the end of the cache
// (src/model.rs:367-374), so both are tracked.
struct SeqState {
  uint32_t pos;        // RoPE position of the token being processed
  uint32_t len;        // KV entries already stored (write index of this token)
  uint32_t token;      // token to process when the feed is exhausted
  uint32_t step;       // steps completed (index into ids)
  uint32_t fed;        // feed entries consumed
  uint32_t n_feed;     // feed length
  uint32_t err;        // kErr* flags raised on the device
  uint32_t pad;
  unsigned long long argmax_key;  // (float_key(max logit) << 32) | ~index
};

// ---- GEMV prologue / epilogue modes ----
enum : int {
  kProPlain = 0,    // x = in[k]
  kProRmsNorm = 1,  // x = in[k] * (1/sqrt(sum(ssq)/n + eps)) * norm_w[k]      (src/tensor.rs:280-290)
  kProAttn = 2,     // x = decode attention output combined from its split partials:
                    //   x[h*hd + d] = sum_s o_s[d] e_s / sum_s l_s e_s, e_s = exp(m_s - max_s m_s)
  kProSwiglu = 3,   // x = silu(in[k]) * in2[k] (gate and up sums of a kEpiRed launch) (src/model.rs:413-417)
};
enum : int {
  kEpiStore = 0,    // y[col] = v
  kEpiResid = 1,    // resid[col] += v ; ssq partial of the new resid       (src/model.rs:401, :423)
  kEpiQkv = 2,      // RoPE(q,k) (src/model.rs:367-368), q -> qbuf, k/v -> KV cache at pos (src/kv_cache.rs:50-54)
  kEpiSwiglu = 3,   // h[n] = silu(gate[n]) * up[n]                         (src/model.rs:413-417)
  kEpiLogits = 4,   // logits[col] = v ; running argmax in SeqState          (src/model.rs:436-452)
  kEpiRed = 5,      // out[col] += v by every contributing CTA (vector red.add, no last arriver):
                    //   red_half = 0: out[out_col + i]; else the chunk's gate half to out[out_col/2 + i]
                    //   and its up half to out[red_half + out_col/2 + i - width/2]
};

struct KvView {
  void *base;            // layer-0 base; layer l at base + l * layer_stride (elements)
  uint64_t layer_stride; // elements per layer
  const uint32_t *page_table;  // [n_seq][max_pages]
  uint32_t max_pages;
  uint32_t n_kv, head_dim;
  int f16;               // 1: __half storage, 0: float
};
// element offset of (page, k/v, kv head, slot, dim) inside one layer
__host__ __device__ inline uint64_t kv_index(uint32_t page, int is_v, uint32_t h, uint32_t slot, uint32_t d,
                                             uint32_t n_kv, uint32_t hd) {
  return ((((uint64_t)page * 2 + (uint64_t)is_v) * n_kv + h) * 16 + slot) * hd + d;
}

// most CTAs contributing to one GEMV chunk (the MMA path's last arriver
// keeps their partial slots in shared memory)
constexpr uint32_t kGemvMaxContrib = 256;

struct GemvParams {
  const uint8_t *w;
  const ChunkDesc *chunks;
  uint32_t n_chunks;
  const CtaRange *ranges;  // [n_ctas]
  const uint32_t *contrib; // per chunk: partial slots of the CTAs with rows in it (ChunkDesc::contrib_off)
  uint32_t n_ctas;
  uint32_t max_chunks_per_cta;
  uint32_t K, K8;
  int mma;                 // 1: MMA tile layout (k_gemv_mma, 16-row groups), 0: 8-row groups (k_gemv)
  uint32_t CW;             // chunk width: 256, 512 or 1024
  uint32_t stage_bytes;    // capacity of one pipeline stage (multiple of 16)
  uint32_t n_stages;       // k_gemv_mma ring depth
  uint32_t max_units;      // k_gemv_mma: most 16-row units of any CTA (x buffer size)
  uint32_t x_slot;         // floats of x (and norm weight) per stage slot
  float *part;             // [n_ctas * max_chunks_per_cta][CW] chunk partials
  uint32_t *counters;      // [n_chunks] arrival counters (zero between launches)
  uint32_t *done;          // optional: +1 per completed chunk (launches that wait on this one)
  // prologue (inputs padded with zeros to K8)
  int pro;
  const float *in;         // [K8]
  const float *norm_w;     // [K8]
  const float *in2;        // kProSwiglu: the up sums
  const float *ssq;        // sum-of-squares partials of `in` (n_ssq = 0: the prologue sums the squares of in)
  uint32_t n_ssq;
  float *zero;             // optional: zeroed by the launch after it waits for the previous one
  uint32_t n_zero;         // floats at `zero` (multiple of 4)
  float eps;
  // epilogue
  int epi;
  float *out;              // store / swiglu / logits / qkv(q part)
  const float *attn_part;  // kProAttn: [K / attn_hd heads][attn_splits][2 + attn_hd] (max, sum, o)
  uint32_t attn_splits, attn_hd;
  float *resid;            // kEpiResid
  float *ssq_out;          // kEpiResid: [n_chunks]
  uint32_t red_half;       // kEpiRed: offset of the up half of a gate/up launch (0: plain columns)
  // qkv
  uint32_t q_dim, kv_dim;
  const float *rope_tab;   // [max_pos][head_dim]: cos,sin pairs
  uint32_t rope_max;       // positions in rope_tab
  KvView kv;
  uint32_t seq, layer;
  SeqState *state;         // pos / argmax
  // failure-path testing (k_gemv_mma): the producer issues no weight copies,
  // so every consumer wait runs out; wait limit in ns (0: kWaitLimitNs)
  uint32_t withhold_weights;
  uint64_t wait_limit_ns;
};

// one-time per-device kernel attributes (dynamic smem)
// launch_gemv dispatches on p.mma
int gemv_init();
int launch_gemv(const GemvParams &p, bool pdl, cudaStream_t st);
size_t gemv_smem_bytes(const GemvParams &p);
int gemv_mma_init();
int launch_gemv_mma(const GemvParams &p, bool pdl, cudaStream_t st);
size_t gemv_mma_smem_bytes(const GemvParams &p);
// ring depth that fits the shared-memory budget of one CTA (0: does not fit)
uint32_t gemv_mma_stages(uint32_t stage_bytes, uint32_t max_units, size_t smem_budget);
// shared-memory offsets of the GEMV layout: the coefficient tables, and the
// ring after the x slice of max_units row groups
uint32_t gemv_mma_table_offset();
uint32_t gemv_mma_table_words();  // 32-bit words of the table area (kProAttn's head weights live there)
uint32_t gemv_mma_ring_offset(uint32_t max_units);
// row groups per pipeline stage for chunks of this type and group size
uint32_t gemv_mma_stage_groups(uint32_t gbytes, int type);

struct AttnParams {
  const float *q;          // [H*hd] (per query row when q_rows > 1)
  const float *kc, *vc;    // contiguous f32 K/V [T][n_kv*hd] (reference KVCache layout); null: paged kv
  uint32_t t_fixed;        // positions when kc/vc are used (0: from state)
  uint32_t q_rows;         // query rows (grid z); rows are independent (no mask)
  KvView kv;
  uint32_t seq, layer;
  uint32_t n_heads, splits;
  float scale;             // 1/sqrt(hd), computed as the reference does
  float *part;             // [H][splits][2 + hd] split partials
  uint32_t *counters;      // [n_kv] arrival counters (zero between launches)
  float *out;              // [H*hd] combined attention output
  SeqState *state;         // T = len + 1
  int partials_only;       // batch-1 paged kernel: leave the split partials for the consumer (kProAttn)
  int early_kv;            // batch-1 paged kernel inside a step graph: K/V tiles of positions below
                           // len are fetched before the wait for the qkv launch (earlier steps,
                           // i.e. earlier graph launches, wrote them)
  const float *qkv_raw;    // batch-1 paged kernel: non-null -> this token's q | k | v are the qkv launch's
                           // red.add sums [H*hd | n_kv*hd | n_kv*hd]: the kernel applies RoPE to q and k
                           // (src/model.rs:367-368), uses the new k / v for position len and appends
                           // them to the cache (src/kv_cache.rs:50-54); q is unused
  const float *rope_tab;   // with qkv_raw: [rope_max][hd] cos, sin pairs
  uint32_t rope_max;
  const SeqState *row_states;  // batched decode: per query row state (T = len + 1), cache sequence row_seq0 + row
  uint32_t row_seq0;
  void *out_h;             // batched decode: non-null -> the combined output as f16 [rows][H*hd] here
                           // instead of out (values beyond the f16 range flag kErrRange in err)
  uint32_t *err;
};
// attention_init: once per device (current), before the first launch_attention
// of a stream capture; launch_attention calls it as well
int attention_init();
int launch_attention(const AttnParams &p, bool pdl, cudaStream_t st);
// batch-1 paged decode attention with bulk-copy tiles (attn_paged.cu); the
// launcher above routes to it when attn_paged_supported holds
bool attn_paged_supported(const AttnParams &p);
int attn_paged_init();
int launch_attn_paged(const AttnParams &p, bool pdl, cudaStream_t st);

struct EmbedParams {
  const uint8_t *emb;      // native [V][d] blocks
  const uint32_t *feed;    // tokens to feed first (state->n_feed of them)
  int type;
  uint32_t d, vocab;
  float *x;                // [d] residual stream
  float *ssq_out;          // [n_ssq] partial sums of squares
  uint32_t n_ssq;          // CTAs
  SeqState *state;
};
int launch_embed(const EmbedParams &p, bool pdl, cudaStream_t st);

// ---- persistent decode step: every phase of one token in one launch ----
enum : uint32_t { kPhEmbed = 0, kPhGemv = 1, kPhAttn = 2 };
struct StepPhase {
  uint32_t kind;       // kPh*
  uint32_t idx;        // GEMV: index into StepParams::gemv; attention: layer
  uint32_t dep;        // phase this one waits for (~0u: none)
  uint32_t dep_count;  // completions of `dep` per step
};
struct StepParams {
  const StepPhase *phases;
  uint32_t n_phases;
  const GemvParams *gemv;   // full launch parameters of every GEMV phase (one ring geometry)
  AttnParams attn;          // attention parameters; layer taken from the phase
  EmbedParams embed;        // n_ssq = the grid size (one partial per CTA)
  uint32_t *done;           // [n_phases] completion counters, monotonic across steps
  uint32_t *sync;           // [0] steps completed, [1] CTAs finished (monotonic)
  uint32_t *ids;            // generated ids (or null)
  uint32_t max_ids;
  uint32_t n_stages, stage_bytes, max_units;  // ring geometry of the GEMV phases
  uint32_t attn_groups;     // attention work groups (4 warps each) per CTA
  uint32_t n_ctas;
};
// bytes of shared memory one attention work group needs, and the launch
int step_attn_group_bytes(uint32_t rep, uint32_t hd);
int step_init();
// returns the cudaError_t of the launch (0: success)
int launch_step(const StepParams &p, size_t smem, cudaStream_t st);
}  // namespace fa
#include <string>
namespace fa {
std::string step_occupancy_report(const StepParams &p, size_t smem);

// step bookkeeping: token <- argmax, ids[step] = token, pos++, len++, step++, fed++
int launch_step_end(SeqState *state, uint32_t *ids, uint32_t max_ids, bool pdl, cudaStream_t st);

// tied output head (no output.weight): logits[j] = dot(xn, E[j]) with E
// native [V][d] (transpose_2d + matmul, src/model.rs:447-452)
// ---- token-parallel dequant-GEMM on tcgen05 (prefill, batched decode) ----
struct QgTile {        // 128-column output tile of one chunk
  uint32_t chunk, col0, ncols, pad;
};
enum : int { kQgStore = 0, kQgResid = 1 };
struct QgParams {
  const uint8_t *w;          // MMA-layout weight buffer of the projection group
  const ChunkDesc *chunks;
  const QgTile *tiles;
  uint32_t n_tiles;
  uint32_t K;                // rows (multiple of 16)
  uint32_t T;                // tokens
  float *out;                // Y[t][out_col] (launch output space), row stride ldo
  uint32_t ldo;
  int epi;                   // kQgStore: Y = X W; kQgResid: Y += X W
  uint32_t *err;             // kErrWaitTimeout on a bounded-wait expiry (may be null)
  float *part;               // stream-K partial tiles: 2 slots per CTA of 128 x BN floats
  uint64_t part_floats;      // capacity of part (>= qgemm_part_floats(bn, n_sm))
  uint32_t prefetch;         // kQ8_0 / kQ4_0: every chunk has that type (weights through the prefetch ring);
                             // kPfAny: any mix of the MMA types through the same ring; 0: direct loads
  uint32_t red;              // 1: the pieces of split tiles are added into out by red.add (out holds zeros for
                             // kQgStore, the residual for kQgResid) and no fixup launch runs; 0: partial slots + fixup
  float *zero;               // optional: cleared by the epilogue warps after the wait for the previous kernel
  uint64_t n_zero;           // floats at `zero` (multiple of 4)
};
constexpr uint32_t kPfAny = 1;  // QgParams::prefetch: mixed-type prefetch ring
struct QgXMap {              // TMA tensor map of an f16 activation buffer X[T_rows][K]
  alignas(64) unsigned char bytes[128];
  uint32_t bn;               // tokens per tile: 64, 128 or 256
};
int qgemm_init();
int qgemm_make_xmap(QgXMap *map, const void *x_f16, uint32_t K, uint32_t T_rows, uint32_t bn);
int launch_qgemm(const QgParams &p, const QgXMap &map, uint32_t n_sm, cudaStream_t st);
// floats of the partial-tile buffer a launch with tiles of bn tokens needs
uint64_t qgemm_part_floats(uint32_t bn, uint32_t n_sm);

// ---- token-parallel forward pieces (prefill.cu) ----
struct AttnRowsParams {
  const void *qh;            // f16 [T][Hq*hd], rotated
  uint32_t T, Hq, Hkv, hd;
  uint32_t len0;             // cache slots before the first token; token t sees [0, len0 + t]
  KvView kv;
  uint32_t seq, layer;
  float scale_log2;          // log2(e) / sqrt(hd)
  void *out;                 // f16 [T][Hq*hd]
};
int launch_embed_rows(const void *emb, int type, const uint32_t *tok, uint32_t T, uint32_t d, uint32_t vocab, float *x,
                      uint32_t *err, cudaStream_t st);
int launch_norm_rows_h(const float *x, const float *w, float eps, uint32_t T, uint32_t d, void *out, uint32_t *err,
                       cudaStream_t st);
int launch_rope_kv_rows(const float *qkv, uint32_t T, uint32_t Hq, uint32_t Hkv, uint32_t hd, const float *rope,
                        uint32_t rope_max, uint32_t pos0, uint32_t len0, const KvView &kv, uint32_t seq, uint32_t layer,
                        void *qh, uint32_t *err, cudaStream_t st);
int launch_attn_rows(const AttnRowsParams &p, cudaStream_t st);
int launch_swiglu_rows(const float *gu, uint32_t T, uint32_t F, uint32_t CW, void *h, uint32_t *err, cudaStream_t st);
int launch_last_row(const float *X, uint32_t row, uint32_t d, float *x, float *ssq, uint32_t n_ssq, cudaStream_t st);
// batched decode: per-row RoPE + KV append (row r = cache sequence seq0 + r at
// states[r].pos / .len, q -> qf f32), f32 -> f16 with the range flag, and the
// per-step bookkeeping (positions + 1, ids -> hist[step][r], step + 1)
int launch_rope_kv_batch(const float *qkv, uint32_t b, uint32_t Hq, uint32_t Hkv, uint32_t hd, const float *rope,
                         uint32_t rope_max, const SeqState *states, const KvView &kv, uint32_t seq0, uint32_t layer,
                         float *qf, uint32_t *err, cudaStream_t st);
// batched decode attention on the tensor cores (mma.sync): grid (splits,
// kv heads, q_rows), row r of AttnParams uses row_states[r] and cache
// sequence row_seq0 + r; p.scale as in launch_attention
int attn_rows_init();
int launch_attn_decode_rows(const AttnParams &p, cudaStream_t st);
int launch_batch_step_end(SeqState *states, uint32_t b, const uint32_t *ids, uint32_t *hist, uint32_t max_steps,
                          uint32_t *step, cudaStream_t st);

// ---- Sampler::sample (src/sampling.rs:110-152), one CTA per sequence ----
constexpr uint32_t kSampleFastK = 2048;  // top-k up to this many candidates stays in shared memory
struct SamplerParams {
  float temperature, top_p, rep, freq_pen, pres_pen;
  uint32_t top_k;
  uint32_t n;                 // logits per row (the vector Sampler::sample receives)
  uint32_t row0;              // first sequence row of the launch (CTA i samples row row0 + i)
  const float *logits;        // row r at logits + (r - row0) * ld
  uint32_t ld;
  uint32_t vocab;             // allocated row length of freq / probs
  uint32_t *freq;             // [n_seq][vocab] token_freq (token_present == freq > 0)
  const uint64_t *seeds;      // [n_seq] Philox4x32-10 keys
  uint64_t *counters;         // [n_seq] samples drawn so far (the Philox counter)
  float *probs;               // [n_seq][vocab] scratch
  unsigned long long *keys;   // [n_seq][pow2] scratch of the full-sort path (null if unused)
  uint32_t pow2;
  uint32_t *ids;              // [n_seq] sampled id per row (may be null)
  // decode-loop hookup (b = 1 generation): sample only steps >= sample_from,
  // then the id becomes the next input token and is observed
  SeqState *state;
  uint32_t *gen_ids, max_ids, sample_from;
  int observe;
};
int sampler_init();
int launch_sample(const SamplerParams &p, uint32_t rows, cudaStream_t st);
int launch_sampler_observe(uint32_t *freq, uint32_t vocab, uint32_t seq, uint32_t token, cudaStream_t st);
// true when a launch with these settings sorts the whole row (needs p.keys)
inline bool sample_needs_sort(const SamplerParams &p) {
  const bool topk = p.top_k > 0 && p.top_k < p.n, topp = p.top_p > 0.0f && p.top_p < 1.0f;
  const bool fast = topk && p.top_k <= kSampleFastK;
  return !fast && (topk || topp);
}

struct TiedHeadParams {
  const uint8_t *emb;
  int type;
  uint32_t d, vocab;
  const float *x;          // residual stream [d] (normalised in-kernel)
  const float *norm_w;
  const float *ssq;
  uint32_t n_ssq;
  float eps;
  float *logits;
  SeqState *state;
};
int launch_tied_head(const TiedHeadParams &p, bool pdl, cudaStream_t st);

// dequantisation / layout
int launch_dequant_native(int type, const void *data, uint64_t count, float *out, cudaStream_t st);
int launch_repack(int type, const void *src_a, const void *src_b, uint32_t K, uint32_t N, uint32_t CW, void *dst,
                  uint64_t dst_off, cudaStream_t st);
// native -> MMA tile layout (K a multiple of 16, CW a multiple of 64)
int launch_repack_mma(int type, const void *src_a, const void *src_b, uint32_t K, uint32_t N, uint32_t CW, void *dst,
                      uint64_t dst_off, cudaStream_t st);
int launch_unpack(int type, const void *src, uint64_t src_off, uint32_t K, uint32_t N, uint32_t CW, float *out,
                  cudaStream_t st);

}  // namespace fa
