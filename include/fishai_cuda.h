/*
 * fishai_cuda.h — C ABI of the B200 (sm_100a) token loop that replaces the
 * CPU forward pass of the fishai-engine crate.
 *
 * Every entry point returns an int status (FA_OK = 0, negative = error) and
 * takes plain pointers and sizes.  Pointers named *_host are host memory
 * owned by the caller; the library owns all device memory it allocates.
 * A handle is not thread-safe: one thread (one stream) per model/kv/sampler.
 * fa_last_error() returns the message of the calling thread's last failure.
 *
 * Each declaration names the reference item (file:line inside the reference
 * crate) whose behaviour it provides.
 */
#ifndef FISHAI_CUDA_H
#define FISHAI_CUDA_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status */
#define FA_OK 0
#define FA_ERR_INVALID (-1)      /* bad argument (reference: panics on misuse) */
#define FA_ERR_GGUF (-2)         /* unreadable / corrupt GGUF (src/gguf.rs:438-561 Err) */
#define FA_ERR_UNSUPPORTED (-3)  /* ggml type or architecture not supported */
#define FA_ERR_OOM (-4)          /* device or host allocation failed */
#define FA_ERR_CUDA (-5)         /* CUDA runtime error */
#define FA_ERR_NCCL (-6)         /* collective error */
#define FA_ERR_CONTEXT (-7)      /* KV cache full: context overflow */
#define FA_ERR_TIMEOUT (-8)      /* a bounded device wait gave up */

/* Copies the calling thread's last error message; returns its full length. */
size_t fa_last_error(char *buf, size_t cap);
/* Library version string. */
const char *fa_version(void);

/* ggml type ids (src/quant.rs:17-29) */
#define FA_GGML_F32 0
#define FA_GGML_F16 1
#define FA_GGML_Q4_0 2
#define FA_GGML_Q4_1 3
#define FA_GGML_Q5_0 6
#define FA_GGML_Q8_0 8
#define FA_GGML_Q4_K 12
#define FA_GGML_Q6_K 14

/* ------------------------------------------------------------------ GGUF */
typedef struct fa_gguf fa_gguf;

/* GGUFFile::open (src/gguf.rs:438-561): mmap, header, metadata, tensor
 * table, data offset aligned to general.alignment (default 32). */
int fa_gguf_open(const char *path, fa_gguf **out);
void fa_gguf_close(fa_gguf *g);
int fa_gguf_version(const fa_gguf *g, uint32_t *version);
int fa_gguf_alignment(const fa_gguf *g, uint64_t *alignment);
int fa_gguf_tensor_count(const fa_gguf *g, size_t *count);
/* tensor_names / tensor_info (src/gguf.rs:623-640): by index */
int fa_gguf_tensor_at(const fa_gguf *g, size_t i, char *name, size_t name_cap, uint32_t *n_dims,
                      uint64_t dims[4], uint32_t *ggml_type, uint64_t *offset);
/* tensor_info by name; FA_ERR_INVALID if absent */
int fa_gguf_tensor_info(const fa_gguf *g, const char *name, uint32_t *n_dims, uint64_t dims[4],
                        uint32_t *ggml_type, uint64_t *offset);
/* read_tensor_data (src/gguf.rs:645-672): byte size by the next-offset rule;
 * copies min(size, cap) bytes when out_host != NULL; *size = 0 when empty */
int fa_gguf_read_tensor_data(const fa_gguf *g, const char *name, void *out_host, size_t cap, size_t *size);
/* metadata_u64 / _i64 / _f32 / _bool / _string (src/gguf.rs:570-614):
 * *found = 0 when the key is absent or has another type */
int fa_gguf_meta_u64(const fa_gguf *g, const char *key, uint64_t *v, int *found);
int fa_gguf_meta_i64(const fa_gguf *g, const char *key, int64_t *v, int *found);
int fa_gguf_meta_f32(const fa_gguf *g, const char *key, float *v, int *found);
int fa_gguf_meta_bool(const fa_gguf *g, const char *key, int *v, int *found);
int fa_gguf_meta_string(const fa_gguf *g, const char *key, char *buf, size_t cap, int *found);
/* vocab_size (src/gguf.rs:748-758) */
int fa_gguf_vocab_size(const fa_gguf *g, uint64_t *v, int *found);

/* -------------------------------------------------------- ModelConfig */
typedef struct {
  uint32_t n_layers, n_heads, n_kv_heads, head_dim, n_embd, vocab_size, context_len;
  float ffn_dim_multiplier, norm_eps, rope_base;
  uint32_t rope_freq_dim;
  uint32_t n_ff;        /* ModelConfig::n_ff() exactly as the reference computes it */
  uint32_t n_ff_used;   /* width of the ffn tensors actually loaded */
  int32_t tied_output;  /* 1 when output.weight is absent (embedding transpose) */
} fa_config;

/* ModelConfig::from_gguf (src/model.rs:92-180) */
int fa_config_from_gguf(const fa_gguf *g, fa_config *cfg);
/* ModelConfig::n_ff (src/model.rs:66-70) */
uint32_t fa_config_n_ff(uint32_t n_embd, float ffn_dim_multiplier);

/* ------------------------------------------------------- dequantisation */
/* quant::dequantize (src/quant.rs:312-338), run on the device: host bytes
 * in, host f32 out.  Supports F32, F16, Q4_0 (high nibble first), Q4_1,
 * Q5_0, Q8_0 and the K-quants Q4_K, Q6_K.  *n_out may be < count when the
 * data is short, as in the reference. */
int fa_dequantize(int ggml_type, const void *bytes_host, size_t nbytes, size_t count, float *out_host,
                  size_t *n_out);
/* same on device buffers, enqueued on `stream` (cudaStream_t or NULL) */
int fa_dequantize_device(int ggml_type, const void *bytes_dev, size_t nbytes, size_t count, float *out_dev,
                         void *stream);

/* ---------------------------------------------------------------- model */
typedef struct fa_model fa_model;
typedef struct {
  int32_t device;       /* CUDA device ordinal */
  int32_t use_graphs;   /* capture the decode step in a CUDA graph (default 1) */
  int32_t use_pdl;      /* programmatic dependent launch between kernels (default 1) */
  int32_t tp_rank, tp_world;  /* tensor parallel rank/world (1 = no TP): rank r keeps query heads
                                 [r*H/W, (r+1)*H/W), their KV heads and FFN columns [r*F/W, ...) of
                                 wq/wk/wv/gate/up, the matching rows of wo/down, and an NCCL all-reduce
                                 completes each o / down projection (src/model.rs:360-420 are the
                                 projections split); embedding, norms and output head replicated */
  const void *nccl_id;  /* 128-byte ncclUniqueId from fa_tp_unique_id on rank 0, when tp_world > 1 */
  int32_t use_step_kernel;  /* run each decode step as one persistent kernel when the
                               model qualifies (MMA-layout projections, untied head) */
  int32_t use_tc_prefill;   /* fa_prefill on the f16 tensor-core path (tcgen05 GEMMs, flash
                               attention): max-abs-rel 1e-2 of the f32 path instead of 1e-4 */
} fa_model_opts;
void fa_model_opts_default(fa_model_opts *o);

/* Tensor parallelism (no reference counterpart: the reference runs on one
 * CPU thread).  fa_tp_unique_id: a fresh 128-byte ncclUniqueId (rank 0 makes
 * it and hands it to every rank's fa_model_load).  Every rank must then make
 * the same sequence of model calls (each forward step runs collectives). */
int fa_tp_unique_id(void *out128);
/* the rank's share of a native weight W[K][N] (GGML blocks along N): axis 0
 * rows [r*K/W, (r+1)*K/W), axis 1 columns [r*N/W, (r+1)*N/W) of every row.
 * A Q4_K column share of 128 columns (half of a 256-column super-block, one
 * KV head at eight-way parallelism) comes back as whole 144-byte blocks whose
 * lower 128 columns hold the share and whose upper 128 dequantise to 0.
 * *out_bytes = shard bytes, *row_bytes = its row stride; out_host NULL only
 * reports sizes.  Host memory only: the load path's own shard step. */
int fa_tp_shard(int32_t ggml_type, const void *bytes_host, uint32_t K, uint32_t N, int32_t axis, uint32_t rank,
                uint32_t world, void *out_host, size_t cap, size_t *out_bytes, uint32_t *row_bytes);

/* GGUFFile::open + ModelConfig::from_gguf + ModelWeights::load_from_gguf
 * (src/model.rs:252-298): weights are uploaded once in their native GGML
 * blocks and re-laid in device memory into the column-chunk layout the
 * kernels stream (same bytes per block, regrouped per 8 rows and 32 columns). */
int fa_model_load(const char *path, const fa_model_opts *opts, fa_model **out);
void fa_model_free(fa_model *m);
int fa_model_config(const fa_model *m, fa_config *cfg);
/* tensor-parallel placement of this model: rank, world and the rank's share
 * of query heads, KV heads (its KV cache holds these) and FFN columns */
int fa_model_tp(const fa_model *m, int32_t *rank, int32_t *world, uint32_t *local_heads, uint32_t *local_kv_heads,
                uint32_t *local_ff);
/* bytes of weights resident on the device, and the algorithmic bytes one
 * decode step streams (all weight tensors + one embedding row) */
int fa_model_weight_bytes(const fa_model *m, uint64_t *device_bytes, uint64_t *step_bytes);
/* the stream the model enqueues on (cudaStream_t) */
void *fa_model_stream(fa_model *m);
/* 1 when decode steps run as the persistent step kernel, else 0 */
int fa_model_step_kernel_active(const fa_model *m);
/* Routes fa_prefill to the f16 tensor-core path (on = 1) or to the f32 token
 * steps (on = 0) from now on; the load option use_tc_prefill sets the
 * initial choice.  FA_ERR_UNSUPPORTED when the model cannot take the
 * tensor-core path.  (No reference counterpart: the reference prefills token
 * by token, src/model.rs:644-650.) */
int fa_model_set_tc_prefill(fa_model *m, int32_t on);
/* Kernel launches in one replay of the captured single-sequence decode step
 * (the CUDA graph behind fa_forward / fa_decode_greedy / fa_generate); 0
 * before the first capture. */
int fa_model_step_launches(const fa_model *m, uint32_t *n);
/* Failure-path testing (no reference counterpart; the reference has no
 * device waits).  FA_DEBUG_WAIT_LIMIT_NS: the bounded waits of the decode
 * GEMV give up after `value` ns instead of 2 s (0 restores the default).
 * FA_DEBUG_WITHHOLD_WEIGHTS: value 1 makes the decode GEMV's producer issue
 * no weight copies, so its consumers' waits run out, the kernel returns and
 * the call reports FA_ERR_TIMEOUT; 0 restores normal operation.  Nothing
 * faults or hangs: every wait is bounded and the context stays usable. */
#define FA_DEBUG_WAIT_LIMIT_NS 1
#define FA_DEBUG_WITHHOLD_WEIGHTS 2
/* FA_DEBUG_FIXED_ORDER_SUMS: value 1 makes the batch-1 o, gate/up and down
 * projections sum their split-K pieces in a fixed order (the last CTA of a
 * chunk adds the published partials), so a step is bit-reproducible run to
 * run; 0 (the default) lets every CTA add its piece into the destination with
 * a vector red.add, which removes a reduction pass per launch but leaves the
 * order of the f32 additions to the hardware. */
#define FA_DEBUG_FIXED_ORDER_SUMS 3
int fa_debug_set(fa_model *m, int32_t key, uint64_t value);

/* ------------------------------------------------------------- KV cache */
typedef struct fa_kv fa_kv;
#define FA_KV_F32 0
#define FA_KV_F16 1
/* KVCache::new (src/kv_cache.rs:27-40), device resident and paged:
 * n_seq sequences, each up to max_ctx positions, pages of 16 positions. */
int fa_kv_create(fa_model *m, uint32_t n_seq, uint32_t max_ctx, int32_t dtype, fa_kv **out);
void fa_kv_free(fa_kv *kv);
/* KVCache::clear (src/kv_cache.rs:98-103); seq < 0 clears every sequence */
int fa_kv_clear(fa_kv *kv, int32_t seq);
/* KVCache::seq_len_with_dim (src/kv_cache.rs:90-96) */
int fa_kv_seq_len(const fa_kv *kv, uint32_t seq, uint32_t *len);
/* KVCache::get (src/kv_cache.rs:66-69): k/v rows [0, len) of one layer as
 * f32 [len][n_kv*head_dim]; FA_ERR_INVALID for a bad layer (the reference panics) */
int fa_kv_get(const fa_kv *kv, uint32_t seq, uint32_t layer, float *k_host, float *v_host);

/* -------------------------------------------------------------- forward */
/* ModelWeights::forward (src/model.rs:316-455), reference semantics: all n
 * tokens at position `pos`, no causal mask, KV appended for every token.
 * logits_host: n*vocab floats or NULL; argmax_host: n ids or NULL (first
 * index of the maximum logit); hidden_host: n_layers*n*n_embd residual
 * values after each layer, or NULL. */
int fa_forward(fa_model *m, fa_kv *kv, uint32_t seq, const uint32_t *tokens_host, uint32_t n, uint32_t pos,
               float *logits_host, uint32_t *argmax_host, float *hidden_host);
/* Causal prefill: token t at position start_pos+t attends to positions
 * [0, start_pos+t].  Equal to n single-token fa_forward calls.
 * last_logits_host: vocab floats of the last token or NULL. */
int fa_prefill(fa_model *m, fa_kv *kv, uint32_t seq, const uint32_t *tokens_host, uint32_t n, uint32_t start_pos,
               float *last_logits_host, uint32_t *last_argmax_host);

/* ------------------------------------------------------------ attention */
/* tensor::scaled_dot_product_attention (src/tensor.rs:451-551) with the GQA
 * head expansion of src/model.rs:500-526 folded in, on device buffers:
 * q [q_len][n_heads*head_dim], k/v [kv_len][n_kv_heads*head_dim] f32 (the
 * full K/V, cache rows first: the reference's full_k/full_v), out
 * [q_len][n_heads*head_dim].  Every query row attends to all kv_len rows (no
 * mask), scores scaled by 1/sqrt(head_dim).  Split-K over positions with a
 * deterministic combine; scratch comes from a per-device buffer the library
 * allocates on first use and grows as needed (calls must not overlap).
 * head_dim <= 128; n_heads / n_kv_heads in {1, 2, 4, 8}. */
int fa_sdpa(const float *q_dev, const float *k_dev, const float *v_dev, uint32_t q_len, uint32_t kv_len,
            uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, float *out_dev, void *stream);
/* the same on host buffers (tensor::scaled_dot_product_attention's own
 * calling convention: slices in, a vector out); device buffers are
 * allocated, filled, and freed inside the call */
int fa_sdpa_host(const float *q_host, const float *k_host, const float *v_host, uint32_t q_len, uint32_t kv_len,
                 uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, float *out_host);

/* No counterpart in the reference.  fa_sdpa without any device allocation,
 * for callers that must not call cudaMalloc: code whose device memory is
 * handed out by its own allocator or pool (a cudaMalloc there would go around
 * that budget), and code on a latency-critical path where an implicit
 * allocation and the device-wide synchronisation that may come with it are
 * not allowed.  Same arguments, numbers and limits as fa_sdpa; the caller
 * passes every input and output buffer.  The split-K scratch is a fixed
 * static device array inside the library (2 MiB + 4 KiB, held on every GPU
 * that loads the library until the process exits), so
 *   q_len * n_heads * 32 * (head_dim + 2) <= 524288 and
 *   q_len * n_kv_heads <= 1024,
 * else FA_ERR_INVALID (e.g. head_dim 128 allows q_len * n_heads <= 126).
 * The first call on each device looks up the array's device address with
 * that device current; make that first call before any stream capture.  The
 * address is kept for the life of the process: after cudaDeviceReset (or
 * anything else that destroys and re-creates the device's primary context)
 * it is stale, so do not call this entry point on that device again.
 * Every call on a device shares the one array: calls that overlap on the GPU
 * (different streams, no ordering between them) race and give wrong output.
 * The counters it needs at zero are cleared on `stream` by every call. */
int fa_sdpa_noalloc(const float *q_dev, const float *k_dev, const float *v_dev, uint32_t q_len, uint32_t kv_len,
                    uint32_t n_heads, uint32_t n_kv_heads, uint32_t head_dim, float *out_dev, void *stream);

/* ------------------------------------------------------------ tokenizer */
/* BpeTokenizer (src/tokenizer.rs:148-600): the text step before the token
 * loop.  Ids -1 mean "none" (the reference's Option<u32>). */
typedef struct {
  int64_t bos_token_id, eos_token_id, eot_token_id, eom_token_id, unk_token_id;
  int32_t add_bos, add_eos, add_space_prefix, remove_special_whitespaces, prepend_bos;
} fa_tokenizer_config;
typedef struct fa_tokenizer fa_tokenizer;
/* TokenizerConfig::default (src/tokenizer.rs:130-144) */
void fa_tokenizer_config_default(fa_tokenizer_config *cfg);
/* BpeTokenizer::from_gguf (src/tokenizer.rs:202-286): token texts (UTF-8),
 * scores and token types (shorter arrays leave the rest at 0 / Normal),
 * merges as "left right" lines (rank = line index) or NULL, cfg or NULL for
 * the default. */
int fa_tokenizer_create(const char *const *texts, uint32_t n_tokens, const float *scores, uint32_t n_scores,
                        const int32_t *types, uint32_t n_types, const char *merges, const fa_tokenizer_config *cfg,
                        fa_tokenizer **out);
/* the tokenizer a GGUF file carries: tokenizer.ggml.tokens / scores /
 * token_type / merges and the config keys of parse_tokenizer_config_from_gguf
 * (src/tokenizer.rs:520-553); FA_ERR_GGUF when the file has no token list */
int fa_tokenizer_from_gguf(const fa_gguf *g, fa_tokenizer **out);
void fa_tokenizer_free(fa_tokenizer *t);
/* encode (src/tokenizer.rs:290-344) or, with with_special = 1,
 * encode_with_special (src/tokenizer.rs:347-391); *n = ids produced (ids
 * receives min(n, cap) of them) */
int fa_tokenizer_encode(const fa_tokenizer *t, const char *text_utf8, size_t len, int32_t add_special,
                        int32_t with_special, uint32_t *ids, size_t cap, size_t *n);
/* decode (src/tokenizer.rs:394-408): *len = UTF-8 bytes (buf gets a NUL-
 * terminated prefix of at most cap - 1) */
int fa_tokenizer_decode(const fa_tokenizer *t, const uint32_t *ids, size_t n, char *buf, size_t cap, size_t *len);
/* vocab_size / bos_token / eos_token (src/tokenizer.rs:420-433) and the config */
int fa_tokenizer_info(const fa_tokenizer *t, uint32_t *vocab_size, fa_tokenizer_config *cfg);
/* token_to_piece (src/tokenizer.rs:411-418) and the token's type; id out of range: FA_ERR_INVALID */
int fa_tokenizer_piece(const fa_tokenizer *t, uint32_t id, char *buf, size_t cap, size_t *len, int32_t *type);
/* the byte-fallback token of a byte value (bytes_to_tokens, src/tokenizer.rs:441-447) */
int fa_tokenizer_byte_token(const fa_tokenizer *t, uint32_t byte_value, uint32_t *id);

/* ------------------------------------------------------------- sampling */
typedef struct {
  float temperature;            /* 0 = greedy */
  uint32_t top_k;               /* 0 = off */
  float top_p;                  /* 0 < p < 1 enables the reference's fixed-0.999 nucleus cut */
  float repetition_penalty;     /* 1 = off */
  float frequency_penalty, presence_penalty;
} fa_sampler_config;
typedef struct fa_sampler fa_sampler;
/* Sampler::new (src/sampling.rs:95-104): n_seq independent samplers,
 * sequence i draws its categorical uniforms from Philox4x32-10 keyed by
 * seeds_host[i] (counter = its sample index). */
int fa_sampler_create(const fa_sampler_config *cfg, uint32_t n_seq, uint32_t vocab, const uint64_t *seeds_host,
                      fa_sampler **out);
void fa_sampler_free(fa_sampler *s);
/* Sampler::sample (src/sampling.rs:110-152) on device logits [n_seq][vocab]
 * (or the first n rows); ids written to ids_dev (device) and, if non-NULL,
 * ids_host. */
int fa_sample_device(fa_sampler *s, const float *logits_dev, uint32_t n, uint32_t *ids_dev, uint32_t *ids_host,
                     void *stream);
/* Sampler::sample on host logits (copies in and out; the /api/sample path) */
int fa_sample(fa_sampler *s, uint32_t seq, const float *logits_host, uint32_t vocab, uint32_t *id_host);
/* Sampler::observe_token / reset (src/sampling.rs:155-165) */
int fa_sampler_observe(fa_sampler *s, uint32_t seq, uint32_t token);
int fa_sampler_reset(fa_sampler *s, int32_t seq);  /* seq < 0: every sequence */
/* token_freq[token] of sequence seq (0 for ids never observed) */
int fa_sampler_freq(fa_sampler *s, uint32_t seq, uint32_t token, uint32_t *count);

/* ------------------------------------------------ token-parallel GEMM */
/* Y[T][n_out] = X[T][K] . W for one weight group of the model (proj 0 qkv,
 * 1 o, 2 gate/up interleaved per 1024-column chunk, 3 down, 4 output head)
 * on the tcgen05 path that prefill and batched decode use: X rounded to f16,
 * W dequantised to f16 (d*sc*q - dmin*m in f32, rounded once), f32
 * accumulation.  Host buffers; y_host NULL only reports n_out. */
int fa_gemm_tokens(fa_model *m, int32_t proj, uint32_t layer, const float *x_host, uint32_t T, float *y_host,
                   uint32_t *n_out);

/* device time (ms, average of reps launches) of that GEMM for T tokens on
 * device-resident operands, and its flop count 2*T*K*n_out */
int fa_profile_gemm(fa_model *m, int32_t proj, uint32_t layer, uint32_t T, uint32_t reps, float *avg_ms,
                    double *flop);

/* Batched decode: sequences 0..b-1 of kv advance `steps` tokens together.
 * Row r starts from tokens[r] at RoPE position pos[r], appended after its
 * cached positions; every step forwards all rows (f16 tensor-core GEMMs at
 * T = b, attention per row over its own cache), samples row r with sampler
 * row r (Sampler::sample, then observe_token) and feeds the id back.
 * ids_out [steps][b]; logits_out (NULL or [steps][b][vocab]) also returns
 * every step's logits.  Only ids cross PCIe when logits_out is NULL. */
int fa_decode_batch(fa_model *m, fa_kv *kv, uint32_t b, const uint32_t *tokens, const uint32_t *pos, fa_sampler *s,
                    uint32_t steps, uint32_t *ids_out, float *logits_out);

/* ----------------------------------------------------------- generation */
typedef struct {
  uint32_t max_tokens;          /* includes the prompt, as in src/model.rs:683-686 */
  fa_sampler_config sampler;
  const uint32_t *stop_ids; uint32_t n_stop;
  uint64_t seed;
  int32_t kv_dtype;             /* FA_KV_F32 (reference values) or FA_KV_F16 */
} fa_gen_config;

/* GenerationState::generate (src/model.rs:638-674): prefill, re-feed the
 * last prompt token, then decode until max_tokens (prompt included) or a
 * stop id.  Only token ids cross PCIe.  *n_out = generated ids. */
int fa_generate(fa_model *m, const fa_gen_config *cfg, const uint32_t *prompt_host, uint32_t n_prompt,
                uint32_t *out_host, uint32_t cap, uint32_t *n_out);

/* Decode driver for benchmarks and the bench harness: after a prefill of
 * `seq` in `kv`, run `steps` greedy decode steps starting from token
 * `first_token` at position `pos` entirely on the device (CUDA graph per
 * step), writing the ids to ids_host.  Used to time steady-state decode. */
int fa_decode_greedy(fa_model *m, fa_kv *kv, uint32_t seq, uint32_t first_token, uint32_t pos, uint32_t steps,
                     uint32_t *ids_host);

/* Kernel timing for the roofline report: launches the decode GEMV of one
 * kind (0 qkv, 1 attn_output, 2 ffn gate+up, 3 ffn_down, 4 output head)
 * `reps` times, cycling through the layers so the weights stream from HBM
 * (every layer's weights together exceed L2), and returns the average
 * device time per launch (CUDA events on the model stream) and the
 * algorithmic bytes one launch streams (native GGML block bytes). */
int fa_profile_gemv(fa_model *m, int32_t kind, uint32_t reps, float *avg_ms, uint64_t *bytes_per_launch);

/* ------------------------------------------------------ synthetic GGUF */
typedef struct {
  uint32_t n_layers, n_embd, n_heads, n_kv_heads, n_ff, vocab, context_len;
  float rope_base, norm_eps, sigma;
  int32_t type_embd, type_q, type_k, type_v, type_o, type_gate, type_up, type_down;
  int32_t type_out;             /* -1: no output.weight (tied embedding head) */
  uint32_t threads;             /* 0 = all cores */
} fa_synth_spec;
/* Writes a llama-architecture GGUF v3 with weights N(0, sigma) drawn from
 * Philox4x32-10 (key = seed, tensor index) + Box-Muller, quantised by the
 * reference's own Q8_0/Q4_0 rules (src/quant.rs:393-471) or this library's
 * Q4_K/Q6_K encoders; norms are 1.0 in F32.  Metadata keys use the types
 * the reference reads (feed_forward_length as FLOAT32). */
int fa_synth_write(const char *path, const fa_synth_spec *spec, uint64_t seed);

#ifdef __cplusplus
}
#endif
#endif
