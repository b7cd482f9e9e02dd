/*
 * ORACLE — test infrastructure only.
 *
 * CPU restatement of the fishai-engine reference CPU path (a Rust crate that
 * cannot be compiled in this image: no cargo/rustc).  Only tests/, the
 * __graft_entry__ smoke check and bench.py's CPU-baseline leg may load this
 * library, and only as the test oracle or as the timed CPU baseline; the product
 * (fishai-engine_b200/) never links or calls it.
 *
 * Every function cites the reference file:line whose behaviour it restates.
 * Bit-faithfulness recipe: sums run sequentially in the reference's order,
 * the library is compiled with -ffp-contract=off (Rust never fuses a*b+c),
 * expf/powf/sinf/cosf/sqrtf come from glibc (what Rust's f32 methods call on
 * Linux), f16->f32 is exact and f32->f16 rounds to nearest even (half crate).
 *
 * Deviations from the reference (each labelled where it happens):
 *  D1 Q4_K / Q6_K dequantisation (reference returns Err, src/quant.rs:333-337):
 *     restated from the public GGUF block format and cross-checked against
 *     gguf-py 0.19.0 in tests.  Parity for these types is unpinned by the
 *     reference's own tests.
 *  D2 n_ff: the reference computes roundup256(n_embd*mult) (src/model.rs:66-70)
 *     which for a 1408-wide FFN gives 1536 and panics in matmul
 *     (src/tensor.rs:246).  The oracle uses the ffn_gate tensor's own width
 *     whenever it disagrees with n_ff(), and reports that it did.
 *  D3 weights may stay quantised and be dequantised per use (values are
 *     identical to dequantise-at-load, src/model.rs:252-298).
 *  D4 categorical sampling draws its uniform from Philox4x32-10 keyed by a
 *     seed and a step counter instead of the unseeded rand::rng()
 *     (src/sampling.rs:283-294); the subtraction rule is unchanged.
 */
#ifndef FA_ORACLE_H
#define FA_ORACLE_H
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ggml type ids, src/quant.rs:17-29 */
enum {
  OR_F32 = 0, OR_F16 = 1, OR_Q4_0 = 2, OR_Q4_1 = 3, OR_Q5_0 = 6, OR_Q5_1 = 7,
  OR_Q8_0 = 8, OR_Q8_1 = 9, OR_Q2_K = 10, OR_Q3_K = 11, OR_Q4_K = 12,
  OR_Q5_K = 13, OR_Q6_K = 14
};

float or_f16_to_f32(uint16_t h);
uint16_t or_f32_to_f16(float f);

size_t or_block_size(int ggml_type);   /* src/quant.rs:345-361 */
size_t or_type_size(int ggml_type);    /* src/quant.rs:364-382 */

/* quant::dequantize (src/quant.rs:312-338) plus D1.  Returns the number of
 * values written (may be < count when data is short, as in the reference),
 * or -1 for an unsupported type, -2 for short F32 data. */
long or_dequantize(const uint8_t *data, size_t nbytes, int ggml_type, size_t count, float *out);

/* the reference's own test quantisers, src/quant.rs:393-471 */
size_t or_quantize_q4_0(const float *v, size_t n, uint8_t *out);
size_t or_quantize_q8_0(const float *v, size_t n, uint8_t *out);

/* tensor math, src/tensor.rs */
void or_matmul(const float *a, const float *b, size_t m, size_t k, size_t n, float *c);
void or_rms_norm(const float *x, const float *w, size_t n, float eps, float *y);
void or_silu(const float *x, size_t n, float *y);
void or_softmax_inplace(float *x, size_t n);
void or_rope_emb(size_t pos, size_t dim, float base, float *emb);
void or_apply_rope_to_tensor(float *data, size_t len, size_t n_h, size_t head_dim, size_t pos, float base);
void or_sdpa(const float *q, const float *k, const float *v, size_t q_len, size_t kv_len,
             size_t n_heads, size_t head_dim, float *out);

/* Philox4x32-10 (Salmon et al., SC'11) */
void or_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]);
float or_philox_uniform(uint64_t seed, uint64_t step);

/* ---- GGUF (src/gguf.rs:438-689) ---- */
typedef struct or_gguf or_gguf;
or_gguf *or_gguf_open(const char *path, char *err, size_t errlen);
void or_gguf_close(or_gguf *g);
uint32_t or_gguf_version(const or_gguf *g);
uint64_t or_gguf_alignment(const or_gguf *g);
size_t or_gguf_tensor_count(const or_gguf *g);
const char *or_gguf_tensor_name(const or_gguf *g, size_t i);
/* returns 0 if found */
int or_gguf_tensor_info(const or_gguf *g, const char *name, uint32_t *n_dims, uint64_t dims[4],
                        uint32_t *ggml_type, uint64_t *offset);
/* read_tensor_data: copies into out (if non-NULL) and returns the byte size (0 = empty) */
size_t or_gguf_read_tensor_data(const or_gguf *g, const char *name, uint8_t *out, size_t cap);
/* metadata accessors: return 1 if present with a matching type */
int or_gguf_meta_u64(const or_gguf *g, const char *key, uint64_t *v);
int or_gguf_meta_i64(const or_gguf *g, const char *key, int64_t *v);
int or_gguf_meta_f32(const or_gguf *g, const char *key, float *v);
int or_gguf_meta_bool(const or_gguf *g, const char *key, int *v);
int or_gguf_meta_string(const or_gguf *g, const char *key, char *buf, size_t cap);
int or_gguf_vocab_size(const or_gguf *g, uint64_t *v);

/* ---- model (src/model.rs) ---- */
typedef struct {
  size_t n_layers, n_heads, n_kv_heads, head_dim, n_embd, vocab_size, context_len;
  float ffn_dim_multiplier, norm_eps, rope_base;
  size_t rope_freq_dim;
  size_t n_ff;          /* ModelConfig::n_ff() as the reference computes it */
  size_t n_ff_used;     /* width actually used (D2) */
  int n_ff_deviation;   /* 1 when n_ff_used != n_ff */
  int tied_output;      /* 1 when output.weight is absent */
} or_config;

int or_config_from_gguf(const or_gguf *g, or_config *cfg, char *err, size_t errlen);
size_t or_config_n_ff(size_t n_embd, float mult);

typedef struct or_model or_model;
/* resident: 1 = dequantise every tensor to f32 at load (the reference's
 * behaviour), 0 = keep native blocks and dequantise per use (D3). */
or_model *or_model_load(const char *path, int resident, char *err, size_t errlen);
void or_model_free(or_model *m);
void or_model_config(const or_model *m, or_config *cfg);
void or_model_set_threads(or_model *m, int threads);

typedef struct or_kv or_kv;
/* kv_f16: round stored K/V to f16 (models the device's f16 cache; not a
 * reference behaviour - the reference stores f32, src/kv_cache.rs:13-54) */
or_kv *or_kv_new(const or_model *m, size_t max_ctx, int kv_f16);
void or_kv_free(or_kv *kv);
void or_kv_clear(or_kv *kv);
size_t or_kv_len(const or_kv *kv);
/* copies layer `layer` K and V rows [0, len) into k/v (len*n_kv*hd floats) */
int or_kv_get(const or_kv *kv, size_t layer, float *k, float *v);
/* test helper: layer `layer` rows [0, len) from k/v; the cache length
 * becomes len (set every layer before a forward) */
int or_kv_set(or_kv *kv, size_t layer, const float *k, const float *v, size_t len);

/* ModelWeights::forward (src/model.rs:316-455): reference semantics, every
 * token of the batch at the same position, no mask.  logits: n*V floats.
 * hidden (optional): n_layers*n*d residual-stream values after each layer.
 * algo: 0 = reference i-j-p matmul, 1 = fast mode (same sums, reordered loops) */
int or_forward(or_model *m, const uint32_t *tokens, size_t n, size_t pos, or_kv *kv,
               float *logits, float *hidden, int algo);
/* Causal batch: token t at position pos0+t attends to cache[0..pos0+t].
 * Bit-identical to n sequential single-token or_forward calls.  Logits of
 * the last token only (if logits != NULL); hidden as above for all tokens. */
int or_prefill(or_model *m, const uint32_t *tokens, size_t n, size_t pos0, or_kv *kv,
               float *last_logits, float *hidden);

/* CPU-baseline sample: seconds for one token's matmuls of one layer in the
 * reference's i-j-p order; *macs receives the multiply-add count */
double or_time_layer(or_model *m, size_t layer, double *macs);
/* CPU baseline: one decode token in the reference's order and data movement
 * (all matmuls i-j-p, RoPE, expand_kv_heads, attention, output head, greedy
 * pick), one thread, weights dequantised outside the timed region; the first
 * n_layers_timed layers (0: all).  out[0] / out[1]: seconds in the layers /
 * in the head and pick.  Returns the picked id or -1 (cache full, bad id). */
long or_time_token(or_model *m, or_kv *kv, uint32_t token, size_t pos, size_t n_layers_timed, double out[2]);
/* timing only: rows [0, len) of every layer's K/V set to deterministic
 * pseudo-random values in [-0.5, 0.5), len = the cache length afterwards */
void or_kv_fill_synthetic(or_kv *kv, size_t len, uint64_t seed);

/* ---- sampler (src/sampling.rs:14-310) ---- */
typedef struct {
  float temperature; size_t top_k; float top_p;
  float repetition_penalty, frequency_penalty, presence_penalty;
} or_sampler_cfg;
typedef struct or_sampler or_sampler;
or_sampler *or_sampler_new(const or_sampler_cfg *cfg);
void or_sampler_free(or_sampler *s);
/* r: the uniform draw used only when the pipeline reaches categorical_sample */
size_t or_sampler_sample(or_sampler *s, const float *logits, size_t n, float r, int *used_r);
void or_sampler_observe(or_sampler *s, size_t token);
void or_sampler_reset(or_sampler *s);
size_t or_sampler_freq(const or_sampler *s, size_t token);
/* free helpers exposed for the reference's own unit tests */
void or_softmax_probs(const float *logits, size_t n, float *out);   /* src/sampling.rs:222-231 */
void or_top_k_filter(const float *probs, size_t n, size_t k, float *out);
void or_top_p_filter(float *probs, size_t n);
size_t or_categorical_sample(const float *probs, size_t n, float r);
size_t or_argmax(const float *v, size_t n);

/* ---- generation (src/model.rs:546-716) ---- */
typedef struct {
  size_t max_tokens; float temperature; size_t top_k; float top_p; float repetition_penalty;
  const uint32_t *stop_ids; size_t n_stop;
  uint64_t seed;        /* Philox seed for categorical draws (D4) */
  int fast;             /* 1: prompt through or_prefill, steps through fast matmul */
} or_gen_cfg;
/* Returns the number of generated ids written to out (<= cap), -1 on error. */
long or_generate(or_model *m, const or_gen_cfg *cfg, const uint32_t *prompt, size_t n_prompt,
                 uint32_t *out, size_t cap, int kv_f16);

#ifdef __cplusplus
}
#endif
#endif
