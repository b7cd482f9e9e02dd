/*
 * ORACLE — test infrastructure only (see fa_oracle.h for the contract and the
 * list of deviations D1-D4).  CPU restatement of the fishai-engine reference
 * path: src/quant.rs, src/tensor.rs, src/gguf.rs, src/kv_cache.rs,
 * src/model.rs and src/sampling.rs.  Build: oracle/Makefile
 * (-O2 -ffp-contract=off, glibc libm).
 */
#define _GNU_SOURCE
#include "fa_oracle.h"

#include <fcntl.h>
#include <math.h>
#include <pthread.h>
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

static void set_err(char *err, size_t errlen, const char *fmt, ...) {
  if (!err || !errlen) return;
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(err, errlen, fmt, ap);
  va_end(ap);
}

/* ------------------------------------------------------------------------ */
/* f16 <-> f32 (half crate semantics: exact widening, RNE narrowing)         */
/* ------------------------------------------------------------------------ */
float or_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1Fu;
  uint32_t man = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else { /* subnormal: normalise */
      int e = -1;
      do { man <<= 1; ++e; } while (!(man & 0x400u));
      man &= 0x3FFu;
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t or_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t exp = (x >> 23) & 0xFFu;
  uint32_t man = x & 0x7FFFFFu;
  if (exp == 0xFF) { /* inf / nan (keep a quiet payload bit for nan) */
    return (uint16_t)(sign | 0x7C00u | (man ? (0x200u | (man >> 13)) : 0));
  }
  int e = (int)exp - 127 + 15;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) { /* subnormal or zero in f16 */
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    int shift = 14 - e; /* 24-bit significand -> 10-bit subnormal field */
    uint32_t half_man = man >> shift;
    uint32_t rem = man & ((1u << shift) - 1);
    uint32_t halfway = 1u << (shift - 1);
    if (rem > halfway || (rem == halfway && (half_man & 1u))) half_man++;
    return (uint16_t)(sign | half_man);
  }
  uint32_t half_man = man >> 13;
  uint32_t rem = man & 0x1FFFu;
  uint32_t out = sign | ((uint32_t)e << 10) | half_man;
  if (rem > 0x1000u || (rem == 0x1000u && (half_man & 1u))) out++; /* carries into exp ok */
  return (uint16_t)out;
}

static inline float ld_f16(const uint8_t *p) { return or_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

/* ------------------------------------------------------------------------ */
/* block / type sizes, src/quant.rs:345-382                                  */
/* ------------------------------------------------------------------------ */
size_t or_block_size(int t) {
  switch (t) {
    case OR_F32: case OR_F16: return 1;
    case OR_Q4_0: case OR_Q4_1: case OR_Q5_0: case OR_Q5_1: case OR_Q8_0: case OR_Q8_1: return 32;
    case OR_Q2_K: case OR_Q3_K: case OR_Q4_K: case OR_Q5_K: case OR_Q6_K: return 256;
    default: return 1;
  }
}

size_t or_type_size(int t) {
  switch (t) {
    case OR_F32: return 4; case OR_F16: return 2; case OR_Q4_0: return 18; case OR_Q4_1: return 20;
    case OR_Q5_0: return 22; case OR_Q5_1: return 24; case OR_Q8_0: return 34; case OR_Q8_1: return 40;
    case OR_Q2_K: return 84; case OR_Q3_K: return 110; case OR_Q4_K: return 144; case OR_Q5_K: return 176;
    case OR_Q6_K: return 210; default: return 4;
  }
}

/* ------------------------------------------------------------------------ */
/* dequantisation, src/quant.rs:123-338 (+ D1 for Q4_K/Q6_K)                 */
/* ------------------------------------------------------------------------ */
/* Q4_0: src/quant.rs:123-157.  Element 2j is the HIGH nibble of byte j. */
static size_t dq_q4_0(const uint8_t *data, size_t nbytes, size_t count, float *out) {
  size_t n = 0, nb = (count + 31) / 32, off = 0;
  for (size_t b = 0; b < nb; ++b) {
    if (off + 18 > nbytes) break;
    float d = ld_f16(data + off);
    off += 2;
    for (int i = 0; i < 32; ++i) {
      if (n >= count) break;
      uint8_t byte = data[off + i / 2];
      int nib = (i % 2 == 0) ? (byte >> 4) : (byte & 0x0F);
      out[n++] = (float)(nib - 8) * d;
    }
    off += 16;
  }
  return n;
}

/* Q4_1: src/quant.rs:163-200 */
static size_t dq_q4_1(const uint8_t *data, size_t nbytes, size_t count, float *out) {
  size_t n = 0, nb = (count + 31) / 32, off = 0;
  for (size_t b = 0; b < nb; ++b) {
    if (off + 20 > nbytes) break;
    float d = ld_f16(data + off);
    float m = ld_f16(data + off + 2);
    off += 4;
    for (int i = 0; i < 32; ++i) {
      if (n >= count) break;
      uint8_t byte = data[off + i / 2];
      int nib = (i % 2 == 0) ? (byte >> 4) : (byte & 0x0F);
      float prod = (float)nib * d;
      out[n++] = prod + m;
    }
    off += 16;
  }
  return n;
}

/* Q5_0: src/quant.rs:206-255 */
static size_t dq_q5_0(const uint8_t *data, size_t nbytes, size_t count, float *out) {
  size_t n = 0, nb = (count + 31) / 32, off = 0;
  for (size_t b = 0; b < nb; ++b) {
    if (off + 22 > nbytes) break;
    float d = ld_f16(data + off);
    off += 2;
    uint32_t qh = (uint32_t)data[off] | ((uint32_t)data[off + 1] << 8) |
                  ((uint32_t)data[off + 2] << 16) | ((uint32_t)data[off + 3] << 24);
    off += 4;
    for (int i = 0; i < 32; ++i) {
      if (n >= count) break;
      uint8_t byte = data[off + i / 2];
      uint32_t lo = (i % 2 == 0) ? (byte >> 4) : (byte & 0x0F);
      uint32_t hb = (qh >> i) & 1u;
      int v = (int)(lo | (hb << 4)) - 16;
      out[n++] = (float)v * d;
    }
    off += 16;
  }
  return n;
}

/* Q8_0: src/quant.rs:261-290 */
static size_t dq_q8_0(const uint8_t *data, size_t nbytes, size_t count, float *out) {
  size_t n = 0, nb = (count + 31) / 32, off = 0;
  for (size_t b = 0; b < nb; ++b) {
    if (off + 34 > nbytes) break;
    float d = ld_f16(data + off);
    off += 2;
    for (int i = 0; i < 32; ++i) {
      if (n >= count) break;
      out[n++] = (float)(int8_t)data[off + i] * d;
    }
    off += 32;
  }
  return n;
}

/* F16: src/quant.rs:295-307 */
static size_t dq_f16(const uint8_t *data, size_t nbytes, size_t count, float *out) {
  size_t n = 0;
  for (; n < count && 2 * n + 2 <= nbytes; ++n) out[n] = ld_f16(data + 2 * n);
  return n;
}

/* D1: Q4_K per the public GGUF block layout (d, dmin, 12 B packed 6-bit
 * scales/mins, 128 B of 4-bit codes; sub-block 2j = low nibbles of
 * qs[32j..32j+32), 2j+1 = high nibbles).  value = (d*sc)*q - dmin*m. */
static void q4k_scale_min(int j, const uint8_t *q, int *sc, int *m) {
  if (j < 4) {
    *sc = q[j] & 63;
    *m = q[j + 4] & 63;
  } else {
    *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
    *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

static size_t dq_q4_k(const uint8_t *data, size_t nbytes, size_t count, float *out) {
  size_t n = 0, nb = (count + 255) / 256, off = 0;
  for (size_t b = 0; b < nb; ++b) {
    if (off + 144 > nbytes) break;
    const uint8_t *blk = data + off;
    float d = ld_f16(blk), dmin = ld_f16(blk + 2);
    const uint8_t *scales = blk + 4, *qs = blk + 16;
    for (int j = 0; j < 4; ++j) {
      int sc, m;
      q4k_scale_min(2 * j, scales, &sc, &m);
      float d1 = d * (float)sc, m1 = dmin * (float)m;
      q4k_scale_min(2 * j + 1, scales, &sc, &m);
      float d2 = d * (float)sc, m2 = dmin * (float)m;
      for (int l = 0; l < 32 && n < count; ++l) { float p = d1 * (float)(qs[32 * j + l] & 0xF); out[n++] = p - m1; }
      for (int l = 0; l < 32 && n < count; ++l) { float p = d2 * (float)(qs[32 * j + l] >> 4); out[n++] = p - m2; }
    }
    off += 144;
  }
  return n;
}

/* D1: Q6_K (ql[128], qh[64], int8 scales[16], f16 d).  value = (d*sc)*(q-32). */
static size_t dq_q6_k(const uint8_t *data, size_t nbytes, size_t count, float *out) {
  size_t n = 0, nb = (count + 255) / 256, off = 0;
  float y[256];
  for (size_t b = 0; b < nb; ++b) {
    if (off + 210 > nbytes) break;
    const uint8_t *blk = data + off;
    const uint8_t *ql = blk, *qh = blk + 128;
    const int8_t *sc = (const int8_t *)(blk + 192);
    float d = ld_f16(blk + 208);
    for (int h = 0; h < 2; ++h) {
      const uint8_t *L = ql + 64 * h, *H = qh + 32 * h;
      const int8_t *S = sc + 8 * h;
      float *Y = y + 128 * h;
      for (int l = 0; l < 32; ++l) {
        int is = l / 16;
        int q1 = (int)((L[l] & 0xF) | (((H[l] >> 0) & 3) << 4)) - 32;
        int q2 = (int)((L[l + 32] & 0xF) | (((H[l] >> 2) & 3) << 4)) - 32;
        int q3 = (int)((L[l] >> 4) | (((H[l] >> 4) & 3) << 4)) - 32;
        int q4 = (int)((L[l + 32] >> 4) | (((H[l] >> 6) & 3) << 4)) - 32;
        float s1 = d * (float)S[is + 0], s2 = d * (float)S[is + 2];
        float s3 = d * (float)S[is + 4], s4 = d * (float)S[is + 6];
        Y[l] = s1 * (float)q1;
        Y[l + 32] = s2 * (float)q2;
        Y[l + 64] = s3 * (float)q3;
        Y[l + 96] = s4 * (float)q4;
      }
    }
    for (int i = 0; i < 256 && n < count; ++i) out[n++] = y[i];
    off += 210;
  }
  return n;
}

/* dispatcher, src/quant.rs:312-338 */
long or_dequantize(const uint8_t *data, size_t nbytes, int t, size_t count, float *out) {
  switch (t) {
    case OR_F32: {
      if (nbytes < count * 4) return -2;
      memcpy(out, data, count * 4);
      return (long)count;
    }
    case OR_F16: return (long)dq_f16(data, nbytes, count, out);
    case OR_Q4_0: return (long)dq_q4_0(data, nbytes, count, out);
    case OR_Q4_1: return (long)dq_q4_1(data, nbytes, count, out);
    case OR_Q5_0: return (long)dq_q5_0(data, nbytes, count, out);
    case OR_Q8_0: return (long)dq_q8_0(data, nbytes, count, out);
    case OR_Q4_K: return (long)dq_q4_k(data, nbytes, count, out);
    case OR_Q6_K: return (long)dq_q6_k(data, nbytes, count, out);
    default: return -1;
  }
}

/* ------------------------------------------------------------------------ */
/* reference test quantisers, src/quant.rs:393-471                           */
/* ------------------------------------------------------------------------ */
static int32_t sat_i32(float v) { /* Rust `as i32` */
  if (v != v) return 0;
  if (v >= 2147483647.0f) return 2147483647;
  if (v <= -2147483648.0f) return (int32_t)0x80000000u;
  return (int32_t)v;
}
static int16_t sat_i16(float v) {
  if (v != v) return 0;
  if (v >= 32767.0f) return 32767;
  if (v <= -32768.0f) return -32768;
  return (int16_t)v;
}

size_t or_quantize_q4_0(const float *v, size_t n, uint8_t *out) {
  size_t nb = (n + 31) / 32, o = 0;
  for (size_t b = 0; b < nb; ++b) {
    size_t s = b * 32, e = s + 32 < n ? s + 32 : n;
    float max_abs = 0.0f;
    for (size_t i = s; i < e; ++i) max_abs = fmaxf(max_abs, fabsf(v[i]));
    float d = max_abs == 0.0f ? 1.0f : max_abs / 8.0f;
    uint16_t dh = or_f32_to_f16(d);
    out[o++] = (uint8_t)(dh & 0xFF);
    out[o++] = (uint8_t)(dh >> 8);
    float inv_d = d != 0.0f ? 1.0f / d : 0.0f;
    uint8_t nib[32];
    size_t c = 0;
    for (size_t i = s; i < e; ++i) {
      int32_t sc = sat_i32(roundf(v[i] * inv_d + 8.0f));
      nib[c++] = (uint8_t)(sc < 0 ? 0 : (sc > 15 ? 15 : sc));
    }
    while (c < 32) nib[c++] = 8;
    for (int i = 0; i < 32; i += 2) out[o++] = (uint8_t)((nib[i] << 4) | nib[i + 1]);
  }
  return o;
}

size_t or_quantize_q8_0(const float *v, size_t n, uint8_t *out) {
  size_t nb = (n + 31) / 32, o = 0;
  for (size_t b = 0; b < nb; ++b) {
    size_t s = b * 32, e = s + 32 < n ? s + 32 : n;
    float max_abs = 0.0f;
    for (size_t i = s; i < e; ++i) max_abs = fmaxf(max_abs, fabsf(v[i]));
    float d = max_abs == 0.0f ? 1.0f : max_abs / 127.0f;
    uint16_t dh = or_f32_to_f16(d);
    out[o++] = (uint8_t)(dh & 0xFF);
    out[o++] = (uint8_t)(dh >> 8);
    float inv_d = d != 0.0f ? 1.0f / d : 0.0f;
    for (size_t i = s; i < e; ++i) {
      int16_t sc = sat_i16(roundf(v[i] * inv_d));
      int8_t q = (int8_t)(sc < -128 ? -128 : (sc > 127 ? 127 : sc));
      out[o++] = (uint8_t)q;
    }
    for (size_t i = e; i < s + 32; ++i) out[o++] = 0;
  }
  return o;
}

/* ------------------------------------------------------------------------ */
/* tensor math, src/tensor.rs                                                */
/* ------------------------------------------------------------------------ */
/* matmul, src/tensor.rs:244-258: i-j-p, sum from 0.0 in ascending p */
void or_matmul(const float *a, const float *b, size_t m, size_t k, size_t n, float *c) {
  for (size_t i = 0; i < m; ++i)
    for (size_t j = 0; j < n; ++j) {
      float sum = 0.0f;
      for (size_t p = 0; p < k; ++p) sum += a[i * k + p] * b[p * n + j];
      c[i * n + j] = sum;
    }
}

/* rms_norm, src/tensor.rs:280-290 */
void or_rms_norm(const float *x, const float *w, size_t n, float eps, float *y) {
  float ss = 0.0f;
  for (size_t i = 0; i < n; ++i) ss += x[i] * x[i];
  float mean_sq = ss / (float)n;
  float inv = 1.0f / sqrtf(mean_sq + eps);
  for (size_t i = 0; i < n; ++i) y[i] = x[i] * inv * w[i];
}

/* sigmoid / silu, src/tensor.rs:307-309, :589-591 */
static inline float sigmoidf_ref(float x) { return 1.0f / (1.0f + expf(-x)); }
void or_silu(const float *x, size_t n, float *y) {
  for (size_t i = 0; i < n; ++i) y[i] = x[i] * sigmoidf_ref(x[i]);
}

/* softmax (in place), src/tensor.rs:325-344 */
void or_softmax_inplace(float *x, size_t n) {
  if (!n) return;
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = fmaxf(mx, x[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) { x[i] = expf(x[i] - mx); sum += x[i]; }
  float inv = 1.0f / sum;
  for (size_t i = 0; i < n; ++i) x[i] *= inv;
}

/* rope_emb, src/tensor.rs:386-397: [cos0, sin0, cos1, sin1, ...] */
void or_rope_emb(size_t pos, size_t dim, float base, float *emb) {
  size_t half = dim / 2;
  for (size_t i = 0; i < half; ++i) {
    float freq = 1.0f / powf(base, (2.0f * (float)i) / (float)dim);
    float angle = (float)pos * freq;
    emb[2 * i] = cosf(angle);
    emb[2 * i + 1] = sinf(angle);
  }
}

/* apply_rope_to_tensor, src/model.rs:469-491: half-split pairs (d, d+hd/2) */
void or_apply_rope_to_tensor(float *data, size_t len, size_t n_h, size_t hd, size_t pos, float base) {
  if (!n_h || !hd) return;
  size_t seq = len / (n_h * hd);
  if (!seq) return;
  float *emb = (float *)malloc(hd * sizeof(float));
  or_rope_emb(pos, hd, base, emb);
  size_t half = hd / 2;
  for (size_t s = 0; s < seq; ++s)
    for (size_t h = 0; h < n_h; ++h) {
      float *p = data + s * n_h * hd + h * hd;
      for (size_t d = 0; d < half; ++d) {
        float c = emb[2 * d], sn = emb[2 * d + 1];
        float x0 = p[d], x1 = p[d + half];
        p[d] = x0 * c - x1 * sn;
        p[d + half] = x0 * sn + x1 * c;
      }
    }
  free(emb);
}

/* scaled_dot_product_attention without cache/mask (src/tensor.rs:451-551)
 * with GQA expansion folded in: q head h reads kv head h / (n_heads/n_kv)
 * exactly as expand_kv_heads (src/model.rs:500-526) lays it out.
 * k, v: kv_len rows of n_kv*hd. */
static void sdpa_gqa(const float *q, const float *k, const float *v, size_t q_len, size_t kv_len,
                     size_t n_heads, size_t n_kv, size_t hd, float *out, float *scores) {
  size_t n_rep = n_heads / n_kv;
  size_t kvd = n_kv * hd, qd = n_heads * hd;
  float scale = 1.0f / sqrtf((float)hd);
  for (size_t h = 0; h < n_heads; ++h) {
    size_t kh = h / n_rep;
    for (size_t qi = 0; qi < q_len; ++qi) {
      const float *qv = q + qi * qd + h * hd;
      float mx = -INFINITY;
      for (size_t ki = 0; ki < kv_len; ++ki) {
        const float *kv_ = k + ki * kvd + kh * hd;
        float dot = 0.0f;
        for (size_t d = 0; d < hd; ++d) dot += qv[d] * kv_[d];
        scores[ki] = dot * scale;
        if (scores[ki] > mx) mx = scores[ki];
      }
      float es = 0.0f;
      for (size_t ki = 0; ki < kv_len; ++ki) { scores[ki] = expf(scores[ki] - mx); es += scores[ki]; }
      float inv = 1.0f / es;
      for (size_t ki = 0; ki < kv_len; ++ki) scores[ki] *= inv;
      float *o = out + qi * qd + h * hd;
      for (size_t d = 0; d < hd; ++d) {
        float val = 0.0f;
        for (size_t ki = 0; ki < kv_len; ++ki) val += scores[ki] * v[ki * kvd + kh * hd + d];
        o[d] = val;
      }
    }
  }
}

void or_sdpa(const float *q, const float *k, const float *v, size_t q_len, size_t kv_len,
             size_t n_heads, size_t hd, float *out) {
  float *scores = (float *)malloc((kv_len ? kv_len : 1) * sizeof(float));
  sdpa_gqa(q, k, v, q_len, kv_len, n_heads, n_heads, hd, out, scores);
  free(scores);
}

/* ------------------------------------------------------------------------ */
/* Philox4x32-10 (Salmon, Moraes, Dror, Shaw: "Parallel random numbers: as   */
/* easy as 1, 2, 3", SC'11).  Round constants and Weyl key increments are    */
/* the published ones.                                                       */
/* ------------------------------------------------------------------------ */
void or_philox4x32_10(const uint32_t ctr[4], const uint32_t key[2], uint32_t out[4]) {
  uint32_t c0 = ctr[0], c1 = ctr[1], c2 = ctr[2], c3 = ctr[3], k0 = key[0], k1 = key[1];
  for (int r = 0; r < 10; ++r) {
    uint64_t p0 = (uint64_t)0xD2511F53u * c0, p1 = (uint64_t)0xCD9E8D57u * c2;
    uint32_t hi0 = (uint32_t)(p0 >> 32), lo0 = (uint32_t)p0;
    uint32_t hi1 = (uint32_t)(p1 >> 32), lo1 = (uint32_t)p1;
    uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0; c1 = lo1; c2 = n2; c3 = lo0;
    k0 += 0x9E3779B9u; k1 += 0xBB67AE85u;
  }
  out[0] = c0; out[1] = c1; out[2] = c2; out[3] = c3;
}

/* uniform in [0,1): top 24 bits of the first Philox word, key = seed,
 * counter = (step, 0, 0, 0) */
float or_philox_uniform(uint64_t seed, uint64_t step) {
  uint32_t ctr[4] = {(uint32_t)step, (uint32_t)(step >> 32), 0, 0};
  uint32_t key[2] = {(uint32_t)seed, (uint32_t)(seed >> 32)};
  uint32_t o[4];
  or_philox4x32_10(ctr, key, o);
  return (float)(o[0] >> 8) * (1.0f / 16777216.0f);
}

/* ------------------------------------------------------------------------ */
/* GGUF parser, src/gguf.rs:438-689                                          */
/* ------------------------------------------------------------------------ */
enum { GV_U8 = 0, GV_I8, GV_U16, GV_I16, GV_U32, GV_I32, GV_F32, GV_BOOL, GV_STR, GV_ARR, GV_U64, GV_I64, GV_F64 };

typedef struct {
  char *key;
  uint32_t type;
  uint64_t u; int64_t i; double f; float f32; int b;
  char *s;
  uint32_t arr_type; uint64_t arr_len;
} or_meta;

typedef struct {
  char *name;
  uint32_t n_dims;
  uint64_t dims[4];
  uint32_t ggml_type;
  uint64_t offset;
} or_tinfo;

struct or_gguf {
  uint32_t version;
  uint64_t alignment;
  or_meta *meta; size_t n_meta;
  or_tinfo *ti; size_t n_ti;
  const uint8_t *map; size_t map_len;
  size_t data_offset;
};

typedef struct { const uint8_t *p; size_t len, pos; } cur_t;

static int rd(cur_t *c, void *dst, size_t n) {
  if (c->pos + n > c->len) return -1;
  memcpy(dst, c->p + c->pos, n);
  c->pos += n;
  return 0;
}

/* read_string, src/gguf.rs:264-282 (length cap 256 MiB) */
static int rd_str(cur_t *c, char **out, char *err, size_t errlen) {
  uint64_t len;
  if (rd(c, &len, 8)) { set_err(err, errlen, "failed to read string length"); return -1; }
  if (len > 256ull * 1024 * 1024) { set_err(err, errlen, "string length too large: %llu", (unsigned long long)len); return -1; }
  if (c->pos + len > c->len) { set_err(err, errlen, "failed to read string data (want %llu bytes)", (unsigned long long)len); return -1; }
  char *s = (char *)malloc(len + 1);
  memcpy(s, c->p + c->pos, len);
  s[len] = 0;
  c->pos += len;
  *out = s;
  return 0;
}

static const size_t gv_size[13] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};

/* read_value_at, src/gguf.rs:287-401 */
static int rd_value(cur_t *c, uint32_t t, or_meta *m, int depth, char *err, size_t errlen) {
  m->type = t;
  switch (t) {
    case GV_U8: { uint8_t v; if (rd(c, &v, 1)) goto short_; m->u = v; return 0; }
    case GV_I8: { int8_t v; if (rd(c, &v, 1)) goto short_; m->i = v; return 0; }
    case GV_U16: { uint16_t v; if (rd(c, &v, 2)) goto short_; m->u = v; return 0; }
    case GV_I16: { int16_t v; if (rd(c, &v, 2)) goto short_; m->i = v; return 0; }
    case GV_U32: { uint32_t v; if (rd(c, &v, 4)) goto short_; m->u = v; return 0; }
    case GV_I32: { int32_t v; if (rd(c, &v, 4)) goto short_; m->i = v; return 0; }
    case GV_F32: { float v; if (rd(c, &v, 4)) goto short_; m->f32 = v; return 0; }
    case GV_BOOL: { uint8_t v; if (rd(c, &v, 1)) goto short_; m->b = v != 0; return 0; }
    case GV_STR: return rd_str(c, &m->s, err, errlen);
    case GV_U64: { uint64_t v; if (rd(c, &v, 8)) goto short_; m->u = v; return 0; }
    case GV_I64: { int64_t v; if (rd(c, &v, 8)) goto short_; m->i = v; return 0; }
    case GV_F64: { double v; if (rd(c, &v, 8)) goto short_; m->f = v; return 0; }
    case GV_ARR: {
      uint32_t it; uint64_t cnt;
      if (rd(c, &it, 4)) goto short_;
      if (it > GV_F64) { set_err(err, errlen, "unknown array item type: %u", it); return -1; }
      if (rd(c, &cnt, 8)) goto short_;
      if (cnt > 10000000ull) { set_err(err, errlen, "array too large: %llu", (unsigned long long)cnt); return -1; }
      m->arr_type = it; m->arr_len = cnt;
      for (uint64_t i = 0; i < cnt; ++i) {
        if (it == GV_STR) {
          char *s = NULL;
          if (rd_str(c, &s, err, errlen)) return -1;
          free(s);
        } else if (it == GV_ARR) {
          or_meta tmp; memset(&tmp, 0, sizeof tmp);
          if (depth > 8 || rd_value(c, it, &tmp, depth + 1, err, errlen)) return -1;
          free(tmp.s);
        } else {
          if (c->pos + gv_size[it] > c->len) goto short_;
          c->pos += gv_size[it];
        }
      }
      return 0;
    }
    default: set_err(err, errlen, "unknown value type: %u", t); return -1;
  }
short_:
  set_err(err, errlen, "truncated metadata value");
  return -1;
}

void or_gguf_close(or_gguf *g) {
  if (!g) return;
  for (size_t i = 0; i < g->n_meta; ++i) { free(g->meta[i].key); free(g->meta[i].s); }
  for (size_t i = 0; i < g->n_ti; ++i) free(g->ti[i].name);
  free(g->meta); free(g->ti);
  if (g->map && g->map_len) munmap((void *)g->map, g->map_len);
  free(g);
}

static const or_meta *find_meta(const or_gguf *g, const char *key) {
  /* HashMap::insert keeps the last value for a repeated key */
  for (size_t i = g->n_meta; i-- > 0;)
    if (!strcmp(g->meta[i].key, key)) return &g->meta[i];
  return NULL;
}

or_gguf *or_gguf_open(const char *path, char *err, size_t errlen) {
  int fd = open(path, O_RDONLY);
  if (fd < 0) { set_err(err, errlen, "cannot open file '%s'", path); return NULL; }
  struct stat st;
  if (fstat(fd, &st)) { close(fd); set_err(err, errlen, "cannot stat '%s'", path); return NULL; }
  or_gguf *g = (or_gguf *)calloc(1, sizeof *g);
  g->map_len = (size_t)st.st_size;
  if (g->map_len) {
    void *p = mmap(NULL, g->map_len, PROT_READ, MAP_PRIVATE, fd, 0);
    if (p == MAP_FAILED) { close(fd); free(g); set_err(err, errlen, "cannot map '%s'", path); return NULL; }
    g->map = (const uint8_t *)p;
  }
  close(fd);
  cur_t c = {g->map, g->map_len, 0};
  uint32_t magic, version;
  uint64_t n_t, n_kv;
  if (rd(&c, &magic, 4)) { set_err(err, errlen, "failed to read magic"); goto fail; }
  if (magic != 0x46465547u) { set_err(err, errlen, "invalid GGUF magic: expected 0x46465547, got 0x%08X", magic); goto fail; }
  if (rd(&c, &version, 4)) { set_err(err, errlen, "failed to read version"); goto fail; }
  if (version > 3) { set_err(err, errlen, "unsupported GGUF version: %u (max 3)", version); goto fail; }
  if (rd(&c, &n_t, 8) || rd(&c, &n_kv, 8)) { set_err(err, errlen, "failed to read counts"); goto fail; }
  if (n_t > 1000000ull) { set_err(err, errlen, "tensor count out of range: %llu", (unsigned long long)n_t); goto fail; }
  if (n_kv > 10000000ull) { set_err(err, errlen, "metadata count out of range: %llu", (unsigned long long)n_kv); goto fail; }
  g->version = version;
  g->meta = (or_meta *)calloc(n_kv ? n_kv : 1, sizeof(or_meta));
  for (uint64_t i = 0; i < n_kv; ++i) {
    or_meta *m = &g->meta[i];
    if (rd_str(&c, &m->key, err, errlen)) goto fail;
    g->n_meta = i + 1;
    uint32_t vt;
    if (rd(&c, &vt, 4)) { set_err(err, errlen, "failed to read value type"); goto fail; }
    if (vt > GV_F64) { set_err(err, errlen, "unknown value type: %u", vt); goto fail; }
    if (rd_value(&c, vt, m, 0, err, errlen)) goto fail;
  }
  g->alignment = 32;
  const or_meta *am = find_meta(g, "general.alignment");
  if (am && (am->type == GV_U64 || am->type == GV_U32)) g->alignment = am->u;
  if (g->alignment == 0 || (g->alignment & (g->alignment - 1))) {
    set_err(err, errlen, "invalid alignment: %llu (must be a power of two)", (unsigned long long)g->alignment);
    goto fail;
  }
  g->ti = (or_tinfo *)calloc(n_t ? n_t : 1, sizeof(or_tinfo));
  for (uint64_t i = 0; i < n_t; ++i) {
    or_tinfo *t = &g->ti[i];
    if (rd_str(&c, &t->name, err, errlen)) goto fail;
    g->n_ti = i + 1;
    if (rd(&c, &t->n_dims, 4)) { set_err(err, errlen, "failed to read n_dims"); goto fail; }
    if (t->n_dims > 4) { set_err(err, errlen, "tensor n_dims %u exceeds 4", t->n_dims); goto fail; }
    for (uint32_t d = 0; d < t->n_dims; ++d)
      if (rd(&c, &t->dims[d], 8)) { set_err(err, errlen, "failed to read dim"); goto fail; }
    if (rd(&c, &t->ggml_type, 4) || rd(&c, &t->offset, 8)) { set_err(err, errlen, "failed to read tensor type/offset"); goto fail; }
  }
  g->data_offset = (c.pos + g->alignment - 1) & ~(size_t)(g->alignment - 1);
  return g;
fail:
  or_gguf_close(g);
  return NULL;
}

uint32_t or_gguf_version(const or_gguf *g) { return g->version; }
uint64_t or_gguf_alignment(const or_gguf *g) { return g->alignment; }
size_t or_gguf_tensor_count(const or_gguf *g) { return g->n_ti; }
const char *or_gguf_tensor_name(const or_gguf *g, size_t i) { return i < g->n_ti ? g->ti[i].name : NULL; }

static const or_tinfo *find_tensor(const or_gguf *g, const char *name) {
  for (size_t i = 0; i < g->n_ti; ++i)
    if (!strcmp(g->ti[i].name, name)) return &g->ti[i];
  return NULL;
}

int or_gguf_tensor_info(const or_gguf *g, const char *name, uint32_t *n_dims, uint64_t dims[4],
                        uint32_t *ggml_type, uint64_t *offset) {
  const or_tinfo *t = find_tensor(g, name);
  if (!t) return -1;
  if (n_dims) *n_dims = t->n_dims;
  if (dims) for (int i = 0; i < 4; ++i) dims[i] = i < (int)t->n_dims ? t->dims[i] : 0;
  if (ggml_type) *ggml_type = t->ggml_type;
  if (offset) *offset = t->offset;
  return 0;
}

static uint64_t tinfo_nelement(const or_tinfo *t) {
  uint64_t n = 1;
  for (uint32_t d = 0; d < t->n_dims; ++d) n *= t->dims[d];
  return n;
}

/* tensor_byte_size (src/gguf.rs:645-658) + read_tensor_data (:663-672):
 * size runs to the next larger tensor offset, else to the end of file;
 * out-of-range reads yield an empty result. */
static const uint8_t *tensor_bytes(const or_gguf *g, const or_tinfo *t, size_t *nbytes) {
  size_t data_end = g->map_len > g->data_offset ? g->map_len - g->data_offset : 0;
  uint64_t next = data_end;
  for (size_t i = 0; i < g->n_ti; ++i)
    if (g->ti[i].offset > t->offset && g->ti[i].offset < next) next = g->ti[i].offset;
  if (next < t->offset) { *nbytes = 0; return NULL; }
  size_t sz = (size_t)(next - t->offset);
  size_t start = g->data_offset + (size_t)t->offset;
  if (start + sz > g->map_len || sz == 0) { *nbytes = 0; return NULL; }
  *nbytes = sz;
  return g->map + start;
}

size_t or_gguf_read_tensor_data(const or_gguf *g, const char *name, uint8_t *out, size_t cap) {
  const or_tinfo *t = find_tensor(g, name);
  if (!t) return 0;
  size_t n;
  const uint8_t *p = tensor_bytes(g, t, &n);
  if (!p) return 0;
  if (out) memcpy(out, p, n < cap ? n : cap);
  return n;
}

int or_gguf_meta_u64(const or_gguf *g, const char *key, uint64_t *v) {
  const or_meta *m = find_meta(g, key);
  if (!m || (m->type != GV_U64 && m->type != GV_U32)) return 0;
  *v = m->u;
  return 1;
}
int or_gguf_meta_i64(const or_gguf *g, const char *key, int64_t *v) {
  const or_meta *m = find_meta(g, key);
  if (!m || (m->type != GV_I64 && m->type != GV_I32)) return 0;
  *v = m->i;
  return 1;
}
int or_gguf_meta_f32(const or_gguf *g, const char *key, float *v) {
  const or_meta *m = find_meta(g, key);
  if (!m || m->type != GV_F32) return 0;
  *v = m->f32;
  return 1;
}
int or_gguf_meta_bool(const or_gguf *g, const char *key, int *v) {
  const or_meta *m = find_meta(g, key);
  if (!m || m->type != GV_BOOL) return 0;
  *v = m->b;
  return 1;
}
int or_gguf_meta_string(const or_gguf *g, const char *key, char *buf, size_t cap) {
  const or_meta *m = find_meta(g, key);
  if (!m || m->type != GV_STR) return 0;
  if (buf && cap) { strncpy(buf, m->s, cap - 1); buf[cap - 1] = 0; }
  return 1;
}
/* vocab_size, src/gguf.rs:748-758 */
int or_gguf_vocab_size(const or_gguf *g, uint64_t *v) {
  if (or_gguf_meta_u64(g, "general.tokenizer.ggml.vocab_size", v)) return 1;
  const or_meta *m = find_meta(g, "general.tokenizer.ggml.tokens");
  if (m && m->type == GV_ARR) { *v = m->arr_len; return 1; }
  return 0;
}

/* ------------------------------------------------------------------------ */
/* ModelConfig, src/model.rs:66-180                                          */
/* ------------------------------------------------------------------------ */
size_t or_config_n_ff(size_t n_embd, float mult) {
  float raw = (float)n_embd * mult;
  size_t r = raw != raw || raw <= 0.0f ? 0 : (size_t)raw; /* Rust saturating cast */
  return ((r + 255) / 256) * 256;
}

int or_config_from_gguf(const or_gguf *g, or_config *cfg, char *err, size_t errlen) {
  char arch[64];
  memset(cfg, 0, sizeof *cfg);
  if (!or_gguf_meta_string(g, "general.architecture", arch, sizeof arch)) {
    set_err(err, errlen, "missing general.architecture");
    return -1;
  }
  if (strcmp(arch, "llama") && strcmp(arch, "qwen2") && strcmp(arch, "mistral") && strcmp(arch, "phi")) {
    set_err(err, errlen, "unsupported architecture: %s", arch);
    return -1;
  }
  char key[160];
  uint64_t v;
#define REQ(field, suffix)                                                    \
  snprintf(key, sizeof key, "%s." suffix, arch);                              \
  if (!or_gguf_meta_u64(g, key, &v)) { set_err(err, errlen, "missing %s", key); return -1; } \
  cfg->field = (size_t)v;
  REQ(n_layers, "block_count");
  REQ(n_heads, "attention.head_count");
  snprintf(key, sizeof key, "%s.attention.head_count_kv", arch);
  cfg->n_kv_heads = or_gguf_meta_u64(g, key, &v) ? (size_t)v : cfg->n_heads;
  REQ(n_embd, "embedding_length");
  REQ(context_len, "context_length");
#undef REQ
  if (or_gguf_vocab_size(g, &v)) {
    cfg->vocab_size = (size_t)v;
  } else {
    const or_tinfo *t = find_tensor(g, "token_embd.weight");
    if (!t) { set_err(err, errlen, "cannot determine vocab size"); return -1; }
    cfg->vocab_size = cfg->n_embd ? (size_t)(tinfo_nelement(t) / cfg->n_embd) : 0;
  }
  if (cfg->n_heads == 0) { set_err(err, errlen, "attention.head_count is 0"); return -1; }
  cfg->head_dim = cfg->n_embd / cfg->n_heads;
  if (cfg->head_dim == 0) { set_err(err, errlen, "n_embd %zu not divisible by heads %zu", cfg->n_embd, cfg->n_heads); return -1; }
  float f;
  snprintf(key, sizeof key, "%s.feed_forward_length", arch);
  cfg->ffn_dim_multiplier = or_gguf_meta_f32(g, key, &f) ? f / (float)cfg->n_embd : 2.667f;
  snprintf(key, sizeof key, "%s.attention.layer_norm_rms_epsilon", arch);
  cfg->norm_eps = or_gguf_meta_f32(g, key, &f) ? f : 1e-5f;
  snprintf(key, sizeof key, "%s.rope.freq_base", arch);
  cfg->rope_base = or_gguf_meta_f32(g, key, &f) ? f : 10000.0f;
  cfg->rope_freq_dim = cfg->head_dim / 2;
  cfg->n_ff = or_config_n_ff(cfg->n_embd, cfg->ffn_dim_multiplier);
  cfg->n_ff_used = cfg->n_ff;
  cfg->tied_output = find_tensor(g, "output.weight") == NULL;
  return 0;
}

/* ------------------------------------------------------------------------ */
/* model weights (src/model.rs:193-298)                                      */
/* ------------------------------------------------------------------------ */
typedef struct {
  int type;
  size_t nelem;
  const uint8_t *raw; size_t nbytes;  /* native blocks (mmap) */
  float *f32;                         /* resident dequantised copy or NULL */
} or_tensor;

enum { T_NORM1, T_Q, T_K, T_V, T_O, T_NORM2, T_GATE, T_UP, T_DOWN, T_PER_LAYER };

struct or_model {
  or_gguf *g;
  or_config cfg;
  or_tensor embd, out_norm, out;
  or_tensor *layers; /* n_layers * T_PER_LAYER */
  int resident;
  int threads;
};

static int load_tensor(or_model *m, const char *name, or_tensor *t, int required, char *err, size_t errlen) {
  const or_tinfo *ti = find_tensor(m->g, name);
  memset(t, 0, sizeof *t);
  if (!ti) {
    if (required) set_err(err, errlen, "tensor not found: %s", name);
    return required ? -1 : 1;
  }
  t->type = (int)ti->ggml_type;
  t->nelem = (size_t)tinfo_nelement(ti);
  t->raw = tensor_bytes(m->g, ti, &t->nbytes);
  if (!t->raw) { set_err(err, errlen, "tensor '%s' has no data", name); return -1; }
  if (t->type != OR_F32 && t->type != OR_F16 && t->type != OR_Q4_0 && t->type != OR_Q4_1 &&
      t->type != OR_Q5_0 && t->type != OR_Q8_0 && t->type != OR_Q4_K && t->type != OR_Q6_K) {
    set_err(err, errlen, "unsupported ggml type for dequantization: %d", t->type);
    return -1;
  }
  if (m->resident) {
    t->f32 = (float *)malloc(t->nelem * sizeof(float));
    if (!t->f32) { set_err(err, errlen, "out of memory"); return -1; }
    long got = or_dequantize(t->raw, t->nbytes, t->type, t->nelem, t->f32);
    if (got < 0 || (size_t)got != t->nelem) { set_err(err, errlen, "tensor '%s': short data", name); return -1; }
  }
  return 0;
}

static void free_tensor(or_tensor *t) { free(t->f32); t->f32 = NULL; }

void or_model_free(or_model *m) {
  if (!m) return;
  free_tensor(&m->embd); free_tensor(&m->out_norm); free_tensor(&m->out);
  if (m->layers) for (size_t i = 0; i < m->cfg.n_layers * T_PER_LAYER; ++i) free_tensor(&m->layers[i]);
  free(m->layers);
  or_gguf_close(m->g);
  free(m);
}

or_model *or_model_load(const char *path, int resident, char *err, size_t errlen) {
  or_model *m = (or_model *)calloc(1, sizeof *m);
  m->resident = resident;
  m->threads = 1;
  m->g = or_gguf_open(path, err, errlen);
  if (!m->g) { free(m); return NULL; }
  if (or_config_from_gguf(m->g, &m->cfg, err, errlen)) goto fail;
  if (load_tensor(m, "token_embd.weight", &m->embd, 1, err, errlen)) goto fail;
  m->layers = (or_tensor *)calloc(m->cfg.n_layers * T_PER_LAYER, sizeof(or_tensor));
  static const char *names[T_PER_LAYER] = {"attn_norm", "attn_q", "attn_k", "attn_v", "attn_output",
                                           "ffn_norm", "ffn_gate", "ffn_up", "ffn_down"};
  for (size_t l = 0; l < m->cfg.n_layers; ++l)
    for (int j = 0; j < T_PER_LAYER; ++j) {
      char nm[96];
      snprintf(nm, sizeof nm, "blk.%zu.%s.weight", l, names[j]);
      if (load_tensor(m, nm, &m->layers[l * T_PER_LAYER + j], 1, err, errlen)) goto fail;
    }
  if (load_tensor(m, "output_norm.weight", &m->out_norm, 1, err, errlen)) goto fail;
  {
    int r = load_tensor(m, "output.weight", &m->out, 0, err, errlen);
    if (r < 0) goto fail;
    m->cfg.tied_output = r == 1;
  }
  /* D2: use the FFN tensor's own width when n_ff() disagrees */
  {
    size_t gate_n = m->layers[T_GATE].nelem / m->cfg.n_embd;
    m->cfg.n_ff_used = gate_n;
    m->cfg.n_ff_deviation = gate_n != m->cfg.n_ff;
  }
  return m;
fail:
  or_model_free(m);
  return NULL;
}

void or_model_config(const or_model *m, or_config *cfg) { *cfg = m->cfg; }
void or_model_set_threads(or_model *m, int threads) { m->threads = threads < 1 ? 1 : threads; }

/* dequantise elements [e0, e0+n) of a tensor (both block aligned) */
static void tensor_slice(const or_tensor *t, size_t e0, size_t n, float *out) {
  if (t->f32) { memcpy(out, t->f32 + e0, n * sizeof(float)); return; }
  size_t bs = or_block_size(t->type), ts = or_type_size(t->type);
  size_t b0 = e0 / bs;
  size_t off = b0 * ts;
  or_dequantize(t->raw + off, t->nbytes > off ? t->nbytes - off : 0, t->type, n, out);
}

/* ------------------------------------------------------------------------ */
/* threads                                                                   */
/* ------------------------------------------------------------------------ */
typedef void (*task_fn)(void *ctx, size_t task);
typedef struct { task_fn fn; void *ctx; size_t n; size_t next; pthread_mutex_t mu; } pool_t;

static void *pool_worker(void *arg) {
  pool_t *p = (pool_t *)arg;
  for (;;) {
    pthread_mutex_lock(&p->mu);
    size_t t = p->next++;
    pthread_mutex_unlock(&p->mu);
    if (t >= p->n) break;
    p->fn(p->ctx, t);
  }
  return NULL;
}

static void parallel_for(int threads, size_t n, task_fn fn, void *ctx) {
  if (threads <= 1 || n <= 1) {
    for (size_t i = 0; i < n; ++i) fn(ctx, i);
    return;
  }
  pool_t p = {fn, ctx, n, 0, PTHREAD_MUTEX_INITIALIZER};
  int nt = threads < (int)n ? threads : (int)n;
  pthread_t th[256];
  if (nt > 256) nt = 256;
  for (int i = 0; i < nt; ++i) pthread_create(&th[i], NULL, pool_worker, &p);
  for (int i = 0; i < nt; ++i) pthread_join(th[i], NULL);
}

/* ------------------------------------------------------------------------ */
/* matmul against a (possibly quantised) weight W[K][N]                      */
/* ------------------------------------------------------------------------ */
/* algo 0: reference i-j-p order on a resident f32 copy (dequantised into a
 *         temporary when the model keeps blocks).
 * algo 1: fast mode.  Every c[i][j] still accumulates a[i][p]*w[p][j] in
 *         ascending p starting from 0.0f with separate multiply and add, so
 *         the result is bit-identical to algo 0; loops are tiled over
 *         (column tile, row block) and columns are split across threads. */
typedef struct {
  const float *a; const or_tensor *w; size_t m, k, n; float *c;
  size_t tile; size_t bs;
} mm_ctx;
static void or__mm_wide(const or_model *m, mm_ctx *x);

#define MM_TILE 64
typedef float v8f __attribute__((vector_size(32)));

static void mm_task(void *vctx, size_t task) {
  mm_ctx *x = (mm_ctx *)vctx;
  size_t j0 = task * x->tile;
  size_t nj = j0 + x->tile <= x->n ? x->tile : x->n - j0;
  size_t K = x->k, N = x->n, M = x->m;
  /* dequantised column tile wt[p][0..nj) */
  float *wt = (float *)aligned_alloc(64, ((K * MM_TILE * sizeof(float)) + 63) & ~(size_t)63);
  float *row = (float *)malloc(x->bs > nj ? x->bs * sizeof(float) : nj * sizeof(float) + 64);
  for (size_t p = 0; p < K; ++p) {
    tensor_slice(x->w, p * N + j0, nj, row);
    memcpy(wt + p * MM_TILE, row, nj * sizeof(float));
    for (size_t j = nj; j < MM_TILE; ++j) wt[p * MM_TILE + j] = 0.0f;
  }
  free(row);
  size_t i = 0;
  for (; i + 2 <= M; i += 2) {
    v8f acc0[MM_TILE / 8], acc1[MM_TILE / 8];
    for (int v = 0; v < MM_TILE / 8; ++v) { acc0[v] = (v8f){0}; acc1[v] = (v8f){0}; }
    const float *a0 = x->a + i * K, *a1 = a0 + K;
    for (size_t p = 0; p < K; ++p) {
      const v8f *w = (const v8f *)(wt + p * MM_TILE);
      v8f b0 = (v8f){0} + a0[p], b1 = (v8f){0} + a1[p];
      for (int v = 0; v < MM_TILE / 8; ++v) {
        v8f t0 = b0 * w[v];
        v8f t1 = b1 * w[v];
        acc0[v] = acc0[v] + t0;
        acc1[v] = acc1[v] + t1;
      }
    }
    float *c0 = x->c + i * N + j0, *c1 = c0 + N;
    for (size_t j = 0; j < nj; ++j) { c0[j] = acc0[j / 8][j % 8]; c1[j] = acc1[j / 8][j % 8]; }
  }
  for (; i < M; ++i) {
    v8f acc0[MM_TILE / 8];
    for (int v = 0; v < MM_TILE / 8; ++v) acc0[v] = (v8f){0};
    const float *a0 = x->a + i * K;
    for (size_t p = 0; p < K; ++p) {
      const v8f *w = (const v8f *)(wt + p * MM_TILE);
      v8f b0 = (v8f){0} + a0[p];
      for (int v = 0; v < MM_TILE / 8; ++v) { v8f t0 = b0 * w[v]; acc0[v] = acc0[v] + t0; }
    }
    float *c0 = x->c + i * N + j0;
    for (size_t j = 0; j < nj; ++j) c0[j] = acc0[j / 8][j % 8];
  }
  free(wt);
}

static void wmatmul(const or_model *m, const float *a, const or_tensor *w, size_t M, size_t K, size_t N,
                    float *c, int algo) {
  if (algo == 0) {
    if (w->f32) { or_matmul(a, w->f32, M, K, N, c); return; }
    float *tmp = (float *)malloc(K * N * sizeof(float));
    tensor_slice(w, 0, K * N, tmp);
    or_matmul(a, tmp, M, K, N, c);
    free(tmp);
    return;
  }
  size_t bs = or_block_size(w->type);
  mm_ctx x = {a, w, M, K, N, c, MM_TILE, bs};
  if (bs <= MM_TILE) { /* 64-column tiles stay block aligned for 1/32-element blocks */
    parallel_for(m->threads, (N + MM_TILE - 1) / MM_TILE, mm_task, &x);
    return;
  }
  /* 256-element blocks: one task owns a whole super-block column tile */
  or__mm_wide(m, &x);
}

/* wide-tile variant for 256-element blocks: each task owns 256 columns */
typedef struct { mm_ctx *x; } wide_ctx;
static void mm_wide_task(void *vctx, size_t task) {
  mm_ctx *x = ((wide_ctx *)vctx)->x;
  size_t j0 = task * 256;
  size_t nj = j0 + 256 <= x->n ? 256 : x->n - j0;
  size_t K = x->k, N = x->n, M = x->m;
  float *wt = (float *)aligned_alloc(64, K * 256 * sizeof(float));
  float *row = (float *)malloc(256 * sizeof(float));
  for (size_t p = 0; p < K; ++p) {
    tensor_slice(x->w, p * N + j0, nj, row);
    memcpy(wt + p * 256, row, nj * sizeof(float));
    for (size_t j = nj; j < 256; ++j) wt[p * 256 + j] = 0.0f;
  }
  free(row);
  for (size_t sub = 0; sub < 4; ++sub) {
    size_t s0 = sub * 64;
    if (s0 >= nj) break;
    size_t sn = s0 + 64 <= nj ? 64 : nj - s0;
    size_t i = 0;
    for (; i + 2 <= M; i += 2) {
      v8f acc0[8], acc1[8];
      for (int v = 0; v < 8; ++v) { acc0[v] = (v8f){0}; acc1[v] = (v8f){0}; }
      const float *a0 = x->a + i * K, *a1 = a0 + K;
      for (size_t p = 0; p < K; ++p) {
        const v8f *w = (const v8f *)(wt + p * 256 + s0);
        v8f b0 = (v8f){0} + a0[p], b1 = (v8f){0} + a1[p];
        for (int v = 0; v < 8; ++v) {
          v8f t0 = b0 * w[v];
          v8f t1 = b1 * w[v];
          acc0[v] = acc0[v] + t0;
          acc1[v] = acc1[v] + t1;
        }
      }
      float *c0 = x->c + i * N + j0 + s0, *c1 = c0 + N;
      for (size_t j = 0; j < sn; ++j) { c0[j] = acc0[j / 8][j % 8]; c1[j] = acc1[j / 8][j % 8]; }
    }
    for (; i < M; ++i) {
      v8f acc0[8];
      for (int v = 0; v < 8; ++v) acc0[v] = (v8f){0};
      const float *a0 = x->a + i * K;
      for (size_t p = 0; p < K; ++p) {
        const v8f *w = (const v8f *)(wt + p * 256 + s0);
        v8f b0 = (v8f){0} + a0[p];
        for (int v = 0; v < 8; ++v) { v8f t0 = b0 * w[v]; acc0[v] = acc0[v] + t0; }
      }
      float *c0 = x->c + i * N + j0 + s0;
      for (size_t j = 0; j < sn; ++j) c0[j] = acc0[j / 8][j % 8];
    }
  }
  free(wt);
}

static void or__mm_wide(const or_model *m, mm_ctx *x) {
  wide_ctx w = {x};
  parallel_for(m->threads, (x->n + 255) / 256, mm_wide_task, &w);
}

/* tied output head: logits[j] = sum_p xf[p] * E[j][p] (transpose_2d,
 * src/model.rs:531-539, then matmul) */
typedef struct { const or_model *m; const float *xf; size_t M; float *out; } tied_ctx;
static void tied_task(void *vctx, size_t task) {
  tied_ctx *x = (tied_ctx *)vctx;
  size_t d = x->m->cfg.n_embd, V = x->m->cfg.vocab_size;
  size_t j0 = task * 64, j1 = j0 + 64 < V ? j0 + 64 : V;
  float *row = (float *)malloc(d * sizeof(float));
  for (size_t j = j0; j < j1; ++j) {
    tensor_slice(&x->m->embd, j * d, d, row);
    for (size_t i = 0; i < x->M; ++i) {
      float s = 0.0f;
      for (size_t p = 0; p < d; ++p) s += x->xf[i * d + p] * row[p];
      x->out[i * V + j] = s;
    }
  }
  free(row);
}

/* ------------------------------------------------------------------------ */
/* KV cache, src/kv_cache.rs:13-110 (preallocated rows; same contents)       */
/* ------------------------------------------------------------------------ */
struct or_kv {
  size_t n_layers, kvd, max_ctx, len;
  int f16;
  float **k, **v;
};

or_kv *or_kv_new(const or_model *m, size_t max_ctx, int kv_f16) {
  or_kv *kv = (or_kv *)calloc(1, sizeof *kv);
  kv->n_layers = m->cfg.n_layers;
  kv->kvd = m->cfg.n_kv_heads * m->cfg.head_dim;
  kv->max_ctx = max_ctx;
  kv->f16 = kv_f16;
  kv->k = (float **)calloc(kv->n_layers, sizeof(float *));
  kv->v = (float **)calloc(kv->n_layers, sizeof(float *));
  for (size_t l = 0; l < kv->n_layers; ++l) {
    kv->k[l] = (float *)malloc(max_ctx * kv->kvd * sizeof(float));
    kv->v[l] = (float *)malloc(max_ctx * kv->kvd * sizeof(float));
  }
  return kv;
}
void or_kv_free(or_kv *kv) {
  if (!kv) return;
  for (size_t l = 0; l < kv->n_layers; ++l) { free(kv->k[l]); free(kv->v[l]); }
  free(kv->k); free(kv->v); free(kv);
}
void or_kv_clear(or_kv *kv) { kv->len = 0; }
size_t or_kv_len(const or_kv *kv) { return kv->len; }
int or_kv_get(const or_kv *kv, size_t layer, float *k, float *v) {
  if (layer >= kv->n_layers) return -1; /* reference panics, src/kv_cache.rs:66-69 */
  memcpy(k, kv->k[layer], kv->len * kv->kvd * sizeof(float));
  memcpy(v, kv->v[layer], kv->len * kv->kvd * sizeof(float));
  return 0;
}
int or_kv_set(or_kv *kv, size_t layer, const float *k, const float *v, size_t len) {
  if (layer >= kv->n_layers || len > kv->max_ctx) return -1;
  memcpy(kv->k[layer], k, len * kv->kvd * sizeof(float));
  memcpy(kv->v[layer], v, len * kv->kvd * sizeof(float));
  kv->len = len;
  return 0;
}
static float kv_round(const or_kv *kv, float x) { return kv->f16 ? or_f16_to_f32(or_f32_to_f16(x)) : x; }

/* ------------------------------------------------------------------------ */
/* forward, src/model.rs:316-455                                             */
/* ------------------------------------------------------------------------ */
typedef struct {
  const or_model *m; const float *q; const or_kv *kv; size_t layer;
  size_t n; size_t base; int causal; float *out;
} attn_ctx;

/* one query head over all its keys; task = token*n_heads + head.  The dot
 * products, softmax and weighted sum follow src/tensor.rs:496-545. */
static void attn_task(void *vctx, size_t task) {
  attn_ctx *x = (attn_ctx *)vctx;
  const or_config *c = &x->m->cfg;
  size_t H = c->n_heads, hd = c->head_dim, kvd = x->kv->kvd;
  size_t t = task / H, h = task % H;
  size_t kh = h / (H / c->n_kv_heads);
  size_t T = x->causal ? x->base + t + 1 : x->base + x->n;
  const float *K = x->kv->k[x->layer], *V = x->kv->v[x->layer];
  const float *qv = x->q + t * H * hd + h * hd;
  float *sc = (float *)malloc(T * sizeof(float));
  float scale = 1.0f / sqrtf((float)hd);
  float mx = -INFINITY;
  for (size_t ki = 0; ki < T; ++ki) {
    const float *kr = K + ki * kvd + kh * hd;
    float dot = 0.0f;
    for (size_t d = 0; d < hd; ++d) dot += qv[d] * kr[d];
    sc[ki] = dot * scale;
    if (sc[ki] > mx) mx = sc[ki];
  }
  float es = 0.0f;
  for (size_t ki = 0; ki < T; ++ki) { sc[ki] = expf(sc[ki] - mx); es += sc[ki]; }
  float inv = 1.0f / es;
  for (size_t ki = 0; ki < T; ++ki) sc[ki] *= inv;
  float *o = x->out + t * H * hd + h * hd;
  float acc[512];
  for (size_t d = 0; d < hd; ++d) acc[d] = 0.0f;
  for (size_t ki = 0; ki < T; ++ki) {
    const float *vr = V + ki * kvd + kh * hd;
    float p = sc[ki];
    for (size_t d = 0; d < hd; ++d) { float pr = p * vr[d]; acc[d] = acc[d] + pr; }
  }
  for (size_t d = 0; d < hd; ++d) o[d] = acc[d];
  free(sc);
}

static void embed_rows(const or_model *m, const uint32_t *tokens, size_t n, float *x) {
  size_t d = m->cfg.n_embd;
  for (size_t b = 0; b < n; ++b) tensor_slice(&m->embd, (size_t)tokens[b] * d, d, x + b * d);
}

static void rope_rows(float *data, size_t rows, size_t n_h, size_t hd, const size_t *pos, float base) {
  for (size_t r = 0; r < rows; ++r) or_apply_rope_to_tensor(data + r * n_h * hd, n_h * hd, n_h, hd, pos[r], base);
}

/* shared body: causal=0 is the reference forward (all rows at pos, attend to
 * the whole cache), causal=1 gives row t position pos+t and a prefix mask. */
static int forward_impl(or_model *m, const uint32_t *tokens, size_t n, size_t pos, or_kv *kv,
                        float *logits, float *hidden, int algo, int causal, int last_only) {
  const or_config *c = &m->cfg;
  size_t d = c->n_embd, H = c->n_heads, KVH = c->n_kv_heads, hd = c->head_dim;
  size_t qd = H * hd, kvd = KVH * hd, F = c->n_ff_used, V = c->vocab_size;
  if (!n) return -1;
  for (size_t i = 0; i < n; ++i)
    if (tokens[i] >= V) return -2;
  if (kv->len + n > kv->max_ctx) return -3;
  if (H % KVH) return -4;
  float *x = (float *)calloc(n * d, sizeof(float));
  float *xn = (float *)malloc(n * d * sizeof(float));
  float *q = (float *)malloc(n * qd * sizeof(float));
  float *k = (float *)malloc(n * kvd * sizeof(float));
  float *v = (float *)malloc(n * kvd * sizeof(float));
  float *att = (float *)malloc(n * qd * sizeof(float));
  float *proj = (float *)malloc(n * d * sizeof(float));
  float *g = (float *)malloc(n * F * sizeof(float));
  float *u = (float *)malloc(n * F * sizeof(float));
  size_t *rp = (size_t *)malloc(n * sizeof(size_t));
  for (size_t t = 0; t < n; ++t) rp[t] = causal ? pos + t : pos;
  embed_rows(m, tokens, n, x);
  size_t base = kv->len;
  for (size_t l = 0; l < c->n_layers; ++l) {
    const or_tensor *L = &m->layers[l * T_PER_LAYER];
    float *w1 = (float *)malloc(d * sizeof(float));
    tensor_slice(&L[T_NORM1], 0, d, w1);
    for (size_t b = 0; b < n; ++b) or_rms_norm(x + b * d, w1, d, c->norm_eps, xn + b * d);
    wmatmul(m, xn, &L[T_Q], n, d, qd, q, algo);
    wmatmul(m, xn, &L[T_K], n, d, kvd, k, algo);
    wmatmul(m, xn, &L[T_V], n, d, kvd, v, algo);
    rope_rows(q, n, H, hd, rp, c->rope_base);
    rope_rows(k, n, KVH, hd, rp, c->rope_base);
    for (size_t b = 0; b < n; ++b)
      for (size_t j = 0; j < kvd; ++j) {
        kv->k[l][(base + b) * kvd + j] = kv_round(kv, k[b * kvd + j]);
        kv->v[l][(base + b) * kvd + j] = kv_round(kv, v[b * kvd + j]);
      }
    attn_ctx ac = {m, q, kv, l, n, base, causal, att};
    parallel_for(algo ? m->threads : 1, n * H, attn_task, &ac);
    wmatmul(m, att, &L[T_O], n, qd, d, proj, algo);
    for (size_t i = 0; i < n * d; ++i) x[i] = x[i] + proj[i];
    tensor_slice(&L[T_NORM2], 0, d, w1);
    for (size_t b = 0; b < n; ++b) or_rms_norm(x + b * d, w1, d, c->norm_eps, xn + b * d);
    free(w1);
    wmatmul(m, xn, &L[T_GATE], n, d, F, g, algo);
    for (size_t i = 0; i < n * F; ++i) g[i] = g[i] * sigmoidf_ref(g[i]);
    wmatmul(m, xn, &L[T_UP], n, d, F, u, algo);
    for (size_t i = 0; i < n * F; ++i) g[i] = g[i] * u[i];
    wmatmul(m, g, &L[T_DOWN], n, F, d, proj, algo);
    for (size_t i = 0; i < n * d; ++i) x[i] = x[i] + proj[i];
    if (hidden) memcpy(hidden + l * n * d, x, n * d * sizeof(float));
  }
  kv->len = base + n;
  if (logits) {
    float *wn = (float *)malloc(d * sizeof(float));
    tensor_slice(&m->out_norm, 0, d, wn);
    size_t r0 = last_only ? n - 1 : 0, rows = n - r0;
    for (size_t b = 0; b < rows; ++b) or_rms_norm(x + (r0 + b) * d, wn, d, c->norm_eps, xn + b * d);
    free(wn);
    if (!c->tied_output) {
      wmatmul(m, xn, &m->out, rows, d, V, logits, algo);
    } else {
      tied_ctx tc = {m, xn, rows, logits};
      parallel_for(algo ? m->threads : 1, (V + 63) / 64, tied_task, &tc);
    }
  }
  free(x); free(xn); free(q); free(k); free(v); free(att); free(proj); free(g); free(u); free(rp);
  return 0;
}

int or_forward(or_model *m, const uint32_t *tokens, size_t n, size_t pos, or_kv *kv,
               float *logits, float *hidden, int algo) {
  return forward_impl(m, tokens, n, pos, kv, logits, hidden, algo, 0, 0);
}

int or_prefill(or_model *m, const uint32_t *tokens, size_t n, size_t pos0, or_kv *kv,
               float *last_logits, float *hidden) {
  return forward_impl(m, tokens, n, pos0, kv, last_logits, hidden, 1, 1, 1);
}

/* CPU-baseline sample: the matmuls of one layer in the reference's i-j-p
 * order (src/tensor.rs:244-258) on f32 weights dequantised beforehand (the
 * reference dequantises at load, src/model.rs:252-298).  Returns seconds
 * spent in the matmuls for one token; *macs = multiply-adds performed. */
double or_time_layer(or_model *m, size_t layer, double *macs) {
  const or_config *c = &m->cfg;
  size_t d = c->n_embd, qd = c->n_heads * c->head_dim, kvd = c->n_kv_heads * c->head_dim, F = c->n_ff_used;
  const or_tensor *L = &m->layers[layer * T_PER_LAYER];
  const int ids[7] = {T_Q, T_K, T_V, T_O, T_GATE, T_UP, T_DOWN};
  const size_t Ks[7] = {d, d, d, qd, d, d, F}, Ns[7] = {qd, kvd, kvd, d, F, F, d};
  float *w[7];
  for (int i = 0; i < 7; ++i) {
    w[i] = (float *)malloc(Ks[i] * Ns[i] * sizeof(float));
    tensor_slice(&L[ids[i]], 0, Ks[i] * Ns[i], w[i]);
  }
  float *x = (float *)malloc(F * sizeof(float)), *y = (float *)malloc((F > qd ? F : qd) * sizeof(float));
  for (size_t i = 0; i < F; ++i) x[i] = 0.01f * (float)((i * 37) % 101) - 0.5f;
  struct timespec t0, t1;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  *macs = 0.0;
  for (int i = 0; i < 7; ++i) {
    or_matmul(x, w[i], 1, Ks[i], Ns[i], y);
    *macs += (double)Ks[i] * Ns[i];
  }
  clock_gettime(CLOCK_MONOTONIC, &t1);
  for (int i = 0; i < 7; ++i) free(w[i]);
  free(x);
  free(y);
  return (double)(t1.tv_sec - t0.tv_sec) + 1e-9 * (double)(t1.tv_nsec - t0.tv_nsec);
}

/* ---- whole-token timing in the reference's order (CPU baseline) ---- */
static double now_s(void) {
  struct timespec t;
  clock_gettime(CLOCK_MONOTONIC, &t);
  return (double)t.tv_sec + 1e-9 * (double)t.tv_nsec;
}

typedef struct { const or_tensor *t; size_t n, chunk; float *out; } dq_ctx;
static void dq_task(void *vctx, size_t task) {
  dq_ctx *x = (dq_ctx *)vctx;
  size_t e0 = task * x->chunk, n = e0 + x->chunk <= x->n ? x->chunk : x->n - e0;
  tensor_slice(x->t, e0, n, x->out + e0);
}
/* the reference holds every weight as f32 after load (src/model.rs:252-298):
 * this rebuilds that copy of one tensor, with all threads, outside the timed
 * region */
static float *dequant_all(const or_model *m, const or_tensor *t, size_t n) {
  float *w = (float *)malloc(n * sizeof(float));
  dq_ctx x = {t, n, (size_t)256 * 4096, w};
  parallel_for(m->threads, (n + x.chunk - 1) / x.chunk, dq_task, &x);
  return w;
}

void or_kv_fill_synthetic(or_kv *kv, size_t len, uint64_t seed) {
  if (len > kv->max_ctx) len = kv->max_ctx;
  uint64_t s = seed * 6364136223846793005ull + 1442695040888963407ull;
  for (size_t l = 0; l < kv->n_layers; ++l)
    for (size_t i = 0; i < len * kv->kvd; ++i) {
      s = s * 6364136223846793005ull + 1442695040888963407ull;
      kv->k[l][i] = (float)((s >> 40) & 0xFFFF) * (1.0f / 65536.0f) - 0.5f;
      kv->v[l][i] = (float)((s >> 24) & 0xFFFF) * (1.0f / 65536.0f) - 0.5f;
    }
  kv->len = len;
}

/* One decode token through ModelWeights::forward in the reference's order and
 * data movement (src/model.rs:316-455): per layer rms_norm, the q/k/v
 * matmuls (i-j-p, src/tensor.rs:244-258), RoPE on q and k with the table
 * rebuilt per call (src/model.rs:469-491), the cache append, expand_kv_heads
 * copying the whole cache to n_heads heads (src/model.rs:500-526), attention
 * over the expanded rows (src/tensor.rs:451-551), the o matmul and residual,
 * rms_norm, gate/up matmuls, SiLU, product, down matmul and residual; then the
 * output norm, the head matmul and the greedy pick (softmax + first argmax,
 * src/sampling.rs:110-152).  Only the first n_layers_timed layers run (all
 * when 0).  Weights are dequantised to f32 before each matmul outside the
 * timed region (the reference does that once at load).  One thread for all
 * timed work.  out[0] = seconds in the layers, out[1] = seconds in the head
 * and the pick.  Returns the picked id, or -1 when the cache is full. */
long or_time_token(or_model *m, or_kv *kv, uint32_t token, size_t pos, size_t n_layers_timed, double out[2]) {
  const or_config *c = &m->cfg;
  const size_t d = c->n_embd, H = c->n_heads, KVH = c->n_kv_heads, hd = c->head_dim;
  const size_t qd = H * hd, kvd = KVH * hd, F = c->n_ff_used, V = c->vocab_size, rep = H / KVH;
  if (kv->len + 1 > kv->max_ctx || token >= V) return -1;
  const size_t NL = n_layers_timed && n_layers_timed < c->n_layers ? n_layers_timed : c->n_layers;
  const size_t T = kv->len + 1;
  float *x = (float *)malloc(d * sizeof(float)), *xn = (float *)malloc(d * sizeof(float));
  float *q = (float *)malloc(qd * sizeof(float)), *k = (float *)malloc(kvd * sizeof(float));
  float *v = (float *)malloc(kvd * sizeof(float)), *att = (float *)malloc(qd * sizeof(float));
  float *proj = (float *)malloc(d * sizeof(float)), *g = (float *)malloc(F * sizeof(float));
  float *u = (float *)malloc(F * sizeof(float)), *sc = (float *)malloc(T * sizeof(float));
  float *ek = (float *)malloc(T * qd * sizeof(float)), *ev = (float *)malloc(T * qd * sizeof(float));
  float *wn = (float *)malloc(d * sizeof(float));
  double t_layers = 0.0, t0;
  tensor_slice(&m->embd, (size_t)token * d, d, x);
  for (size_t l = 0; l < NL; ++l) {
    const or_tensor *L = &m->layers[l * T_PER_LAYER];
    float *w1 = dequant_all(m, &L[T_NORM1], d), *w2 = dequant_all(m, &L[T_NORM2], d);
    float *wq = dequant_all(m, &L[T_Q], d * qd), *wk = dequant_all(m, &L[T_K], d * kvd);
    float *wv = dequant_all(m, &L[T_V], d * kvd), *wo = dequant_all(m, &L[T_O], qd * d);
    t0 = now_s();
    or_rms_norm(x, w1, d, c->norm_eps, xn);
    or_matmul(xn, wq, 1, d, qd, q);
    or_matmul(xn, wk, 1, d, kvd, k);
    or_matmul(xn, wv, 1, d, kvd, v);
    or_apply_rope_to_tensor(q, qd, H, hd, pos, c->rope_base);
    or_apply_rope_to_tensor(k, kvd, KVH, hd, pos, c->rope_base);
    memcpy(kv->k[l] + kv->len * kvd, k, kvd * sizeof(float));
    memcpy(kv->v[l] + kv->len * kvd, v, kvd * sizeof(float));
    for (size_t s = 0; s < T; ++s)
      for (size_t h = 0; h < KVH; ++h)
        for (size_t r = 0; r < rep; ++r) {
          memcpy(ek + s * qd + (h * rep + r) * hd, kv->k[l] + s * kvd + h * hd, hd * sizeof(float));
          memcpy(ev + s * qd + (h * rep + r) * hd, kv->v[l] + s * kvd + h * hd, hd * sizeof(float));
        }
    sdpa_gqa(q, ek, ev, 1, T, H, H, hd, att, sc);
    or_matmul(att, wo, 1, qd, d, proj);
    for (size_t i = 0; i < d; ++i) x[i] = x[i] + proj[i];
    t_layers += now_s() - t0;
    free(wq); free(wk); free(wv); free(wo);
    float *wg = dequant_all(m, &L[T_GATE], d * F), *wu = dequant_all(m, &L[T_UP], d * F);
    t0 = now_s();
    or_rms_norm(x, w2, d, c->norm_eps, xn);
    or_matmul(xn, wg, 1, d, F, g);
    or_silu(g, F, g);
    or_matmul(xn, wu, 1, d, F, u);
    for (size_t i = 0; i < F; ++i) g[i] = g[i] * u[i];
    t_layers += now_s() - t0;
    free(wg); free(wu);
    float *wd = dequant_all(m, &L[T_DOWN], F * d);
    t0 = now_s();
    or_matmul(g, wd, 1, F, d, proj);
    for (size_t i = 0; i < d; ++i) x[i] = x[i] + proj[i];
    t_layers += now_s() - t0;
    free(wd); free(w1); free(w2);
  }
  kv->len += 1;
  float *wo_n = dequant_all(m, &m->out_norm, d);
  float *wh = c->tied_output ? NULL : dequant_all(m, &m->out, d * V);
  float *logits = (float *)malloc(V * sizeof(float)), *probs = (float *)malloc(V * sizeof(float));
  t0 = now_s();
  or_rms_norm(x, wo_n, d, c->norm_eps, wn);
  if (wh) {
    or_matmul(wn, wh, 1, d, V, logits);
  } else {
    for (size_t j = 0; j < V; ++j) logits[j] = 0.0f;
    tied_ctx tc = {m, wn, 1, logits};
    parallel_for(1, (V + 63) / 64, tied_task, &tc);
  }
  or_softmax_probs(logits, V, probs);
  const long id = (long)or_argmax(probs, V);
  out[1] = now_s() - t0;
  out[0] = t_layers;
  free(wo_n); free(wh); free(logits); free(probs);
  free(x); free(xn); free(q); free(k); free(v); free(att); free(proj); free(g); free(u); free(sc);
  free(ek); free(ev); free(wn);
  return id;
}


/* ------------------------------------------------------------------------ */
/* sampler, src/sampling.rs:95-310                                           */
/* ------------------------------------------------------------------------ */
struct or_sampler {
  or_sampler_cfg cfg;
  size_t *freq; unsigned char *present; size_t cap;
};

or_sampler *or_sampler_new(const or_sampler_cfg *cfg) {
  or_sampler *s = (or_sampler *)calloc(1, sizeof *s);
  s->cfg = *cfg;
  return s;
}
void or_sampler_free(or_sampler *s) { if (s) { free(s->freq); free(s->present); free(s); } }

static void ensure_cap(or_sampler *s, size_t n) {  /* src/sampling.rs:167-172 */
  if (s->cap >= n) return;
  s->freq = (size_t *)realloc(s->freq, n * sizeof(size_t));
  s->present = (unsigned char *)realloc(s->present, n);
  memset(s->freq + s->cap, 0, (n - s->cap) * sizeof(size_t));
  memset(s->present + s->cap, 0, n - s->cap);
  s->cap = n;
}
void or_sampler_observe(or_sampler *s, size_t tok) {  /* src/sampling.rs:155-159 */
  ensure_cap(s, tok + 1);
  s->freq[tok] += 1;
  s->present[tok] = 1;
}
void or_sampler_reset(or_sampler *s) { s->cap = 0; free(s->freq); free(s->present); s->freq = NULL; s->present = NULL; }
size_t or_sampler_freq(const or_sampler *s, size_t tok) { return tok < s->cap ? s->freq[tok] : 0; }

/* softmax, src/sampling.rs:222-231: max fold, exp, sequential sum, e/sum */
void or_softmax_probs(const float *logits, size_t n, float *out) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = fmaxf(mx, logits[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) { out[i] = expf(logits[i] - mx); }
  for (size_t i = 0; i < n; ++i) sum += out[i];
  if (sum == 0.0f) return;
  for (size_t i = 0; i < n; ++i) out[i] = out[i] / sum;
}

/* stable descending sort by probability == sort by (p desc, index asc)
 * (sort_by with partial_cmp; NaN inputs are out of scope) */
typedef struct { size_t i; float p; } ip_t;
static int ip_cmp(const void *a, const void *b) {
  const ip_t *x = (const ip_t *)a, *y = (const ip_t *)b;
  if (x->p > y->p) return -1;
  if (x->p < y->p) return 1;
  return x->i < y->i ? -1 : (x->i > y->i ? 1 : 0);
}

/* top_k_filter, src/sampling.rs:234-248 */
void or_top_k_filter(const float *probs, size_t n, size_t k, float *out) {
  if (k == 0) { memcpy(out, probs, n * sizeof(float)); return; }
  ip_t *ix = (ip_t *)malloc(n * sizeof(ip_t));
  for (size_t i = 0; i < n; ++i) { ix[i].i = i; ix[i].p = probs[i]; }
  qsort(ix, n, sizeof(ip_t), ip_cmp);
  for (size_t i = 0; i < n; ++i) out[i] = 0.0f;
  for (size_t r = 0; r < n && r < k; ++r) out[ix[r].i] = probs[ix[r].i];
  free(ix);
}

/* top_p_filter, src/sampling.rs:251-280 (fixed 0.999 cut, not renormalised) */
void or_top_p_filter(float *probs, size_t n) {
  float total = 0.0f;
  for (size_t i = 0; i < n; ++i) total += probs[i];
  if (total <= 0.0f) return;
  ip_t *ix = (ip_t *)malloc(n * sizeof(ip_t));
  for (size_t i = 0; i < n; ++i) { ix[i].i = i; ix[i].p = probs[i]; }
  qsort(ix, n, sizeof(ip_t), ip_cmp);
  unsigned char *zero = (unsigned char *)calloc(n, 1);
  unsigned char *top = (unsigned char *)calloc(n, 1);
  float cum = 0.0f;
  for (size_t r = 0; r < n; ++r) {
    cum += ix[r].p / total;
    if (cum > 0.999f) zero[ix[r].i] = 1;
  }
  for (size_t r = 0; r < n && ix[r].p > 0.0f; ++r) top[ix[r].i] = 1;
  for (size_t i = 0; i < n; ++i)
    if (zero[i] || !top[i]) probs[i] = 0.0f;
  free(ix); free(zero); free(top);
}

/* categorical_sample, src/sampling.rs:283-294 with the uniform supplied (D4) */
size_t or_categorical_sample(const float *probs, size_t n, float r) {
  for (size_t i = 0; i < n; ++i) {
    r -= probs[i];
    if (r <= 0.0f) return i;
  }
  return or_argmax(probs, n);
}

/* argmax, src/sampling.rs:297-310: first index of the maximum */
size_t or_argmax(const float *v, size_t n) {
  if (!n) return 0;
  size_t bi = 0;
  float bv = v[0];
  for (size_t i = 1; i < n; ++i)
    if (v[i] > bv) { bv = v[i]; bi = i; }
  return bi;
}

/* Sampler::sample, src/sampling.rs:110-152 */
size_t or_sampler_sample(or_sampler *s, const float *logits, size_t n, float r, int *used_r) {
  ensure_cap(s, n);
  float *adj = (float *)malloc((n ? n : 1) * sizeof(float));
  float pen = s->cfg.repetition_penalty;
  for (size_t i = 0; i < n; ++i) {
    float l = logits[i];
    if (!(pen == 1.0f) && i < s->cap && s->present[i]) l = l > 0.0f ? l / pen : l * pen;
    adj[i] = l;
  }
  float fp = s->cfg.frequency_penalty, pp = s->cfg.presence_penalty;
  if (!(fp == 0.0f && pp == 0.0f))
    for (size_t i = 0; i < n && i < s->cap; ++i)
      if (s->freq[i] > 0) { adj[i] -= fp * (float)s->freq[i]; adj[i] -= pp; }
  float T = s->cfg.temperature;
  if (T > 0.0f && T != 1.0f)
    for (size_t i = 0; i < n; ++i) adj[i] /= T;
  float *probs = (float *)malloc((n ? n : 1) * sizeof(float));
  or_softmax_probs(adj, n, probs);
  float *filt = adj; /* reuse */
  if (s->cfg.top_k > 0 && s->cfg.top_k < n) or_top_k_filter(probs, n, s->cfg.top_k, filt);
  else memcpy(filt, probs, n * sizeof(float));
  if (s->cfg.top_p > 0.0f && s->cfg.top_p < 1.0f) or_top_p_filter(filt, n);
  int all_zero = 1;
  for (size_t i = 0; i < n; ++i) if (filt[i] > 0.0f) { all_zero = 0; break; }
  size_t tok;
  if (T == 0.0f || all_zero) { tok = or_argmax(filt, n); if (used_r) *used_r = 0; }
  else { tok = or_categorical_sample(filt, n, r); if (used_r) *used_r = 1; }
  free(adj); free(probs);
  return tok;
}

/* ------------------------------------------------------------------------ */
/* GenerationState::generate / generate_step, src/model.rs:638-705           */
/* ------------------------------------------------------------------------ */
long or_generate(or_model *m, const or_gen_cfg *cfg, const uint32_t *prompt, size_t n_prompt,
                 uint32_t *out, size_t cap, int kv_f16) {
  if (n_prompt == 0) return -1; /* token_ids.last().unwrap() panics in the reference */
  size_t max_ctx = n_prompt + cfg->max_tokens + 1;
  or_kv *kv = or_kv_new(m, max_ctx, kv_f16);
  or_sampler_cfg sc = {cfg->temperature, cfg->top_k, cfg->top_p, cfg->repetition_penalty, 0.0f, 0.0f};
  or_sampler *s = or_sampler_new(&sc);
  size_t V = m->cfg.vocab_size;
  float *logits = (float *)malloc(V * sizeof(float));
  size_t pos = 0, n_ids = 0, n_out = 0;
  uint32_t last = 0;
  int algo = cfg->fast ? 1 : 0;
  if (cfg->fast) {
    if (or_prefill(m, prompt, n_prompt, 0, kv, NULL, NULL)) goto err;
    pos = n_prompt;
  } else {
    for (size_t i = 0; i < n_prompt; ++i) {
      if (or_forward(m, &prompt[i], 1, pos, kv, logits, NULL, 0)) goto err;
      ++pos;
    }
  }
  n_ids = n_prompt;
  last = prompt[n_prompt - 1];
  uint64_t step = 0;
  for (size_t it = 0; it < cfg->max_tokens; ++it) {
    /* generate_step */
    if (n_ids >= cfg->max_tokens) break;
    if (or_forward(m, &last, 1, pos, kv, logits, NULL, algo)) goto err;
    float r = or_philox_uniform(cfg->seed, step);
    int used = 0;
    size_t tok = or_sampler_sample(s, logits, V, r, &used);
    ++step;
    or_sampler_observe(s, tok);
    ++n_ids;
    ++pos;
    last = (uint32_t)tok;
    int stop = 0;
    for (size_t j = 0; j < cfg->n_stop; ++j) if (cfg->stop_ids[j] == last) stop = 1;
    if (stop) break;
    if (n_out < cap) out[n_out] = last;
    ++n_out;
  }
  free(logits); or_sampler_free(s); or_kv_free(kv);
  return (long)n_out;
err:
  free(logits); or_sampler_free(s); or_kv_free(kv);
  return -1;
}
