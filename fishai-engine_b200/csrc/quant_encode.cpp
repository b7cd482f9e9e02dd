#include "quant_encode.hpp"

#include <algorithm>
#include <cmath>
#include <cstring>

#include "fa_host.hpp"

namespace fa {

namespace {

inline void put16(uint8_t *p, uint16_t v) {
  p[0] = (uint8_t)v;
  p[1] = (uint8_t)(v >> 8);
}

inline int sat_int(float v, int lo, int hi) {
  if (v != v) return 0;
  if (v <= (float)lo) return lo;
  if (v >= (float)hi) return hi;
  return (int)v;
}

// src/quant.rs:433-471
void q8_0_block(const float *x, uint8_t *o) {
  float amax = 0.0f;
  for (int i = 0; i < 32; ++i) amax = std::fmax(amax, std::fabs(x[i]));
  float d = amax == 0.0f ? 1.0f : amax / 127.0f;
  put16(o, f32_to_f16(d));
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  for (int i = 0; i < 32; ++i) {
    int q = sat_int(std::round(x[i] * id), -32768, 32767);
    o[2 + i] = (uint8_t)(int8_t)std::clamp(q, -128, 127);
  }
}

// src/quant.rs:393-431 (element 2j -> high nibble of byte j)
void q4_0_block(const float *x, uint8_t *o) {
  float amax = 0.0f;
  for (int i = 0; i < 32; ++i) amax = std::fmax(amax, std::fabs(x[i]));
  float d = amax == 0.0f ? 1.0f : amax / 8.0f;
  put16(o, f32_to_f16(d));
  float id = d != 0.0f ? 1.0f / d : 0.0f;
  uint8_t nib[32];
  for (int i = 0; i < 32; ++i) nib[i] = (uint8_t)std::clamp(sat_int(std::round(x[i] * id + 8.0f), INT32_MIN, INT32_MAX), 0, 15);
  for (int j = 0; j < 16; ++j) o[2 + j] = (uint8_t)((nib[2 * j] << 4) | nib[2 * j + 1]);
}

// Q4_K: 8 sub-blocks of 32 with an asymmetric range each; 6-bit sub-scales
// and sub-mins relative to f16 super-scales d and dmin.
void q4_k_block(const float *x, uint8_t *o) {
  float scale[8], mn[8];
  float max_scale = 0.0f, max_min = 0.0f;
  for (int j = 0; j < 8; ++j) {
    float lo = 0.0f, hi = -INFINITY;
    for (int l = 0; l < 32; ++l) {
      lo = std::fmin(lo, x[32 * j + l]);
      hi = std::fmax(hi, x[32 * j + l]);
    }
    if (hi < lo) hi = lo;
    scale[j] = (hi - lo) / 15.0f;
    mn[j] = -lo;
    max_scale = std::fmax(max_scale, scale[j]);
    max_min = std::fmax(max_min, mn[j]);
  }
  uint16_t dh = f32_to_f16(max_scale / 63.0f), mh = f32_to_f16(max_min / 63.0f);
  float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
  uint8_t sc[8], m[8];
  for (int j = 0; j < 8; ++j) {
    sc[j] = d > 0.0f ? (uint8_t)std::clamp((int)std::lround(scale[j] / d), 0, 63) : 0;
    m[j] = dmin > 0.0f ? (uint8_t)std::clamp((int)std::lround(mn[j] / dmin), 0, 63) : 0;
  }
  put16(o, dh);
  put16(o + 2, mh);
  uint8_t *s = o + 4;
  for (int j = 0; j < 4; ++j) {
    s[j] = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
    s[j + 4] = (uint8_t)((m[j] & 63) | ((m[j + 4] >> 4) << 6));
    s[j + 8] = (uint8_t)((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
  }
  uint8_t q[256];
  for (int j = 0; j < 8; ++j) {
    float d1 = d * (float)sc[j], m1 = dmin * (float)m[j];
    for (int l = 0; l < 32; ++l) {
      float v = d1 > 0.0f ? (x[32 * j + l] + m1) / d1 : 0.0f;
      q[32 * j + l] = (uint8_t)std::clamp((int)std::lround(v), 0, 15);
    }
  }
  uint8_t *qs = o + 16;
  for (int j = 0; j < 4; ++j)
    for (int l = 0; l < 32; ++l) qs[32 * j + l] = (uint8_t)(q[64 * j + l] | (q[64 * j + 32 + l] << 4));
}

// Q4_1 (value q*d + m, src/quant.rs:163-200): m = block minimum, d = range/15,
// both f16; element 2j in the HIGH nibble of byte j, as the reference reads it
void q4_1_block(const float *x, uint8_t *o) {
  float lo = x[0], hi = x[0];
  for (int i = 1; i < 32; ++i) {
    lo = std::fmin(lo, x[i]);
    hi = std::fmax(hi, x[i]);
  }
  const uint16_t dh = f32_to_f16((hi - lo) / 15.0f), mh = f32_to_f16(lo);
  const float d = f16_to_f32(dh), m = f16_to_f32(mh);
  put16(o, dh);
  put16(o + 2, mh);
  uint8_t q[32];
  for (int i = 0; i < 32; ++i) q[i] = d > 0.0f ? (uint8_t)std::clamp((int)std::lround((x[i] - m) / d), 0, 15) : 0;
  for (int j = 0; j < 16; ++j) o[4 + j] = (uint8_t)((q[2 * j] << 4) | q[2 * j + 1]);
}

// Q5_0 (value (q-16)*d, q = nibble | qh bit << 4, src/quant.rs:205-255):
// d = max|x|/16 as f16; element 2j in the HIGH nibble of byte j, fifth bits
// of elements 0..31 in the little-endian u32 after d
void q5_0_block(const float *x, uint8_t *o) {
  float amax = 0.0f;
  for (int i = 0; i < 32; ++i) amax = std::fmax(amax, std::fabs(x[i]));
  const uint16_t dh = f32_to_f16(amax / 16.0f);
  const float d = f16_to_f32(dh);
  put16(o, dh);
  uint32_t qh = 0;
  uint8_t q[32];
  for (int i = 0; i < 32; ++i) {
    q[i] = d > 0.0f ? (uint8_t)std::clamp((int)std::lround(x[i] / d) + 16, 0, 31) : 16;
    qh |= (uint32_t)(q[i] >> 4) << i;
  }
  for (int b = 0; b < 4; ++b) o[2 + b] = (uint8_t)(qh >> (8 * b));
  for (int j = 0; j < 16; ++j) o[6 + j] = (uint8_t)(((q[2 * j] & 0xF) << 4) | (q[2 * j + 1] & 0xF));
}

// Q6_K: 16 sub-blocks of 16 with a signed int8 scale each relative to an
// f16 super-scale; 6-bit codes stored as 4 low bits (ql) + 2 high bits (qh).
void q6_k_block(const float *x, uint8_t *o) {
  float scale[16], max_scale = 0.0f;
  for (int i = 0; i < 16; ++i) {
    float amax = 0.0f;
    for (int l = 0; l < 16; ++l) amax = std::fmax(amax, std::fabs(x[16 * i + l]));
    scale[i] = amax / 31.0f;
    max_scale = std::fmax(max_scale, scale[i]);
  }
  uint16_t dh = f32_to_f16(max_scale / 127.0f);
  float d = f16_to_f32(dh);
  int8_t sc[16];
  uint8_t q[256];
  for (int i = 0; i < 16; ++i) {
    sc[i] = d > 0.0f ? (int8_t)std::clamp((int)std::lround(scale[i] / d), -128, 127) : 0;
    float ds = d * (float)sc[i];
    for (int l = 0; l < 16; ++l) {
      float v = ds != 0.0f ? x[16 * i + l] / ds : 0.0f;
      q[16 * i + l] = (uint8_t)(std::clamp((int)std::lround(v), -32, 31) + 32);
    }
  }
  uint8_t *ql = o, *qh = o + 128;
  for (int h = 0; h < 2; ++h)
    for (int l = 0; l < 32; ++l) {
      uint8_t q1 = q[128 * h + l], q2 = q[128 * h + l + 32], q3 = q[128 * h + l + 64], q4 = q[128 * h + l + 96];
      ql[64 * h + l] = (uint8_t)((q1 & 0xF) | ((q3 & 0xF) << 4));
      ql[64 * h + l + 32] = (uint8_t)((q2 & 0xF) | ((q4 & 0xF) << 4));
      qh[32 * h + l] = (uint8_t)((q1 >> 4) | ((q2 >> 4) << 2) | ((q3 >> 4) << 4) | ((q4 >> 4) << 6));
    }
  std::memcpy(o + 192, sc, 16);
  put16(o + 208, dh);
}

}  // namespace

size_t quantize_row(int t, const float *x, size_t n, uint8_t *out) {
  size_t be = block_elems(t), bb = block_bytes(t);
  if (!be || n % be) return 0;
  for (size_t b = 0; b < n / be; ++b) {
    const float *xb = x + b * be;
    uint8_t *ob = out + b * bb;
    switch (t) {
      case FA_GGML_F32: std::memcpy(ob, xb, 4); break;
      case FA_GGML_F16: put16(ob, f32_to_f16(*xb)); break;
      case FA_GGML_Q8_0: q8_0_block(xb, ob); break;
      case FA_GGML_Q4_0: q4_0_block(xb, ob); break;
      case FA_GGML_Q4_1: q4_1_block(xb, ob); break;
      case FA_GGML_Q5_0: q5_0_block(xb, ob); break;
      case FA_GGML_Q4_K: q4_k_block(xb, ob); break;
      case FA_GGML_Q6_K: q6_k_block(xb, ob); break;
      default: return 0;
    }
  }
  return n / be * bb;
}

}  // namespace fa
