#include "fa_host.hpp"

#include <cstring>

namespace fa {

static thread_local std::string g_err;

void set_error(const std::string &msg) { g_err = msg; }
const std::string &last_error() { return g_err; }
int fail(int code, const std::string &msg) {
  g_err = msg;
  return code;
}

float f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16, exp = (h >> 10) & 0x1Fu, man = h & 0x3FFu, bits;
  if (exp == 0) {
    if (man == 0) {
      bits = sign;
    } else {
      int e = -1;
      do {
        man <<= 1;
        ++e;
      } while (!(man & 0x400u));
      bits = sign | ((uint32_t)(112 - e) << 23) | ((man & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (man << 13);
  } else {
    bits = sign | ((exp + 112) << 23) | (man << 13);
  }
  float f;
  std::memcpy(&f, &bits, 4);
  return f;
}

uint16_t f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u, exp = (x >> 23) & 0xFFu, man = x & 0x7FFFFFu;
  if (exp == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? (0x200u | (man >> 13)) : 0));
  int e = (int)exp - 112;
  if (e >= 31) return (uint16_t)(sign | 0x7C00u);
  if (e <= 0) {
    if (e < -10) return (uint16_t)sign;
    man |= 0x800000u;
    int shift = 14 - e;
    uint32_t hm = man >> shift, rem = man & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (hm & 1u))) hm++;
    return (uint16_t)(sign | hm);
  }
  uint32_t hm = man >> 13, rem = man & 0x1FFFu, out = sign | ((uint32_t)e << 10) | hm;
  if (rem > 0x1000u || (rem == 0x1000u && (hm & 1u))) out++;
  return (uint16_t)out;
}

size_t block_elems(int t) {
  switch (t) {
    case FA_GGML_F32: case FA_GGML_F16: return 1;
    case FA_GGML_Q4_0: case FA_GGML_Q4_1: case FA_GGML_Q5_0: case FA_GGML_Q8_0: return 32;
    case FA_GGML_Q4_K: case FA_GGML_Q6_K: return 256;
    default: return 0;
  }
}

size_t block_bytes(int t) {
  switch (t) {
    case FA_GGML_F32: return 4;
    case FA_GGML_F16: return 2;
    case FA_GGML_Q4_0: return 18;
    case FA_GGML_Q4_1: return 20;
    case FA_GGML_Q5_0: return 22;
    case FA_GGML_Q8_0: return 34;
    case FA_GGML_Q4_K: return 144;
    case FA_GGML_Q6_K: return 210;
    default: return 0;
  }
}

bool type_known(int t) { return block_elems(t) != 0; }

}  // namespace fa
