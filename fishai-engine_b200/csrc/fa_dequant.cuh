// Native GGML block dequantisation of one element, bit-exact with
// quant::dequantize (src/quant.rs:123-338) and the public K-quant formats.
// All products are exact in f32 (<= 24 significant bits), so the single
// rounding of the final add/sub matches the reference's separate multiply
// and add.
#pragma once
#include <stdint.h>

#include "fa_device.cuh"
#include "fa_layout.hpp"

namespace fa {

__device__ __forceinline__ float ld_h(const uint8_t *p) { return h2f((uint16_t)(p[0] | (p[1] << 8))); }

__device__ __forceinline__ float dequant_native_elem(int type, const uint8_t *data, uint64_t e) {
  switch (type) {
    case kF32: {
      uint32_t b = (uint32_t)data[4 * e] | ((uint32_t)data[4 * e + 1] << 8) | ((uint32_t)data[4 * e + 2] << 16) |
                   ((uint32_t)data[4 * e + 3] << 24);
      return __uint_as_float(b);
    }
    case kF16: return ld_h(data + 2 * e);
    case kQ4_0: {  // src/quant.rs:123-157: element 2j = high nibble
      const uint8_t *b = data + (e / 32) * 18;
      uint32_t i = e % 32;
      uint8_t byte = b[2 + i / 2];
      int nib = (i & 1) ? (byte & 0xF) : (byte >> 4);
      return __fmul_rn((float)(nib - 8), ld_h(b));
    }
    case kQ4_1: {  // src/quant.rs:163-200
      const uint8_t *b = data + (e / 32) * 20;
      uint32_t i = e % 32;
      uint8_t byte = b[4 + i / 2];
      int nib = (i & 1) ? (byte & 0xF) : (byte >> 4);
      return __fadd_rn(__fmul_rn((float)nib, ld_h(b)), ld_h(b + 2));
    }
    case kQ5_0: {  // src/quant.rs:206-255
      const uint8_t *b = data + (e / 32) * 22;
      uint32_t i = e % 32;
      uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
      uint8_t byte = b[6 + i / 2];
      uint32_t lo = (i & 1) ? (byte & 0xF) : (byte >> 4);
      int v = (int)(lo | (((qh >> i) & 1u) << 4)) - 16;
      return __fmul_rn((float)v, ld_h(b));
    }
    case kQ8_0: {  // src/quant.rs:261-290
      const uint8_t *b = data + (e / 32) * 34;
      return __fmul_rn((float)(int8_t)b[2 + e % 32], ld_h(b));
    }
    case kQ4_K: {  // GGUF Q4_K: (d*sc)*q - dmin*m
      const uint8_t *b = data + (e / 256) * 144;
      uint32_t i = e % 256, j = i / 64, l = i % 32, sb = i / 32;
      const uint8_t *q = b + 4;
      int sc, m;
      if (sb < 4) {
        sc = q[sb] & 63;
        m = q[sb + 4] & 63;
      } else {
        sc = (q[sb + 4] & 0xF) | ((q[sb - 4] >> 6) << 4);
        m = (q[sb + 4] >> 4) | ((q[sb] >> 6) << 4);
      }
      uint8_t byte = b[16 + 32 * j + l];
      int nib = (sb & 1) ? (byte >> 4) : (byte & 0xF);
      float d1 = __fmul_rn(ld_h(b), (float)sc), m1 = __fmul_rn(ld_h(b + 2), (float)m);
      return __fsub_rn(__fmul_rn(d1, (float)nib), m1);
    }
    case kQ6_K: {  // GGUF Q6_K: (d*sc)*(q-32)
      const uint8_t *b = data + (e / 256) * 210;
      uint32_t i = e % 256, h = i / 128, lp = i % 128, quad = lp / 32, l = lp % 32;
      const uint8_t *ql = b + 64 * h, *qh = b + 128 + 32 * h;
      uint32_t lo = (quad & 1) ? ql[32 + l] : ql[l];
      lo = (quad >= 2) ? (lo >> 4) : (lo & 0xF);
      uint32_t hi = (qh[l] >> (2 * quad)) & 3u;
      int q = (int)(lo | (hi << 4)) - 32;
      int8_t sc = (int8_t)b[192 + i / 16];
      return __fmul_rn(__fmul_rn(ld_h(b + 208), (float)sc), (float)q);
    }
    default: return 0.0f;
  }
}

}  // namespace fa
