// Dequantisation (bit-exact with quant::dequantize, src/quant.rs:123-338, and
// the public K-quant block formats) and the native -> chunked weight re-layout.
#include <cuda_runtime.h>

#include "fa_dequant.cuh"
#include "fa_device.cuh"
#include "fa_kernels.hpp"
#include "fa_layout.hpp"

namespace fa {

// ---------------------------------------------------------------------------
// native block dequantisation: one thread per output element.  All products
// below are exact in f32 (<= 24 significant bits), so the single rounding of
// the final add/sub matches the reference's separate multiply and add.
// ---------------------------------------------------------------------------
__global__ void k_dequant_native(int type, const uint8_t *__restrict__ data, uint64_t count, float *__restrict__ out) {
  uint64_t e = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; e < count; e += (uint64_t)gridDim.x * blockDim.x) out[e] = dequant_native_elem(type, data, e);
}

int launch_dequant_native(int type, const void *data, uint64_t count, float *out, cudaStream_t st) {
  if (!count) return 0;
  uint64_t blocks = (count + 255) / 256;
  if (blocks > 148 * 64) blocks = 148 * 64;
  k_dequant_native<<<(unsigned)blocks, 256, 0, st>>>(type, (const uint8_t *)data, count, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ---------------------------------------------------------------------------
// native [K][N] -> chunked row groups.  One thread per (row, 32-col lane).
// With src_b != nullptr two tensors of width F (gate and up) are laid out
// as one virtual [K][2F] weight whose chunk c holds gate columns
// [c*CW/2, ...) followed by the same up columns, so one GEMV chunk carries
// both operands of h = silu(gate) * up.
// ---------------------------------------------------------------------------
__global__ void k_repack(int type, const uint8_t *__restrict__ src_a, const uint8_t *__restrict__ src_b, uint32_t K,
                         uint32_t N, uint32_t K8, uint32_t CW, uint8_t *__restrict__ dst, uint64_t dst_off) {
  const uint32_t Nv = src_b ? 2 * N : N;  // virtual width
  const uint32_t lanes_per_row = Nv / 32;
  uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (uint64_t)K8 * lanes_per_row) return;
  uint32_t k = (uint32_t)(t / lanes_per_row), gl = (uint32_t)(t % lanes_per_row);  // global lane
  uint32_t col0 = gl * 32, c = col0 / CW, w = (Nv - c * CW) < CW ? (Nv - c * CW) : CW;
  uint32_t jc = col0 - c * CW, j = jc / 32, grp = k / 8, r = k % 8;
  const uint8_t *src = src_a;
  uint32_t scol = col0;  // source column of this lane's first element
  if (src_b) {
    uint32_t half = w / 2;
    if (jc < half) {
      scol = c * (CW / 2) + jc;
    } else {
      src = src_b;
      scol = c * (CW / 2) + jc - half;
    }
  }
  uint64_t gb = group_bytes(type, w), full_gb = group_bytes(type, CW);
  uint8_t *G = dst + dst_off + (uint64_t)c * (K8 / 8) * full_gb + (uint64_t)grp * gb;
  const bool pad = k >= K;  // rows beyond K are written as zeros (row 0 is read, never used)
  const uint8_t *row = src + (uint64_t)(pad ? 0 : k) * native_row_bytes(type, N);
  switch (type) {
    case kF32:
      for (int i = 0; i < 128; ++i) G[r * 4 * w + 128 * j + i] = pad ? 0 : row[4 * scol + i];
      break;
    case kF16:
      for (int i = 0; i < 64; ++i) G[r * 2 * w + 64 * j + i] = pad ? 0 : row[2 * scol + i];
      break;
    case kQ8_0: {
      const uint8_t *b = row + (scol / 32) * 34;
      for (int i = 0; i < 32; ++i) G[r * w + 32 * j + i] = pad ? 0 : b[2 + i];
      uint8_t *d = G + 8 * w + (r * (w / 32) + j) * 2;
      d[0] = pad ? 0 : b[0];
      d[1] = pad ? 0 : b[1];
      break;
    }
    case kQ4_0: {
      const uint8_t *b = row + (scol / 32) * 18;
      uint8_t nib[32];
      for (int i = 0; i < 16; ++i) {
        nib[2 * i] = b[2 + i] >> 4;  // element 2i: high nibble (src/quant.rs:143-148)
        nib[2 * i + 1] = b[2 + i] & 0xF;
      }
      for (int i = 0; i < 16; ++i) G[r * (w / 2) + 16 * j + i] = pad ? 0 : (uint8_t)(nib[i] | (nib[i + 16] << 4));
      uint8_t *d = G + 4 * w + (r * (w / 32) + j) * 2;
      d[0] = pad ? 0 : b[0];
      d[1] = pad ? 0 : b[1];
      break;
    }
    case kQ4_1:
    case kQ5_0: {
      const uint32_t bb = type == kQ4_1 ? 20 : 22, co = type == kQ4_1 ? 4 : 6;  // block bytes, code offset
      const uint8_t *b = row + (scol / 32) * bb;
      uint8_t nib[32];
      for (int i = 0; i < 16; ++i) {
        nib[2 * i] = b[co + i] >> 4;  // element 2i: high nibble (src/quant.rs:183-188, :228-233)
        nib[2 * i + 1] = b[co + i] & 0xF;
      }
      for (int i = 0; i < 16; ++i) G[r * (w / 2) + 16 * j + i] = pad ? 0 : (uint8_t)(nib[i] | (nib[i + 16] << 4));
      if (type == kQ4_1) {
        uint8_t *d = G + 4 * w + (r * (w / 32) + j) * 2, *m = d + w / 2;
        for (int i = 0; i < 2; ++i) {
          d[i] = pad ? 0 : b[i];
          m[i] = pad ? 0 : b[2 + i];
        }
      } else {
        uint8_t *qh = G + 4 * w + (r * (w / 32) + j) * 4, *d = G + 5 * w + (r * (w / 32) + j) * 2;
        for (int i = 0; i < 4; ++i) qh[i] = pad ? 0 : b[2 + i];
        d[0] = pad ? 0 : b[0];
        d[1] = pad ? 0 : b[1];
      }
      break;
    }
    case kQ4_K: {
      uint32_t s = j / 8, sb = (scol % 256) / 32;  // dest super-block slot, source sub-block
      const uint8_t *b = row + (scol / 256) * 144;
      const uint8_t *qs = b + 16 + 32 * (sb / 2);
      for (int i = 0; i < 16; ++i) {
        uint8_t lo = (sb & 1) ? (qs[i] >> 4) : (qs[i] & 0xF);
        uint8_t hi = (sb & 1) ? (qs[i + 16] >> 4) : (qs[i + 16] & 0xF);
        G[r * (w / 2) + 16 * j + i] = pad ? 0 : (uint8_t)(lo | (hi << 4));
      }
      if (sb == 0) {
        // d, dmin as stored; the 12 scale bytes re-laid as eight 12-bit
        // fields (sc | m << 6), field f at bit 12f (same 12 bytes)
        uint8_t *h = G + 4 * w + (r * (w / 256) + s) * 16;
        for (int i = 0; i < 4; ++i) h[i] = pad ? 0 : b[i];
        uint32_t words[3] = {0, 0, 0};
        for (int f = 0; f < 8; ++f) {
          int sc, m;
          const uint8_t *q = b + 4;
          if (f < 4) {
            sc = q[f] & 63;
            m = q[f + 4] & 63;
          } else {
            sc = (q[f + 4] & 0xF) | ((q[f - 4] >> 6) << 4);
            m = (q[f + 4] >> 4) | ((q[f] >> 6) << 4);
          }
          const uint64_t v = pad ? 0 : (uint64_t)(sc | (m << 6));
          const uint32_t bit = 12 * f, wi = bit / 32, sh = bit % 32;
          words[wi] |= (uint32_t)(v << sh);
          if (sh + 12 > 32) words[wi + 1] |= (uint32_t)(v >> (32 - sh));
        }
        for (int i = 0; i < 12; ++i) h[4 + i] = (uint8_t)(words[i / 4] >> (8 * (i % 4)));
      }
      break;
    }
    case kQ6_K: {
      uint32_t s = j / 8, sb = (scol % 256) / 32;
      const uint8_t *b = row + (scol / 256) * 210;
      uint8_t code[32];
      for (int i = 0; i < 32; ++i) {
        uint32_t e = 32 * sb + i, h = e / 128, lp = e % 128, quad = lp / 32, l = lp % 32;
        const uint8_t *ql = b + 64 * h, *qh = b + 128 + 32 * h;
        uint32_t lo = (quad & 1) ? ql[32 + l] : ql[l];
        lo = (quad >= 2) ? (lo >> 4) : (lo & 0xF);
        code[i] = (uint8_t)(lo | (((qh[l] >> (2 * quad)) & 3u) << 4));
      }
      for (int i = 0; i < 16; ++i)
        G[r * (w / 2) + 16 * j + i] = pad ? 0 : (uint8_t)((code[i] & 0xF) | ((code[i + 16] & 0xF) << 4));
      for (int i = 0; i < 8; ++i)
        G[4 * w + r * (w / 4) + 8 * j + i] =
            pad ? 0
                : (uint8_t)((code[i] >> 4) | ((code[i + 8] >> 4) << 2) | ((code[i + 16] >> 4) << 4) |
                            ((code[i + 24] >> 4) << 6));
      G[6 * w + r * (w / 16) + 2 * j] = pad ? 0 : b[192 + 2 * sb];
      G[6 * w + r * (w / 16) + 2 * j + 1] = pad ? 0 : b[192 + 2 * sb + 1];
      if (sb == 0) {
        uint8_t *d = G + 6 * w + w / 2 + (r * (w / 256) + s) * 2;
        d[0] = pad ? 0 : b[208];
        d[1] = pad ? 0 : b[209];
      }
      break;
    }
  }
}

// ---------------------------------------------------------------------------
// native [K][N] -> MMA tile layout (fa_layout.hpp), K a multiple of 16.
// Virtual columns and gate/up pairing as in k_repack.
// ---------------------------------------------------------------------------
namespace {

// raw code of (row, col): Q4_0 / Q4_K 0..15, Q6_K 0..63, Q8_0 q + 128
__device__ __forceinline__ uint32_t native_code(int type, const uint8_t *row, uint32_t col) {
  switch (type) {
    case kQ4_0: {
      const uint8_t byte = row[(col / 32) * 18 + 2 + (col % 32) / 2];
      return (col & 1) ? (byte & 0xFu) : (byte >> 4);  // element 2j: high nibble (src/quant.rs:143-148)
    }
    case kQ8_0: return row[(col / 32) * 34 + 2 + col % 32] ^ 0x80u;
    case kQ4_K: {
      const uint32_t i = col % 256, sb = i / 32;
      const uint8_t byte = row[(col / 256) * 144 + 16 + 32 * (i / 64) + i % 32];
      return (sb & 1) ? (byte >> 4) : (byte & 0xFu);
    }
    default: {  // Q6_K
      const uint8_t *b = row + (col / 256) * 210;
      const uint32_t i = col % 256, h = i / 128, lp = i % 128, quad = lp / 32, l = lp % 32;
      uint32_t lo = (quad & 1) ? b[64 * h + 32 + l] : b[64 * h + l];
      lo = (quad >= 2) ? (lo >> 4) : (lo & 0xFu);
      return lo | (((b[128 + 32 * h + l] >> (2 * quad)) & 3u) << 4);
    }
  }
}

struct VCol {
  const uint8_t *src;
  uint32_t col;
};
// virtual column -> (tensor, column): chunk c of a paired weight holds gate
// columns [c*CW/2, c*CW/2 + w/2) then the same up columns
__device__ __forceinline__ VCol vcol_map(const uint8_t *a, const uint8_t *b, uint32_t Nv, uint32_t CW, uint32_t v) {
  if (!b) return {a, v};
  const uint32_t c = v / CW, w = min(CW, Nv - c * CW), jc = v - c * CW, half = w / 2;
  return jc < half ? VCol{a, c * (CW / 2) + jc} : VCol{b, c * (CW / 2) + jc - half};
}

__device__ __forceinline__ uint8_t *mma_group_ptr(uint8_t *dst, int type, uint32_t Nv, uint32_t CW, uint32_t G16,
                                                  uint32_t c, uint32_t grp, uint32_t *w) {
  *w = min(CW, Nv - c * CW);
  return dst + (uint64_t)c * G16 * mma_group_bytes(type, CW) + (uint64_t)grp * mma_group_bytes(type, *w);
}

// one thread per (16-row group, 64-column slice, lane): the codes
__global__ void k_repack_mma_codes(int type, const uint8_t *__restrict__ src_a, const uint8_t *__restrict__ src_b,
                                   uint32_t N, uint32_t K, uint32_t CW, uint8_t *__restrict__ dst) {
  const uint32_t Nv = src_b ? 2 * N : N, G16 = K / 16, nsl = (Nv + 63) / 64;
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (uint64_t)G16 * nsl * 32) return;
  const uint32_t l = (uint32_t)(t % 32), si = (uint32_t)((t / 32) % nsl), grp = (uint32_t)(t / 32 / nsl);
  const uint32_t c = si * 64 / CW, i = si - c * (CW / 64);
  uint32_t w;
  uint8_t *G = mma_group_ptr(dst, type, Nv, CW, G16, c, grp, &w);
  const uint32_t nt = min(64u, w - 64 * i) / 16;
  const uint32_t rb = native_row_bytes(type, N);
  uint32_t hw[2] = {0, 0};
  for (uint32_t tt = 0; tt < nt; ++tt) {
    uint32_t word = 0, q8[2] = {0, 0};
    for (uint32_t e = 0; e < 8; ++e) {
      const uint32_t k = 16 * grp + frag_k(l, e), v = 64 * si + 16 * tt + frag_m(l, e);
      const VCol vc = vcol_map(src_a, src_b, Nv, CW, v);
      const uint32_t q = native_code(type, vc.src + (uint64_t)k * rb, vc.col);
      if (type == kQ8_0) {
        const uint32_t by = frag_q8_byte(e);
        q8[by / 4] |= q << (8 * (by % 4));
      } else {
        word |= (q & 0xFu) << frag_q4_bit(e);
        if (type == kQ6_K) hw[tt / 2] |= (q >> 4) << (frag_q4_bit(e) + 2 * (tt & 1));
      }
    }
    if (type == kQ8_0) {
      uint32_t *p = reinterpret_cast<uint32_t *>(G + 1024 * i + 8 * nt * l + 8 * tt);
      p[0] = q8[0];
      p[1] = q8[1];
    } else {
      *reinterpret_cast<uint32_t *>(G + 512 * i + 4 * nt * l + 4 * tt) = word;
    }
  }
  if (type == kQ6_K) {
    uint32_t *p = reinterpret_cast<uint32_t *>(G + 8 * w + 256 * i + 8 * l);
    p[0] = hw[0];
    p[1] = hw[1];
  }
}

// one thread per (row, 16-column unit): scales and block metadata
__global__ void k_repack_mma_meta(int type, const uint8_t *__restrict__ src_a, const uint8_t *__restrict__ src_b,
                                  uint32_t N, uint32_t K, uint32_t CW, uint8_t *__restrict__ dst) {
  const uint32_t Nv = src_b ? 2 * N : N, G16 = K / 16, units = Nv / 16;
  const uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (uint64_t)K * units) return;
  const uint32_t u = (uint32_t)(t % units), k = (uint32_t)(t / units);
  const uint32_t v = 16 * u, c = v / CW, j16 = (v - c * CW) / 16, grp = k / 16, r = k % 16;
  uint32_t w;
  uint8_t *G = mma_group_ptr(dst, type, Nv, CW, G16, c, grp, &w);
  const VCol vc = vcol_map(src_a, src_b, Nv, CW, v);
  const uint8_t *row = vc.src + (uint64_t)k * native_row_bytes(type, N);
  switch (type) {
    case kQ4_K: {
      if (j16 % 16) break;
      const uint8_t *b = row + (vc.col / 256) * 144;
      uint8_t *h = G + 8 * w + (16 * (j16 / 16) + r) * 16;
      for (int x = 0; x < 4; ++x) h[x] = b[x];
      uint32_t words[3] = {0, 0, 0};
      const uint8_t *q = b + 4;
      for (int f = 0; f < 8; ++f) {
        int sc, m;
        if (f < 4) {
          sc = q[f] & 63;
          m = q[f + 4] & 63;
        } else {
          sc = (q[f + 4] & 0xF) | ((q[f - 4] >> 6) << 4);
          m = (q[f + 4] >> 4) | ((q[f] >> 6) << 4);
        }
        const uint64_t val = (uint64_t)(sc | (m << 6));
        const uint32_t bit = 12 * f, wi = bit / 32, sh = bit % 32;
        words[wi] |= (uint32_t)(val << sh);
        if (sh + 12 > 32) words[wi + 1] |= (uint32_t)(val >> (32 - sh));
      }
      for (int x = 0; x < 12; ++x) h[4 + x] = (uint8_t)(words[x / 4] >> (8 * (x % 4)));
      break;
    }
    case kQ6_K: {
      const uint8_t *b = row + (vc.col / 256) * 210;
      G[12 * w + 16 * j16 + r] = b[192 + (vc.col % 256) / 16];
      if (j16 % 16 == 0) {
        uint8_t *d = G + 13 * w + (16 * (j16 / 16) + r) * 2;
        d[0] = b[208];
        d[1] = b[209];
      }
      break;
    }
    default: {  // Q8_0 / Q4_0: f16 d per 32-column block
      if (j16 % 2) break;
      const uint8_t *b = row + (vc.col / 32) * (type == kQ8_0 ? 34 : 18);
      uint8_t *d = G + (type == kQ8_0 ? 16 : 8) * w + (16 * (j16 / 2) + r) * 2;
      d[0] = b[0];
      d[1] = b[1];
      break;
    }
  }
}

}  // namespace

int launch_repack_mma(int type, const void *src_a, const void *src_b, uint32_t K, uint32_t N, uint32_t CW, void *dst,
                      uint64_t dst_off, cudaStream_t st) {
  if (!mma_type(type) || K % 16 || CW % 64) return -1;
  const uint32_t Nv = src_b ? 2 * N : N;
  uint8_t *d = (uint8_t *)dst + dst_off;
  const uint64_t n1 = (uint64_t)(K / 16) * ((Nv + 63) / 64) * 32, n2 = (uint64_t)K * (Nv / 16);
  k_repack_mma_codes<<<(unsigned)((n1 + 255) / 256), 256, 0, st>>>(type, (const uint8_t *)src_a,
                                                                  (const uint8_t *)src_b, N, K, CW, d);
  k_repack_mma_meta<<<(unsigned)((n2 + 255) / 256), 256, 0, st>>>(type, (const uint8_t *)src_a,
                                                                 (const uint8_t *)src_b, N, K, CW, d);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_repack(int type, const void *src_a, const void *src_b, uint32_t K, uint32_t N, uint32_t CW, void *dst,
                  uint64_t dst_off, cudaStream_t st) {
  uint32_t K8 = (K + 7) / 8 * 8;
  uint64_t n = (uint64_t)K8 * ((src_b ? 2 * N : N) / 32);
  k_repack<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(type, (const uint8_t *)src_a, (const uint8_t *)src_b, K, N,
                                                       K8, CW, (uint8_t *)dst, dst_off);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// ---------------------------------------------------------------------------
// chunked row groups -> f32 [K][N]: the decode the GEMV lanes perform,
// written out value by value (used to verify the re-layout bit for bit).
// ---------------------------------------------------------------------------
__global__ void k_unpack(int type, const uint8_t *__restrict__ src, uint64_t src_off, uint32_t K, uint32_t N,
                         uint32_t K8, uint32_t CW, float *__restrict__ out) {
  uint64_t t = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= (uint64_t)K * N) return;
  uint32_t k = (uint32_t)(t / N), n = (uint32_t)(t % N);
  uint32_t c = n / CW, w = (N - c * CW) < CW ? (N - c * CW) : CW, jc = n - c * CW, j = jc / 32, i = jc % 32;
  uint32_t grp = k / 8, r = k % 8;
  const uint8_t *G = src + src_off + (uint64_t)c * (K8 / 8) * group_bytes(type, CW) + (uint64_t)grp * group_bytes(type, w);
  float v = 0.0f;
  switch (type) {
    case kF32: {
      const uint8_t *p = G + r * 4 * w + 128 * j + 4 * i;
      v = __uint_as_float((uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24));
      break;
    }
    case kF16: v = ld_h(G + r * 2 * w + 64 * j + 2 * i); break;
    case kQ8_0: v = __fmul_rn((float)(int8_t)G[r * w + 32 * j + i], ld_h(G + 8 * w + (r * (w / 32) + j) * 2)); break;
    case kQ4_0: {
      uint8_t byte = G[r * (w / 2) + 16 * j + (i % 16)];
      int q = (i < 16) ? (byte & 0xF) : (byte >> 4);
      v = __fmul_rn((float)(q - 8), ld_h(G + 4 * w + (r * (w / 32) + j) * 2));
      break;
    }
    case kQ4_1: {  // nib * d + m, two roundings as in src/quant.rs:190-191
      uint8_t byte = G[r * (w / 2) + 16 * j + (i % 16)];
      int q = (i < 16) ? (byte & 0xF) : (byte >> 4);
      const uint8_t *d = G + 4 * w + (r * (w / 32) + j) * 2;
      v = __fadd_rn(__fmul_rn((float)q, ld_h(d)), ld_h(d + w / 2));
      break;
    }
    case kQ5_0: {  // ((nib | hb << 4) - 16) * d, src/quant.rs:236-240
      uint8_t byte = G[r * (w / 2) + 16 * j + (i % 16)];
      int q = (i < 16) ? (byte & 0xF) : (byte >> 4);
      const uint8_t *qh = G + 4 * w + (r * (w / 32) + j) * 4;
      const uint32_t hw = (uint32_t)qh[0] | ((uint32_t)qh[1] << 8) | ((uint32_t)qh[2] << 16) | ((uint32_t)qh[3] << 24);
      q |= (int)((hw >> i) & 1u) << 4;
      v = __fmul_rn((float)(q - 16), ld_h(G + 5 * w + (r * (w / 32) + j) * 2));
      break;
    }
    case kQ4_K: {
      uint32_t s = j / 8, sb = j % 8;
      const uint8_t *h = G + 4 * w + (r * (w / 256) + s) * 16;
      uint64_t bits = 0;  // 96-bit field block, little endian
      const uint32_t bit = 12 * sb;
      for (int i = 0; i < 8 && (bit / 8 + i) < 12; ++i) bits |= (uint64_t)h[4 + bit / 8 + i] << (8 * i);
      const uint32_t f = (uint32_t)(bits >> (bit % 8)) & 0xFFFu;
      const int sc = (int)(f & 63u), m = (int)(f >> 6);
      uint8_t byte = G[r * (w / 2) + 16 * j + (i % 16)];
      int nib = (i < 16) ? (byte & 0xF) : (byte >> 4);
      float d1 = __fmul_rn(ld_h(h), (float)sc), m1 = __fmul_rn(ld_h(h + 2), (float)m);
      v = __fsub_rn(__fmul_rn(d1, (float)nib), m1);
      break;
    }
    case kQ6_K: {
      uint32_t s = j / 8;
      uint8_t byte = G[r * (w / 2) + 16 * j + (i % 16)];
      uint32_t lo = (i < 16) ? (byte & 0xF) : (byte >> 4);
      uint8_t hb = G[4 * w + r * (w / 4) + 8 * j + (i % 8)];
      uint32_t hi = (hb >> (2 * (i / 8))) & 3u;
      int q = (int)(lo | (hi << 4)) - 32;
      int8_t sc = (int8_t)G[6 * w + r * (w / 16) + 2 * j + (i / 16)];
      float d = ld_h(G + 6 * w + w / 2 + (r * (w / 256) + s) * 2);
      v = __fmul_rn(__fmul_rn(d, (float)sc), (float)q);
      break;
    }
  }
  out[t] = v;
}

int launch_unpack(int type, const void *src, uint64_t src_off, uint32_t K, uint32_t N, uint32_t CW, float *out,
                  cudaStream_t st) {
  uint32_t K8 = (K + 7) / 8 * 8;
  uint64_t n = (uint64_t)K * N;
  k_unpack<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(type, (const uint8_t *)src, src_off, K, N, K8, CW, out);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace fa
