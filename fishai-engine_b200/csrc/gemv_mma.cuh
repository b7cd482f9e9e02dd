// Device building blocks of the tensor-core dequant-GEMV (see gemv_mma.cu):
// shared-memory layout, coefficient builders, MMA groups, the producer
// (weight stages into the ring) and the consumer (x slice, stages, chunk
// flush and fused epilogue) of one GEMV launch for one CTA.  Used by the
// standalone launch (k_gemv_mma) and by the persistent decode-step kernel,
// which runs many GEMVs back to back through one ring.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "fa_device.cuh"
#include "fa_kernels.hpp"
#include "gemv_epi.cuh"

namespace fa {
namespace mma {


constexpr int kWarps = 16;
constexpr int kThreads = (kWarps + 1) * 32;
constexpr int kMaxStages = 12;              // ring depth is p.n_stages (set from the shared-memory budget)
constexpr uint32_t kMaxStageGroups = 4;     // row groups per stage
constexpr uint32_t kStageTarget = 36 * 1024;
constexpr uint32_t kTblWords = 8 * 24;      // one table: (groups x blocks <= 8) x (3 splits x 4 lanes x 2 words)
constexpr uint32_t kZeroWords = 256;        // B fragment source of the lanes whose column is unused
constexpr uint32_t kSlotWord = kWarps * kTblWords - kGemvMaxContrib;  // epilogue: contributor slots at the table end
// shared memory: mbarriers + flag | reduction scratch | zero area | tables | x | ring
constexpr uint32_t kOffRed = 256, kOffZero = kOffRed + 512, kOffTbl = kOffZero + 4 * kZeroWords,
                   kOffX = kOffTbl + 4 * kWarps * kTblWords;
constexpr float kBScale = 0x1p96f;          // B = c * 2^96
constexpr float kYScale = 0x1p37f;          // A = q * 2^-133  ->  y = D * 2^37

struct Smem {
  uint64_t *full, *empty;
  uint32_t *flag;
  float *red;
  uint32_t *zero, *tbl;
  float *xs;
  uint8_t *ring;
};

__host__ __device__ inline uint32_t ring_offset(uint32_t max_units) {
  return (kOffX + max_units * 64 + 127) / 128 * 128;
}

__device__ __forceinline__ Smem carve(uint8_t *smem, const GemvParams &p) {
  Smem s;
  s.full = reinterpret_cast<uint64_t *>(smem);
  s.empty = s.full + kMaxStages;
  s.flag = reinterpret_cast<uint32_t *>(smem + 16 * kMaxStages);
  s.red = reinterpret_cast<float *>(smem + kOffRed);
  s.zero = reinterpret_cast<uint32_t *>(smem + kOffZero);
  s.tbl = reinterpret_cast<uint32_t *>(smem + kOffTbl);
  s.xs = reinterpret_cast<float *>(smem + kOffX);
  s.ring = smem + ring_offset(p.max_units);
  return s;
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// explicit shared-window accesses (32-bit addresses)
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts32(uint32_t a, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ float2 h2f2_bits(uint32_t w) {
  return __half22float2(*reinterpret_cast<const __half2 *>(&w));
}

__device__ __forceinline__ uint32_t bf2_bits(__nv_bfloat162 v) { return *reinterpret_cast<uint32_t *>(&v); }
__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// v -> hi + mid + lo, each a bf16 pair, exactly (8 + 8 + 8 bits): the
// residuals v - hi and r - mid are exact in f32 (one packed FMA each);
// written to the three split rows of the coefficient table (word stride 8)
__device__ __forceinline__ void split_store(float2 v, uint32_t dst) {
  const float2 m1 = make_float2(-1.0f, -1.0f);
  const uint32_t hi = bf2_bits(__floats2bfloat162_rn(v.x, v.y));
  const float2 r = __ffma2_rn(make_float2(bf_lo(hi), bf_hi(hi)), m1, v);
  const uint32_t mid = bf2_bits(__floats2bfloat162_rn(r.x, r.y));
  const float2 t = __ffma2_rn(make_float2(bf_lo(mid), bf_hi(mid)), m1, r);
  sts32(dst, hi);
  sts32(dst + 32, mid);
  sts32(dst + 64, bf2_bits(__floats2bfloat162_rn(t.x, t.y)));
}

// two small non-negative integers (< 2^23) -> floats, exactly
__device__ __forceinline__ float2 u2f2(uint32_t a, uint32_t b, float bias) {
  return __fadd2_rn(make_float2(__uint_as_float(0x4B000000u | a), __uint_as_float(0x4B000000u | b)),
                    make_float2(-8388608.0f - bias, -8388608.0f - bias));
}

// ---------------------------------------------------------------------------
// per-type geometry: J = blocks (coefficient columns) per 64-column slice,
// kCorr = factor of the per-block correction sum, PAIR_LANES: a builder lane
// takes one row pair for every block of the slice (else lanes split blocks)
template <int T>
struct Geo;
template <>
struct Geo<kQ4_K> {
  static constexpr int J = 2;
  static constexpr float kCorr = 1.0f;  // corr = sum x * (dmin * m)
  static constexpr bool PAIR_LANES = true;
};
template <>
struct Geo<kQ6_K> {
  static constexpr int J = 4;
  static constexpr float kCorr = 0x1p-91f;  // 32 * 2^-96: value (q - 32) * d * sc, corr sums c * 2^96
  static constexpr bool PAIR_LANES = false;
};
template <>
struct Geo<kQ8_0> {
  static constexpr int J = 2;
  static constexpr float kCorr = 0x1p-89f;  // 128 * 2^-96: stored u = q + 128, corr sums c * 2^96
  static constexpr bool PAIR_LANES = false;
};
template <>
struct Geo<kQ4_0> {
  static constexpr int J = 2;
  static constexpr float kCorr = 0x1p-93f;  // 8 * 2^-96: value (q - 8) * d, corr sums c * 2^96
  static constexpr bool PAIR_LANES = true;
};

// groups per stage for a chunk of this type and group size (the coefficient
// table holds groups x blocks <= 8)
__host__ __device__ inline uint32_t stage_groups(uint32_t gbytes, int type) {
  const uint32_t cap = (type == kQ6_K || type == kQ8_0) ? 2u : kMaxStageGroups;
  const uint32_t n = kStageTarget / gbytes;
  return n < 1 ? 1 : (n > cap ? cap : n);
}

// Coefficients of this warp's slice for the stage (ng groups, rows of x at
// xs).  Table word of (group gi, block j, split s, row pair p): (gi*J + j)*24
// + s*8 + (p%4)*2 + (p%8)/4, so fragment lane (g, c) reads words (g*4+c)*2, +1.
// All addresses are shared-window byte addresses.
template <int T>
__device__ __forceinline__ void build(uint32_t stage, uint32_t gbytes, uint32_t w, uint32_t slice, uint32_t nblk,
                                      uint32_t ng, uint32_t xs, uint32_t lane, uint32_t tbl, float (&corr)[2]) {
  constexpr int J = Geo<T>::J;
  const uint32_t p = Geo<T>::PAIR_LANES ? lane : (lane & 15), jb = Geo<T>::PAIR_LANES ? 0 : (lane >> 4);
  if (p >= 8 * ng || jb >= nblk) return;
  const uint2 xb = lds64(xs + 8 * p);
  const float2 x = make_float2(__uint_as_float(xb.x), __uint_as_float(xb.y));
  const float2 xs96 = __fmul2_rn(x, make_float2(kBScale, kBScale));
  const uint32_t gi = p >> 3, rr = 2 * (p & 7);
  const uint32_t G = stage + gi * gbytes;
  const uint32_t dst = tbl + 4 * (gi * J * 24 + (p & 3) * 2 + ((p >> 2) & 1));
  if constexpr (T == kQ4_K) {
    // the slice's two sub-blocks are adjacent 12-bit fields: 24 bits at bit 24*(slice%4)
    const uint32_t s = slice >> 2, q4 = slice & 3, fs = (24 * q4) & 31;
    const uint4 h0 = lds128(G + 8 * w + (16 * s + rr) * 16);
    const uint4 h1 = lds128(G + 8 * w + (16 * s + rr + 1) * 16);
    const uint32_t f0 = __funnelshift_r(q4 < 2 ? h0.y : (q4 == 2 ? h0.z : h0.w), q4 < 2 ? h0.z : h0.w, fs);
    const uint32_t f1 = __funnelshift_r(q4 < 2 ? h1.y : (q4 == 2 ? h1.z : h1.w), q4 < 2 ? h1.z : h1.w, fs);
    const float2 dd0 = h2f2_bits(h0.x), dd1 = h2f2_bits(h1.x);    // (d, dmin) of the two rows
    const float2 xd = __fmul2_rn(xs96, make_float2(dd0.x, dd1.x));  // x * d * 2^96
    const float2 xm = __fmul2_rn(x, make_float2(dd0.y, dd1.y));     // x * dmin
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const float2 sc = u2f2((f0 >> (12 * j)) & 63u, (f1 >> (12 * j)) & 63u, 0.0f);
      const float2 m = u2f2((f0 >> (12 * j + 6)) & 63u, (f1 >> (12 * j + 6)) & 63u, 0.0f);
      corr[j] = fmaf(xm.x, m.x, fmaf(xm.y, m.y, corr[j]));
      split_store(__fmul2_rn(xd, sc), dst + 96 * j);
    }
  } else if constexpr (T == kQ4_0) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      if (j >= (int)nblk) break;
      const float2 c = __fmul2_rn(xs96, h2f2_bits(lds32(G + 8 * w + ((2 * slice + j) * 16 + rr) * 2)));
      corr[j] += c.x + c.y;
      split_store(c, dst + 96 * j);
    }
  } else if constexpr (T == kQ6_K) {
    const uint32_t s = slice >> 2;
    const float2 xd = __fmul2_rn(xs96, h2f2_bits(lds32(G + 13 * w + (16 * s + rr) * 2)));
#pragma unroll
    for (int q = 0; q < 2; ++q) {
      const uint32_t j = jb + 2 * q;
      const uint32_t scw = lds16(G + 12 * w + (4 * slice + j) * 16 + rr);
      const float2 c = __fmul2_rn(xd, u2f2((scw & 0xFFu) ^ 0x80u, (scw >> 8) ^ 0x80u, 128.0f));  // int8 scales
      corr[q] += c.x + c.y;
      split_store(c, dst + 96 * j);
    }
  } else {  // Q8_0: one f16 d per row and 32-column block
    const float2 c = __fmul2_rn(xs96, h2f2_bits(lds32(G + 16 * w + ((2 * slice + jb) * 16 + rr) * 2)));
    corr[0] += c.x + c.y;
    split_store(c, dst + 96 * jb);
  }
}

// the MMAs of one 16-row group for this warp's slice (NT tiles); bsrc is
// this lane's B-fragment source (its table column, or the zero area)
template <int T, int NT>
__device__ __forceinline__ void mma_group(uint32_t G, uint32_t w, uint32_t slice, uint32_t lane, uint32_t bsrc,
                                          float (&D)[4][4], float (&Dh)[4][4]) {
  constexpr int J = Geo<T>::J;
  constexpr int JN = (NT == 4) ? J : J / 2;
  uint2 b[JN];
#pragma unroll
  for (int j = 0; j < JN; ++j) b[j] = lds64(bsrc + 96 * j);
  if constexpr (T == kQ8_0) {
    uint32_t q[2 * NT];
#pragma unroll
    for (int i = 0; i < NT / 2; ++i) {
      const uint4 v = lds128(G + 1024 * slice + 8 * NT * lane + 16 * i);
      q[4 * i] = v.x;
      q[4 * i + 1] = v.y;
      q[4 * i + 2] = v.z;
      q[4 * i + 3] = v.w;
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const uint32_t P = q[2 * t], Q = q[2 * t + 1];
      mma_bf16(D[t], P & 0x00FF00FFu, (P >> 8) & 0x00FF00FFu, Q & 0x00FF00FFu, (Q >> 8) & 0x00FF00FFu,
               b[t >> 1].x, b[t >> 1].y);
    }
  } else {
    uint32_t q[NT];
    if constexpr (NT == 4) {
      const uint4 v = lds128(G + 512 * slice + 16 * lane);
      q[0] = v.x;
      q[1] = v.y;
      q[2] = v.z;
      q[3] = v.w;
    } else {
      const uint2 v = lds64(G + 512 * slice + 8 * lane);
      q[0] = v.x;
      q[1] = v.y;
    }
#pragma unroll
    for (int t = 0; t < NT; ++t) {
      const uint32_t W = q[t], S = W >> 8;
      const int j = (T == kQ6_K) ? t : (t >> 1);
      mma_bf16(D[t], W & 0x000F000Fu, W & 0x00F000F0u, S & 0x000F000Fu, S & 0x00F000F0u, b[j].x, b[j].y);
    }
    if constexpr (T == kQ6_K) {
      const uint2 hw = lds64(G + 8 * w + 256 * slice + 8 * lane);
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint32_t H = (t < 2 ? hw.x : hw.y) >> (2 * (t & 1)), S = H >> 8;
        mma_bf16(Dh[t], H & 0x00030003u, H & 0x00300030u, S & 0x00030003u, S & 0x00300030u, b[t].x, b[t].y);
      }
    }
  }
}

// D -> column values of this warp's slice, minus the block corrections, into
// the chunk partial (rows m >= 8 of the 4-bit layouts carry an extra x16);
// STAGE: into the warp's shared-memory staging row instead (kEpiRed)
template <int T, int NT, bool STAGE = false>
__device__ __forceinline__ void flush_warp(float *dst, uint32_t lane, float (&D)[4][4], float (&Dh)[4][4],
                                           float (&corr)[2]) {
  constexpr int kOff = Geo<T>::PAIR_LANES ? 16 : 8;  // builder lanes sharing a block
#pragma unroll
  for (int o = kOff; o; o >>= 1) {
    corr[0] += __shfl_xor_sync(0xFFFFFFFFu, corr[0], o);
    corr[1] += __shfl_xor_sync(0xFFFFFFFFu, corr[1], o);
  }
  const uint32_t g = lane >> 2, c = lane & 3;
  constexpr float kHi = (T == kQ8_0) ? kYScale : kYScale * 0.0625f;
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float d[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) d[i] = (T == kQ6_K) ? fmaf(16.0f, Dh[t][i], D[t][i]) : D[t][i];
    const float lo0 = __shfl_down_sync(0xFFFFFFFFu, d[0], 1), lo8 = __shfl_down_sync(0xFFFFFFFFu, d[2], 1);
    float cr;
    if constexpr (Geo<T>::PAIR_LANES) cr = corr[t >> 1];
    else if constexpr (T == kQ6_K) cr = __shfl_sync(0xFFFFFFFFu, t < 2 ? corr[0] : corr[1], 16 * (t & 1));
    else cr = __shfl_sync(0xFFFFFFFFu, corr[0], 16 * (t >> 1));
    const float cv = __fmul_rn(Geo<T>::kCorr, cr);
    if (c == 0) {
      const float v0 = __fsub_rn(__fmul_rn(__fadd_rn(__fadd_rn(d[0], d[1]), lo0), kYScale), cv);
      const float v1 = __fsub_rn(__fmul_rn(__fadd_rn(__fadd_rn(d[2], d[3]), lo8), kHi), cv);
      if constexpr (STAGE) {
        dst[16 * t + g] = v0;
        dst[16 * t + g + 8] = v1;
      } else {
        __stcg(dst + 16 * t + g, v0);
        __stcg(dst + 16 * t + g + 8, v1);
      }
    }
  }
}

// stage sequence of a CTA: u = CTA-local index of the stage's first unit,
// (c, g) its chunk and group, ng groups, last = the CTA's rows of chunk c end
struct Stage {
  uint32_t u, c, g, ng;
  bool last;
};
__device__ __forceinline__ void stage_fill(const GemvParams &p, uint32_t n_units, uint32_t G, Stage &st) {
  const uint32_t sg = p.chunks[st.c].sgroups;
  st.ng = min(min(sg, G - st.g), n_units - st.u);
  st.last = (st.g + st.ng == G) || (st.u + st.ng == n_units);
}
__device__ __forceinline__ void stage_advance(const GemvParams &p, uint32_t n_units, uint32_t G, Stage &st) {
  st.u += st.ng;
  st.g += st.ng;
  if (st.g == G) {
    st.g = 0;
    st.c += 1;
  }
  if (st.u < n_units) stage_fill(p, n_units, G, st);
}

// The stages of one chunk segment of the CTA's range (seg groups starting at
// CTA-local unit u): wait, build the coefficients, run the MMAs, release the
// slot.  slot / phase walk the ring.
template <int T>
__device__ __forceinline__ void segment(const uint32_t n_stages, const uint32_t stage_bytes, const uint64_t wait_ns,
                                        const Smem &sm, const ChunkDesc &cd, uint32_t seg,
                                        uint32_t u, uint32_t warp, uint32_t lane, uint32_t tbl, uint32_t bsrc,
                                        uint32_t ring, uint32_t xs0, uint32_t &slot, uint32_t &phase, bool &ok,
                                        float (&D)[4][4], float (&Dh)[4][4], float (&corr)[2]) {
  const uint32_t w = cd.width, sg = cd.sgroups, gbytes = cd.gbytes;
  const bool active = 64 * warp < w;
  const uint32_t nt = active ? min(64u, w - 64 * warp) / 16 : 0;
  const uint32_t nblk = (nt == 4) ? Geo<T>::J : Geo<T>::J / 2;
  for (uint32_t done = 0; done < seg;) {
    const uint32_t ng = min(sg, seg - done);
    // after a timed-out wait the warp keeps the loop structure but skips the
    // work; the error flag tells the host the result is void
    if (ok && !mbar_wait_sleep(&sm.full[slot], phase, wait_ns)) ok = false;
    if (active && ok) {
      const uint32_t base = ring + slot * stage_bytes;
      build<T>(base, gbytes, w, warp, nblk, ng, xs0 + 64 * (u + done), lane, tbl, corr);
      __syncwarp();
      if (nt == 4) {
#pragma unroll
        for (uint32_t gi = 0; gi < kMaxStageGroups; ++gi)
          if (gi < ng) mma_group<T, 4>(base + gi * gbytes, w, warp, lane, bsrc + gi * Geo<T>::J * 96, D, Dh);
      } else {
        for (uint32_t gi = 0; gi < ng; ++gi)
          mma_group<T, 2>(base + gi * gbytes, w, warp, lane, bsrc + gi * Geo<T>::J * 96, D, Dh);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&sm.empty[slot]);
    done += ng;
    if (++slot == n_stages) {
      slot = 0;
      phase ^= 1u;
    }
  }
}

template <int T>
__device__ __forceinline__ void flush_slice(const GemvParams &p, const ChunkDesc &cd, uint32_t slot, uint32_t warp,
                                            uint32_t lane, float (&D)[4][4], float (&Dh)[4][4], float (&corr)[2]) {
  float *dst = p.part + (size_t)slot * p.CW + 64 * warp;
  if (min(64u, cd.width - 64 * warp) == 64) flush_warp<T, 4>(dst, lane, D, Dh, corr);
  else flush_warp<T, 2>(dst, lane, D, Dh, corr);
}

// kEpiRed: the warp's slice values go through its staging row (the warp's
// coefficient table, free between segments) and leave as one 16-byte vector
// red.add per lane into the destination, so split chunks need no partial
// slots, arrival counter or last-arriver pass.  Every column quad lies in one
// half of a gate/up chunk (widths are multiples of 64).
template <int T>
__device__ __forceinline__ void flush_red(const GemvParams &p, const ChunkDesc &cd, float *stage, uint32_t warp,
                                          uint32_t lane, float (&D)[4][4], float (&Dh)[4][4], float (&corr)[2]) {
  const uint32_t ncol = min(64u, cd.width - 64 * warp);
  if (ncol == 64) flush_warp<T, 4, true>(stage, lane, D, Dh, corr);
  else flush_warp<T, 2, true>(stage, lane, D, Dh, corr);
  __syncwarp();
  if (4 * lane < ncol) {
    const float4 v = reinterpret_cast<const float4 *>(stage)[lane];
    const uint32_t i = 64 * warp + 4 * lane, half = cd.width / 2;
    float *dst = !p.red_half ? p.out + cd.out_col + i
                             : p.out + cd.out_col / 2 + (i < half ? i : p.red_half + i - half);
    atomicAdd(reinterpret_cast<float4 *>(dst), v);
  }
  __syncwarp();  // the staging row is the next segment's table
}


// ---------------------------------------------------------------------------
// Producer (one lane): the weight stages of CTA `cta` of launch p, pushed into
// the ring.  s counts stages through the ring across launches (slot s % NS,
// a slot is refilled once its consumers released it).
__device__ __forceinline__ void produce(const GemvParams &p, uint32_t cta, const Smem &sm, uint32_t &s, bool &ok) {
  if (cta >= p.n_ctas || p.withhold_weights) return;
  const CtaRange R = p.ranges[cta];
  const uint32_t G = p.K / 16, start = R.c0 * G + R.g0, end = R.c1 * G + R.g1;
  const uint32_t n_units = end > start ? end - start : 0;
  if (!n_units || !ok) return;
  Stage st{0, R.c0, R.g0, 0, false};
  stage_fill(p, n_units, G, st);
  for (;; ++s) {
    const uint32_t slot = s % p.n_stages;
    if (s >= p.n_stages && !mbar_wait_sleep(&sm.empty[slot], ((s / p.n_stages) - 1) & 1u)) {
      ok = false;  // consumers time out on their own waits and unwind
      return;
    }
    const ChunkDesc &cd = p.chunks[st.c];
    const uint32_t wb = st.ng * cd.gbytes;
    mbar_arrive_expect_tx(&sm.full[slot], wb);
    bulk_g2s(sm.ring + slot * p.stage_bytes, p.w + cd.offset + (uint64_t)st.g * cd.gbytes, wb, &sm.full[slot]);
    if (st.u + st.ng >= n_units) {
      ++s;
      return;
    }
    stage_advance(p, n_units, G, st);
  }
}

// rows units of this CTA in launch p (0 when it has none)
__device__ __forceinline__ uint32_t cta_units(const GemvParams &p, uint32_t cta) {
  if (cta >= p.n_ctas) return 0;
  const CtaRange R = p.ranges[cta];
  const uint32_t G = p.K / 16, start = R.c0 * G + R.g0, end = R.c1 * G + R.g1;
  return end > start ? end - start : 0;
}

// kProAttn prologue: the CTA's rows of x are decode-attention outputs, made
// here from the attention's split partials (max m_s, sum l_s, unnormalised
// o_s per query head and split).  Each warp computes the weights of some
// heads (lane = split: M = max m_s, e_s = exp(m_s - M), L = sum l_s e_s by a
// butterfly) into the table area while every thread's split values of its
// first row are already in flight; then x = (sum_s o_s e_s in split order) /
// L.  One round trip replaces the attention's own split combine.
__device__ __forceinline__ void attn_prologue(const GemvParams &p, const Smem &sm, uint32_t start, uint32_t G,
                                              uint32_t nx, uint32_t tid, uint32_t warp, uint32_t lane) {
  constexpr uint32_t NT = kWarps * 32, kB = 32;
  const uint32_t S = p.attn_splits, hd = p.attn_hd, NH = p.K / hd, stride = hd + 2;
  float *ecoef = reinterpret_cast<float *>(sm.tbl);  // [NH][S], then the sums [NH]
  float *lsum = ecoef + NH * S;
  float ov[kB];
  auto row_of = [&](uint32_t i) { return 16 * ((start + i / 16) % G) + (i & 15); };
  auto load = [&](uint32_t k, uint32_t s0) {
    const float *P = p.attn_part + (size_t)(k / hd) * S * stride + 2 + k % hd;
#pragma unroll
    for (uint32_t s = 0; s < kB; ++s) ov[s] = s0 + s < S ? __ldcg(P + (size_t)(s0 + s) * stride) : 0.0f;
  };
  if (tid < nx) load(row_of(tid), 0);
  for (uint32_t h = warp; h < NH; h += kWarps) {
    const float *P = p.attn_part + (size_t)h * S * stride;
    float mv[2], lv[2];
#pragma unroll
    for (uint32_t j = 0; j < 2; ++j) {
      const uint32_t s = lane + 32 * j;
      mv[j] = s < S ? __ldcg(P + (size_t)s * stride) : -INFINITY;
      lv[j] = s < S ? __ldcg(P + (size_t)s * stride + 1) : 0.0f;
    }
    float M = fmaxf(mv[0], mv[1]);
#pragma unroll
    for (int o = 16; o; o >>= 1) M = fmaxf(M, __shfl_xor_sync(0xFFFFFFFFu, M, o));
    float Ls = 0.0f;
#pragma unroll
    for (uint32_t j = 0; j < 2; ++j) {
      const uint32_t s = lane + 32 * j;
      const float e = mv[j] == -INFINITY ? 0.0f : expf(mv[j] - M);
      if (s < S) ecoef[h * S + s] = e;
      Ls = fmaf(lv[j], e, Ls);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) Ls += __shfl_xor_sync(0xFFFFFFFFu, Ls, o);
    if (lane == 0) lsum[h] = Ls;
  }
  epi::consumer_bar<kWarps>();
  for (uint32_t i = tid; i < nx; i += NT) {
    const uint32_t k = row_of(i), h = k / hd;
    const float *e = ecoef + h * S;
    float acc = 0.0f;
    for (uint32_t s0 = 0; s0 < S; s0 += kB) {
      if (i != tid || s0) load(k, s0);
#pragma unroll
      for (uint32_t s = 0; s < kB; ++s)
        if (s0 + s < S) acc = fmaf(ov[s], e[s0 + s], acc);
    }
    sm.xs[i] = acc / lsum[h];
  }
}

// Consumers (kWarps warps): the CTA's rows of x (normalised when the launch
// has an RMSNorm prologue), then its stages; at the end of each chunk segment
// the partial is published and the last contributing CTA runs the epilogue.
// slot / phase continue through the ring across launches.
// ATTN_PRO: the build that can run the kProAttn prologue (the persistent
// step kernel combines attention itself and leaves it out).
template <bool ATTN_PRO = true>
__device__ __forceinline__ void consume(const GemvParams &p, uint32_t cta, const Smem &sm, uint32_t tid,
                                        uint32_t warp, uint32_t lane, uint32_t &slot, uint32_t &phase, bool &ok) {
  if (cta >= p.n_ctas) return;
  const CtaRange R = p.ranges[cta];
  const bool norm = p.pro == kProRmsNorm, swiglu = p.pro == kProSwiglu;
  const uint32_t G = p.K / 16, start = R.c0 * G + R.g0, end = R.c1 * G + R.g1;
  const uint32_t n_units = end > start ? end - start : 0;
  if (p.zero) {  // this CTA's share of the buffer the launch clears (float4 stores)
    const uint32_t n4 = p.n_zero / 4, per = (n4 + p.n_ctas - 1) / p.n_ctas;
    const uint32_t z0 = min(n4, cta * per), z1 = min(n4, z0 + per);
    for (uint32_t i = z0 + tid; i < z1; i += kWarps * 32)
      reinterpret_cast<float4 *>(p.zero)[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  }
  if (!n_units) return;
  // the CTA's rows of x, in unit order: xs[16u + r] = x[16 g(u) + r]; the
  // first batch of x and norm weights is loaded together with the sum-of-
  // squares partials (one round trip), then normalised once inv is known
  constexpr uint32_t kPre = 8, NT = kWarps * 32;
  const uint32_t nx = n_units * 16;
  uint32_t qkv_pos = 0, qkv_slot = 0;  // qkv launches: read with the first x batch, kept for the epilogue
  if (p.epi == kEpiQkv && tid == 0) qkv_pos = p.state->pos, qkv_slot = p.state->len;
  if (ATTN_PRO && p.pro == kProAttn) {
    attn_prologue(p, sm, start, G, nx, tid, warp, lane);
  } else {
  float xr[kPre], wr[kPre];
  auto load_batch = [&](uint32_t base) {
#pragma unroll
    for (uint32_t j = 0; j < kPre; ++j) {
      const uint32_t i = base + j * NT + tid;
      if (i < nx) {
        const uint32_t k = 16 * ((start + i / 16) % G) + (i & 15);
        xr[j] = __ldcg(p.in + k);
        wr[j] = norm ? __ldg(p.norm_w + k) : (swiglu ? __ldcg(p.in2 + k) : 1.0f);
      }
    }
  };
  load_batch(0);
  float inv_self = 0.0f;  // the norm factor when this CTA summed the squares itself
  if (norm && p.n_ssq == 0) {
    // no sum-of-squares partials (x is the result of a tensor-parallel
    // all-reduce): each consumer thread squares its float4 share of x, the
    // warps' sums are added in warp order (deterministic)
    const float4 *in4 = reinterpret_cast<const float4 *>(p.in);
    const uint32_t n4 = p.K / 4;
    float s = 0.0f;
    for (uint32_t i0 = tid; i0 < n4; i0 += 4 * NT) {
      float4 a[4];
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j) {
        const uint32_t i = i0 + j * NT;
        a[j] = i < n4 ? __ldcg(in4 + i) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
      }
#pragma unroll
      for (uint32_t j = 0; j < 4; ++j)
        s = fmaf(a[j].w, a[j].w, fmaf(a[j].z, a[j].z, fmaf(a[j].y, a[j].y, fmaf(a[j].x, a[j].x, s))));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (lane == 0) sm.red[warp] = s;
    epi::consumer_bar<kWarps>();
    // every thread adds the warps' sums in warp order itself (the same value
    // everywhere), so no second barrier is needed before x is normalised
    float t = 0.0f;
#pragma unroll
    for (uint32_t w = 0; w < (uint32_t)kWarps; ++w) t += sm.red[w];
    inv_self = 1.0f / sqrtf(t / (float)p.K + p.eps);
  } else if (norm) {
    if (warp == 0) {  // lane-strided partial sums in index order, every load in flight
      float s = 0.0f;
      for (uint32_t i0 = 0; i0 < p.n_ssq; i0 += 32 * kPre) {
        float v[kPre];
#pragma unroll
        for (uint32_t j = 0; j < kPre; ++j) {
          const uint32_t i = i0 + 32 * j + lane;
          v[j] = i < p.n_ssq ? __ldcg(p.ssq + i) : 0.0f;
        }
#pragma unroll
        for (uint32_t j = 0; j < kPre; ++j) s += v[j];
      }
#pragma unroll
      for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
      if (lane == 0) sm.red[96] = 1.0f / sqrtf(s / (float)p.K + p.eps);
    }
    epi::consumer_bar<kWarps>();
  }
  {
    const float inv = norm ? (p.n_ssq == 0 ? inv_self : sm.red[96]) : 1.0f;
    for (uint32_t base = 0; base < nx; base += kPre * NT) {
      if (base) load_batch(base);
#pragma unroll
      for (uint32_t j = 0; j < kPre; ++j) {
        const uint32_t i = base + j * NT + tid;
        // rms_norm (src/tensor.rs:280-290): (x * inv) * w; swiglu: silu(gate) * up
        if (i < nx)
          sm.xs[i] = norm ? __fmul_rn(__fmul_rn(xr[j], inv), wr[j])
                          : (swiglu ? __fmul_rn(epi::silu_ref(xr[j]), wr[j]) : xr[j]);
      }
    }
  }
  }
  if (p.epi == kEpiQkv && tid == 0) {
    reinterpret_cast<uint32_t *>(sm.red)[epi::kQkvPos] = qkv_pos;
    reinterpret_cast<uint32_t *>(sm.red)[epi::kQkvSlot] = qkv_slot;
  }
  epi::consumer_bar<kWarps>();
  const uint32_t tbl = smem_u32(sm.tbl + warp * kTblWords);
  const uint32_t bsrc = (lane >> 2) < 3 ? tbl + 8 * ((lane >> 2) * 4 + (lane & 3)) : smem_u32(sm.zero) + 8 * (lane & 3);
  const uint32_t ring = smem_u32(sm.ring), xs0 = smem_u32(sm.xs);
  float D[4][4], Dh[4][4], corr[2] = {0.0f, 0.0f};
#pragma unroll
  for (int t = 0; t < 4; ++t)
#pragma unroll
    for (int i = 0; i < 4; ++i) D[t][i] = Dh[t][i] = 0.0f;
  const uint32_t n_st = p.n_stages, st_bytes = p.stage_bytes;
  const uint64_t wait_ns = p.wait_limit_ns ? p.wait_limit_ns : kWaitLimitNs;
  for (uint32_t u = 0, c = R.c0, g = R.g0; u < n_units; ++c, g = 0) {
    const ChunkDesc cd = p.chunks[c];
    const uint32_t seg = min(G - g, n_units - u);
    // the CTA's rows of chunk c: stages, then its partial into its slot
    const uint32_t slot_p = cta * p.max_chunks_per_cta + (c - R.c0);
    switch (cd.type) {
      case kQ4_K: segment<kQ4_K>(n_st, st_bytes, wait_ns, sm, cd, seg, u, warp, lane, tbl, bsrc, ring, xs0, slot, phase, ok, D, Dh, corr); break;
      case kQ6_K: segment<kQ6_K>(n_st, st_bytes, wait_ns, sm, cd, seg, u, warp, lane, tbl, bsrc, ring, xs0, slot, phase, ok, D, Dh, corr); break;
      case kQ8_0: segment<kQ8_0>(n_st, st_bytes, wait_ns, sm, cd, seg, u, warp, lane, tbl, bsrc, ring, xs0, slot, phase, ok, D, Dh, corr); break;
      default: segment<kQ4_0>(n_st, st_bytes, wait_ns, sm, cd, seg, u, warp, lane, tbl, bsrc, ring, xs0, slot, phase, ok, D, Dh, corr); break;
    }
    const bool red = p.epi == kEpiRed;
    if (ok && red && 64 * warp < cd.width) {
      float *stage = reinterpret_cast<float *>(sm.tbl) + warp * kTblWords;
      switch (cd.type) {
        case kQ4_K: flush_red<kQ4_K>(p, cd, stage, warp, lane, D, Dh, corr); break;
        case kQ6_K: flush_red<kQ6_K>(p, cd, stage, warp, lane, D, Dh, corr); break;
        case kQ8_0: flush_red<kQ8_0>(p, cd, stage, warp, lane, D, Dh, corr); break;
        default: flush_red<kQ4_0>(p, cd, stage, warp, lane, D, Dh, corr); break;
      }
    } else if (ok && 64 * warp < cd.width) {
      switch (cd.type) {
        case kQ4_K: flush_slice<kQ4_K>(p, cd, slot_p, warp, lane, D, Dh, corr); break;
        case kQ6_K: flush_slice<kQ6_K>(p, cd, slot_p, warp, lane, D, Dh, corr); break;
        case kQ8_0: flush_slice<kQ8_0>(p, cd, slot_p, warp, lane, D, Dh, corr); break;
        default: flush_slice<kQ4_0>(p, cd, slot_p, warp, lane, D, Dh, corr); break;
      }
    }
#pragma unroll
    for (int t = 0; t < 4; ++t)
#pragma unroll
      for (int i = 0; i < 4; ++i) D[t][i] = Dh[t][i] = 0.0f;
    corr[0] = corr[1] = 0.0f;
    u += seg;
    if (red) continue;  // the red.adds complete the chunk: no publish, no epilogue
    // publish: the last contributing CTA to arrive sums the partials and runs
    // the epilogue.  The contributors' partial slots are fetched while the
    // arrival atomic is in flight (only the last arriver uses them).
    const uint32_t n = cd.n_contrib;
    uint32_t slot_k = 0;
    if (tid < n) slot_k = __ldg(p.contrib + cd.contrib_off + tid);
    epi::consumer_bar<kWarps>();
    if (tid == 0) {  // releases the CTA's partial (ordered before by the barrier)
      const uint32_t old = atom_add_acq_rel_gpu(p.counters + c, 1u);
      sm.flag[0] = (old + 1 == n) ? 1u : 0u;
    }
    epi::consumer_bar<kWarps>();
    if (sm.flag[0]) {  // the final arrival acquired every contributor's partial
      uint32_t *slots = sm.tbl + kSlotWord;
      if (tid < n) slots[tid] = slot_k;
      epi::consumer_bar<kWarps>();
      epi::epilogue<kWarps>(p, sm.red, reinterpret_cast<float *>(sm.tbl), slots, cd, c, tid, warp, lane, true);
      if (tid == 0) p.counters[c] = 0;  // ready for the next use of the chunk counters
      if (p.done) {  // chunk complete: count it for the launches that wait on this one
        epi::consumer_bar<kWarps>();
        if (tid == 0) red_add_release_gpu(p.done, 1u);
      }
    }
    epi::consumer_bar<kWarps>();
  }
}

}  // namespace mma
}  // namespace fa
