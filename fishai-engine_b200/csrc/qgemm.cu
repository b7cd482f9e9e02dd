// Token-parallel dequant-GEMM on the 5th-generation tensor cores (tcgen05):
// Y[t][n] = sum_k X[t][k] * W[k][n] for T tokens at once (prefill, batched
// decode), W in the MMA tile layout of the decode GEMV (Q4_K, Q6_K, Q8_0,
// Q4_0; src/tensor.rs:244-258 computes the same product in f32).
//
// f16 operands (11 mantissa bits: 8x less rounding than bf16 at the same
// tensor throughput; the activation producers flag values beyond the f16
// range), f32 accumulation in tensor memory:
//   A = W^T tile: 128 weight columns x 64 rows, dequantised by 16 producer
//       warps (one 16-row x 32-column unit each) into the K-major 128-byte
//       swizzled shared-memory layout the MMA reads, every value rounded once
//       to f16: Q4_K / Q6_K in f32 (d*sc*q - dmin*m), Q8_0 / Q4_0 in packed
//       f16 (exact code - z, one rounding multiply by d).  Launches whose
//       chunks all have one of the last two types stage the weight bytes
//       through a per-warp cp.async ring a few k-steps ahead; the others load
//       them directly.
//   B = X tile: BN tokens x 64 rows of f16 activations, loaded by a TMA
//       tensor copy with the same 128-byte swizzle (no multicast)
//   D = 128 x BN f32 accumulator in TMEM (two buffers: the epilogue of one
//       tile overlaps the MMAs of the next)
// Roles per CTA (one persistent CTA per SM): warp 0 TMA for X, warp 1 MMA
// issue (one elected lane) and TMEM owner, warps 2-17 dequantisation, warps
// 18-21 epilogue (tcgen05.ld, optional residual add, f32 stores).  Work is
// split stream-K (below); the pieces of tiles split between CTAs are summed
// in a fixed order by a second kernel.
// Every mbarrier wait is bounded; on expiry the CTA raises p.err, the other
// roles stop at their next wait, the MMA warp drains its last commit and the
// tensor memory is always released.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>

#include "fa_device.cuh"
#include "fa_kernels.hpp"

namespace fa {
namespace {

constexpr uint32_t kBM = 128, kBK = 64;          // weight columns (MMA M) and rows per k-step
constexpr uint32_t kDeq = 16;                    // dequant warps: one (16-row group, 32-column block) each
constexpr uint32_t kEpi0 = 2 + kDeq;             // first epilogue warp
constexpr uint32_t kQThreads = (kEpi0 + 4) * 32; // 704
constexpr uint32_t kATile = kBM * kBK * 2;       // 16 KB

// Shared memory of one weight prefetch slot of a dequant warp (codes + scales):
// Q8_0 / Q4_0 544 bytes, Q4_K 640 (512 code bytes, 8 row headers), Q6_K 448
constexpr uint32_t kPfWarp = 640;

// PF: the launch stages its weight bytes through the prefetch ring (every
// chunk Q8_0 or Q4_0, or kPfAny: any mix of the four MMA types with
// K-quant widths of whole super-blocks); otherwise the dequant warps load
// them directly.
// BN = 512: a token-tile pair — two B tiles of 256 tokens per stage, two
// N = 256 MMAs per 16-row step into the two halves of TMEM, so each
// dequantised A stage serves 512 tokens (the accumulator is not double
// buffered: the epilogue of a pair runs before the next pair's MMAs)
template <uint32_t BN, bool PF>
struct QCfg {
  static constexpr uint32_t kN = BN > 256 ? 256 : BN;          // N of one MMA instruction
  static constexpr uint32_t kHalves = BN / kN;                 // B tiles (TMA boxes, MMAs) per stage
  static constexpr uint32_t kAccBufs = BN > 256 ? 1 : 2;       // accumulators in TMEM
  static constexpr uint32_t kBTile = BN * kBK * 2;
  static constexpr uint32_t kStage = kATile + kBTile;
  // A/B stages (without the ring: as many as 192 KB holds, at most 8) and
  // the ring's depth in k-steps
  static constexpr uint32_t kFit = (192 * 1024) / kStage > 8 ? 8 : (192 * 1024) / kStage;
  static constexpr uint32_t kStages = PF ? (BN == 64 ? 6 : (BN == 128 ? 5 : (BN == 256 ? 3 : 2))) : kFit;
  static constexpr uint32_t kPf = PF ? 4 : 0;
  static constexpr uint32_t kPfStage = kDeq * kPfWarp;  // one region per dequant warp
  static constexpr uint32_t kPfOff = kStages * kStage;
  static constexpr uint32_t kBarOff = kPfOff + kPf * kPfStage;
  static constexpr uint32_t kSmem = 1024 + kBarOff + 256;   // 1 KB alignment slack, barriers
  static_assert(kSmem <= 227 * 1024, "shared memory per CTA");
  static constexpr uint32_t kTmemCols = kAccBufs * BN;
  static_assert(kTmemCols <= 512, "tensor memory columns");
  // tcgen05 instruction descriptor: f32 D, f16 A and B (format 0), both K-major, M = 128, N = kN
  static constexpr uint32_t kIdesc = (1u << 4) | ((kN >> 3) << 17) | ((kBM >> 4) << 24);
};

struct QBars {
  uint64_t full_a[8], full_b[8], empty[8], acc_full[2], acc_empty[2], done;
  uint32_t tmem, abort;
};

// shared-memory matrix descriptor: K-major, 128-byte swizzle, rows of 128 B,
// 8-row groups 1024 B apart; the start address advances 32 B per 16-wide k step
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(acc), "r"(0u), "r"(0u), "r"(0u), "r"(0u));
}
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_2d(void *dst, const void *tmap, int32_t c0, int32_t c1, uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(c0), "r"(c1), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ uint32_t pack_f16(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t *>(&h);
}
__device__ __forceinline__ void sts32(uint32_t addr, uint32_t v) {
  asm volatile("st.shared.u32 [%0], %1;" ::"r"(addr), "r"(v) : "memory");
}
// W^T element pair (column n, rows k and k+1; k even) of the A tile at `a`
__device__ __forceinline__ void put_pair(uint32_t a, uint32_t n, uint32_t k, float lo, float hi) {
  sts32(a + n * 128 + ((((k >> 3) ^ (n & 7)) << 4) | ((k & 7) << 1)), pack_f16(lo, hi));
}

// bounded wait that also gives up once another role has aborted
__device__ __forceinline__ bool qwait(uint64_t *bar, uint32_t parity, QBars &b) {
  if (*reinterpret_cast<volatile uint32_t *>(&b.abort)) return false;
  if (mbar_wait_sleep(bar, parity)) return true;
  atomicExch(&b.abort, 1u);
  return false;
}
// the same, agreed by the whole warp (every lane polls; one failure fails all)
__device__ __forceinline__ bool qwait_warp(uint64_t *bar, uint32_t parity, QBars &b) {
  return __all_sync(0xFFFFFFFFu, qwait(bar, parity, b));
}

__device__ __forceinline__ uint4 ldg128(const uint8_t *p) { return __ldg(reinterpret_cast<const uint4 *>(p)); }
__device__ __forceinline__ uint2 ldg64(const uint8_t *p) { return __ldg(reinterpret_cast<const uint2 *>(p)); }
__device__ __forceinline__ uint32_t ldg32(const uint8_t *p) { return __ldg(reinterpret_cast<const uint32_t *>(p)); }
__device__ __forceinline__ __half2 u32_h2(uint32_t v) { return *reinterpret_cast<const __half2 *>(&v); }
__device__ __forceinline__ uint32_t h2_u32(__half2 v) { return *reinterpret_cast<const uint32_t *>(&v); }

// Dequant units.  A unit is one (16-row group, 32-column block) piece of
// the A tile: block th (0 or 1) of the 64-column slice i.  Lane l = 4g + c
// owns, per 16x16 tile t of the block (t = 2th, 2th + 1), the weight
// columns g and g+8 and the rows 2c, 2c+1, 2c+8, 2c+9 of the group (the
// mma.sync fragment order the layout stores); k0 = the group's first row in
// the tile.  The caller skips a block past the slice's last tile (2th >= nt).

// Q4_K unit of one warp of a pair: all four tiles of the 64-column slice i,
// rows 2c, 2c+1 (th = 0) or 2c+8, 2c+9 (th = 1) of lane l = 4g + c, so each
// warp reads the scale headers of its own two rows only.
// qv: the lane's code words (one per tile), hr[jj]: the header of row
// 2c + 8th + jj of the slice's super-block; i3 = slice index & 3
__device__ __forceinline__ void deq_q4k_vals(uint4 qv, const uint4 (&hr)[2], uint32_t i3, uint32_t th, uint32_t lane,
                                             uint32_t a, uint32_t n0, uint32_t k0) {
  const uint32_t g = lane >> 2, c = lane & 3;
  const uint32_t q[4] = {qv.x, qv.y, qv.z, qv.w};
  const uint32_t r0 = 2 * c + 8 * th;
  float sa[2][2], sb[2][2];  // [row][32-column block]
  // the slice's two 12-bit (sc | m << 6) fields are adjacent: 24 bits at
  // bit 24 * i3 of the 96-bit field area, one funnel shift (i3 is warp-uniform)
  const uint32_t fs = (24 * i3) & 31;
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    const uint4 h = hr[jj];
    const float d = __half2float(__ushort_as_half((unsigned short)(h.x & 0xFFFFu)));
    const float dm = __half2float(__ushort_as_half((unsigned short)(h.x >> 16)));
    const uint32_t F = __funnelshift_r(i3 < 2 ? h.y : (i3 == 2 ? h.z : h.w), i3 < 2 ? h.z : h.w, fs);
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      sa[jj][b] = d * u2f_small((F >> (12 * b)) & 63u);
      sb[jj][b] = dm * u2f_small((F >> (12 * b + 6)) & 63u);
    }
  }
#pragma unroll
  for (uint32_t t = 0; t < 4; ++t) {
    const uint32_t b = t >> 1, W = q[t] >> (8 * th);  // this row half's codes in nibbles 0, 4, 1, 5 of W
    const uint32_t n = n0 + 16 * t + g;
#pragma unroll
    for (int col = 0; col < 2; ++col) {  // column g then g+8
      const uint32_t e0 = (W >> (4 * col)) & 0xFu, e1 = (W >> (16 + 4 * col)) & 0xFu;
      const float2 ef = __fadd2_rn(make_float2(__uint_as_float(0x4B000000u | e0), __uint_as_float(0x4B000000u | e1)),
                                   make_float2(-8388608.0f, -8388608.0f));
      const float2 v = __ffma2_rn(make_float2(sa[0][b], sa[1][b]), ef, make_float2(-sb[0][b], -sb[1][b]));
      put_pair(a, n + 8 * col, k0 + r0, v.x, v.y);
    }
  }
}
__device__ __forceinline__ void deq_unit_q4k_rows(const uint8_t *G, uint32_t w, uint32_t i, uint32_t th,
                                                  uint32_t lane, uint32_t a, uint32_t n0, uint32_t k0) {
  const uint32_t r0 = 2 * (lane & 3) + 8 * th, s = i >> 2;
  const uint4 qv = ldg128(G + 512 * i + 16 * lane);  // Q4_K slices are whole (4 tiles): one word per tile
  const uint4 hr[2] = {ldg128(G + 8 * w + (16 * s + r0) * 16), ldg128(G + 8 * w + (16 * s + r0 + 1) * 16)};
  deq_q4k_vals(qv, hr, i & 3, th, lane, a, n0, k0);
}

// Q6_K unit: value = d * sc * (q - 32), sc per (row, 16-column sub-block
// 4i + t), computed in f32 and rounded once to f16.
// qv: low-nibble words of tiles 2th, 2th+1; hw: their high-bit word; sa:
// the f16 d of rows rr[j]; scb[tt][j]: the int8 sub-scale byte of tile
// 2th + tt, row rr[j]
__device__ __forceinline__ void deq_q6k_vals(uint2 qv, uint32_t hw, const float (&sa)[4], const uint32_t (&scb)[2][4],
                                             uint32_t th, uint32_t lane, uint32_t a, uint32_t n0, uint32_t k0) {
  const uint32_t g = lane >> 2, c = lane & 3;
  const uint32_t rr[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
#pragma unroll
  for (uint32_t tt = 0; tt < 2; ++tt) {
    const uint32_t t = 2 * th + tt;
    float A[4], B[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // the int8 sub-scale s as (s + 128) - 128: exact, without the slow I2F path
      const float sc = u2f_small(scb[tt][j] ^ 0x80u) - 128.0f;
      A[j] = sa[j] * sc;
      B[j] = A[j] * 32.0f;
    }
    // codes of the 8 fragment elements: (col g | g+8) x (rows 2c, 2c+1 | 2c+8, 2c+9)
    const uint32_t W = tt ? qv.y : qv.x, H = hw >> (2 * tt);
    uint32_t e[8] = {W & 0xFu, (W >> 16) & 0xFu, (W >> 4) & 0xFu, (W >> 20) & 0xFu,
                     (W >> 8) & 0xFu, (W >> 24) & 0xFu, (W >> 12) & 0xFu, W >> 28};
    const uint32_t pos[8] = {0, 16, 4, 20, 8, 24, 12, 28};
#pragma unroll
    for (int x = 0; x < 8; ++x) e[x] |= ((H >> pos[x]) & 3u) << 4;
    // element x: col g + 8*((x>>1)&1), row index j = (x&1) + 2*(x>>2)
    const uint32_t n = n0 + 16 * t + g;
#pragma unroll
    for (int half = 0; half < 2; ++half) {     // rows 2c,2c+1 then 2c+8,2c+9
#pragma unroll
      for (int col = 0; col < 2; ++col) {      // column g then g+8
        const int x0 = 4 * half + 2 * col, x1 = x0 + 1;
        const int j0 = 2 * half, j1 = 2 * half + 1;
        // codes to floats by the exponent trick (exact, full-rate adds), then
        // value = A * code - B with one rounding, two lanes per instruction
        const float2 ef = __fadd2_rn(make_float2(__uint_as_float(0x4B000000u | e[x0]), __uint_as_float(0x4B000000u | e[x1])),
                                     make_float2(-8388608.0f, -8388608.0f));
        const float2 v = __ffma2_rn(make_float2(A[j0], A[j1]), ef, make_float2(-B[j0], -B[j1]));
        put_pair(a, n + 8 * col, k0 + rr[j0], v.x, v.y);
      }
    }
  }
}
__device__ __forceinline__ void deq_unit_q6k(const uint8_t *G, uint32_t w, uint32_t i, uint32_t th, uint32_t lane,
                                             uint32_t a, uint32_t n0, uint32_t k0) {
  const uint32_t c = lane & 3, s = i >> 2;
  const uint32_t nt = min(64u, w - 64 * i) / 16;
  const uint32_t rr[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
  const uint2 qv = ldg64(G + 512 * i + 4 * nt * lane + 8 * th);  // low nibbles: a word per tile
  const uint32_t hw = ldg32(G + 8 * w + 256 * i + 8 * lane + 4 * th);  // high bit pairs
  float sa[4];
  uint32_t scb[2][4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    sa[j] = h2f(__ldg(reinterpret_cast<const uint16_t *>(G + 13 * w + (16 * s + rr[j]) * 2)));
#pragma unroll
    for (uint32_t tt = 0; tt < 2; ++tt) scb[tt][j] = __ldg(G + 12 * w + 16 * (4 * i + 2 * th + tt) + rr[j]);
  }
  deq_q6k_vals(qv, hw, sa, scb, th, lane, a, n0, k0);
}

// Q8_0 / Q4_0 unit from its code words q (Q8_0: two words per tile; Q4_0:
// one, in q.x and q.y) and the f16 scales of rows 2c, 2c+1 (d01) and 2c+8,
// 2c+9 (d23).  value = d * (code - z), z = 128 (Q8_0) or 8 (Q4_0), in
// packed f16: a byte permute (or mask) puts two codes into the mantissas of
// 1024.0 (f16 0x6400 | code = 1024 + code, exact), one subtraction of
// 1024 + z leaves the integer code - z (exact), and one multiplication by
// the row scales rounds d * (code - z) once: the same f16 values as the
// exact f32 product rounded to f16 (a zero may carry the scale's sign).  Pairs are stored to the swizzled
// layout at the lane's two row-chunk addresses (the 128-byte swizzle XORs
// the 16-byte chunk index with n & 7 = g).
// s0, s1: the lane's store addresses of rows 2c, 2c+1 and 2c+8, 2c+9 of
// column n0 + g (q0_store_offsets).
template <int T>
__device__ __forceinline__ void deq_pairs_q0(uint4 q, uint32_t d01, uint32_t d23, uint32_t th, uint32_t s0,
                                             uint32_t s1) {
  const __half2 dlo = u32_h2(d01), dhi = u32_h2(d23);
  const __half2 zp = __float2half2_rn(T == kQ8_0 ? 1152.0f : 1032.0f);
#pragma unroll
  for (uint32_t tt = 0; tt < 2; ++tt) {
    const uint32_t o = (2 * th + tt) * 16 * 128;  // tile t: columns n0 + 16t ..
    // pairs (column g | g+8) x (rows 2c, 2c+1 | 2c+8, 2c+9)
    uint32_t pr[4];
    if (T == kQ8_0) {
      const uint32_t P = tt ? q.z : q.x, Q = tt ? q.w : q.y;
      pr[0] = __byte_perm(P, 0x64646464u, 0x4240);
      pr[1] = __byte_perm(P, 0x64646464u, 0x4341);
      pr[2] = __byte_perm(Q, 0x64646464u, 0x4240);
      pr[3] = __byte_perm(Q, 0x64646464u, 0x4341);
    } else {
      const uint32_t W = tt ? q.y : q.x;
      pr[0] = (W & 0x000F000Fu) | 0x64006400u;
      pr[1] = ((W >> 4) & 0x000F000Fu) | 0x64006400u;
      pr[2] = ((W >> 8) & 0x000F000Fu) | 0x64006400u;
      pr[3] = ((W >> 12) & 0x000F000Fu) | 0x64006400u;
    }
    sts32(s0 + o, h2_u32(__hmul2(__hsub2(u32_h2(pr[0]), zp), dlo)));
    sts32(s0 + o + 8 * 128, h2_u32(__hmul2(__hsub2(u32_h2(pr[1]), zp), dlo)));
    sts32(s1 + o, h2_u32(__hmul2(__hsub2(u32_h2(pr[2]), zp), dhi)));
    sts32(s1 + o + 8 * 128, h2_u32(__hmul2(__hsub2(u32_h2(pr[3]), zp), dhi)));
  }
}

// byte offsets in the A tile of the lane's two row chunks of column n0 + g
// (k0 = 16 gi: chunks 2gi and 2gi + 1, XOR-swizzled with n & 7 = g)
__device__ __forceinline__ void q0_store_offsets(uint32_t lane, uint32_t n0, uint32_t k0, uint32_t &o0, uint32_t &o1) {
  const uint32_t g = lane >> 2, c = lane & 3, base = (n0 + g) * 128 + 4 * c;
  o0 = base + (((k0 >> 3) ^ g) << 4);
  o1 = base + ((((k0 >> 3) + 1) ^ g) << 4);
}
template <int T>
__device__ __forceinline__ void deq_unit_q0(uint4 q, uint32_t d01, uint32_t d23, uint32_t th, uint32_t lane,
                                            uint32_t a, uint32_t n0, uint32_t k0) {
  uint32_t o0, o1;
  q0_store_offsets(lane, n0, k0, o0, o1);
  deq_pairs_q0<T>(q, d01, d23, th, a + o0, a + o1);
}

// the Q8_0 / Q4_0 unit's code words and row scales from global memory
template <int T>
__device__ __forceinline__ void load_q0(const uint8_t *G, uint32_t w, uint32_t i, uint32_t th, uint32_t lane,
                                        uint4 &q, uint32_t &d01, uint32_t &d23) {
  const uint32_t nt = min(64u, w - 64 * i) / 16, c = lane & 3;
  const uint8_t *sc = G + (T == kQ8_0 ? 16 : 8) * w + 32 * (2 * i + th) + 4 * c;
  if (T == kQ8_0) {
    q = ldg128(G + 1024 * i + 8 * nt * lane + 16 * th);
  } else {
    const uint2 v = ldg64(G + 512 * i + 4 * nt * lane + 8 * th);
    q = make_uint4(v.x, v.y, 0u, 0u);
  }
  d01 = ldg32(sc);
  d23 = ldg32(sc + 16);
}

// ---- weight prefetch ring (launches whose chunks are all Q8_0 / Q4_0) ----
// Each dequant warp copies the code words and scales of its unit for the
// next kPf - 1 k-steps into its own shared-memory region with cp.async
// (commit groups, one per k-step), so a warp keeps several k-steps of weight
// loads in flight instead of one.  Every byte is copied once per warp (the
// 32-byte scale vector by lanes 0 and 1), so the lanes read each other's
// copies after the group's wait and a __syncwarp.  Region of one warp and
// slot: [0, 512) codes (uint4 or uint2 per lane), [512, 544) the f16 scales
// of the block's 16 rows.
__device__ __forceinline__ void cpa16(uint32_t dst, const void *src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cpa8(uint32_t dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cpa_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cpa_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
  uint16_t v;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t lds8(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.u8 %0, [%1];" : "=r"(v) : "r"(a) : "memory");
  return v;
}

__device__ __forceinline__ void zero_unit(uint32_t th, uint32_t lane, uint32_t a, uint32_t n0, uint32_t k0) {
  const uint32_t g = lane >> 2, c = lane & 3;
  for (uint32_t t = 2 * th; t < 2 * th + 2; ++t)
#pragma unroll
    for (int half = 0; half < 2; ++half)
#pragma unroll
      for (int col = 0; col < 2; ++col) put_pair(a, n0 + 16 * t + g + 8 * col, k0 + 2 * c + 8 * half, 0.0f, 0.0f);
}

// Stream-K work split: the sequence of (output tile, k-step) pairs, tiles in
// order (token tile fastest) and each tile's k-steps in order, is cut into
// gridDim.x equal contiguous ranges of at least kMinSk k-steps; CTA c takes
// [sk_start(c), sk_start(c + 1)).  A range covers whole tiles except possibly
// a piece of a tile at each end: the pieces go to partial slots 2c (the
// range's first segment) and 2c + 1 (its last), and k_qg_fixup adds the
// pieces of each split tile in CTA order.  (Measured against whole tiles in
// strided waves with only the last wave split: that order shares weight
// tiles better in L2 but loses more to the partial wave, and pure stream-K
// gave the faster prefill and batched decode.)
constexpr uint32_t kMinSk = 8;
__host__ __device__ __forceinline__ uint32_t sk_start(uint32_t c, uint64_t W, uint32_t G) {
  return (uint32_t)((uint64_t)c * W / G);
}
struct Seg {
  uint32_t nt, tt, ks0, ks1;
  bool first, whole;
};
struct SegIter {
  uint32_t k, end, KS, t_tiles;
  bool first;
  __device__ SegIter(uint32_t cta, uint32_t G, uint32_t n_tiles, uint32_t t_tiles_, uint32_t ksteps)
      : KS(ksteps), t_tiles(t_tiles_), first(true) {
    const uint64_t W = (uint64_t)n_tiles * t_tiles_ * ksteps;
    k = sk_start(cta, W, G);
    end = sk_start(cta + 1, W, G);
  }
  __device__ bool next(Seg &sg) {
    if (k >= end) return false;
    const uint32_t x = k / KS;
    sg.tt = x % t_tiles;
    sg.nt = x / t_tiles;
    sg.ks0 = k % KS;
    sg.ks1 = min(KS, sg.ks0 + (end - k));
    sg.whole = sg.ks0 == 0 && sg.ks1 == KS;
    sg.first = first;
    first = false;
    k += sg.ks1 - sg.ks0;
    return true;
  }
};

// The prefetch side of a dequant warp: the (weight tile, k-step) sequence
// of the CTA's range one k-step at a time, with the source addresses of
// the warp's unit (code words of lane l, the 32-byte scale vector for lanes
// 0 and 1) in the current k-step's row group; within a tile they advance by
// four row groups per k-step.
template <int PT>
struct PfCursor {
  const uint8_t *code, *sc;
  uint64_t step;
  uint32_t k, ks, tt, nt, gi, si, th, lane;
  bool active;  // this warp's block exists in the tile
  __device__ void tile(const QgParams &p) {
    if (nt >= p.n_tiles) return;
    const QgTile tl = p.tiles[nt];
    const ChunkDesc cd = p.chunks[tl.chunk];
    const uint32_t i = tl.col0 / 64 + si, w = cd.width, nt16 = min(64u, w - 64 * i) / 16;
    active = 64 * si < tl.ncols && 2 * th < nt16;
    const uint8_t *G = p.w + cd.offset + (uint64_t)(4 * ks + gi) * cd.gbytes;
    code = G + (PT == kQ8_0 ? 1024 * i + 8 * nt16 * lane + 16 * th : 512 * i + 4 * nt16 * lane + 8 * th);
    sc = G + (PT == kQ8_0 ? 16 : 8) * w + 32 * (2 * i + th) + 16 * lane;
    step = 4ull * cd.gbytes;
  }
  __device__ PfCursor(const QgParams &p, uint32_t k0, uint32_t KS, uint32_t t_tiles, uint32_t gi_, uint32_t si_,
                      uint32_t th_, uint32_t lane_)
      : gi(gi_), si(si_), th(th_), lane(lane_), active(false) {
    const uint32_t x = k0 / KS;
    k = k0;
    ks = k0 % KS;
    tt = x % t_tiles;
    nt = x / t_tiles;
    tile(p);
  }
  __device__ void next(const QgParams &p, uint32_t KS, uint32_t t_tiles) {
    ++k;
    if (++ks < KS) {
      code += step;
      sc += step;
      return;
    }
    ks = 0;
    if (++tt == t_tiles) {
      tt = 0;
      ++nt;
    }
    tile(p);
  }
};

// The same for launches of mixed types (kPfAny): the warp's group base in
// the current k-step, the chunk's width and type and the slice index; the
// fetch picks the unit's bytes by type.
struct PfCursorAny {
  const uint8_t *G;
  uint64_t step;
  uint32_t k, ks, tt, nt, gi, si, th, lane, w, i, type;
  bool active;
  __device__ void tile(const QgParams &p) {
    if (nt >= p.n_tiles) return;
    const QgTile tl = p.tiles[nt];
    const ChunkDesc cd = p.chunks[tl.chunk];
    i = tl.col0 / 64 + si;
    w = cd.width;
    type = cd.type;
    active = 64 * si < tl.ncols && 2 * th < min(64u, w - 64 * i) / 16;
    G = p.w + cd.offset + (uint64_t)(4 * ks + gi) * cd.gbytes;
    step = 4ull * cd.gbytes;
  }
  __device__ PfCursorAny(const QgParams &p, uint32_t k0, uint32_t KS, uint32_t t_tiles, uint32_t gi_, uint32_t si_,
                         uint32_t th_, uint32_t lane_)
      : gi(gi_), si(si_), th(th_), lane(lane_), active(false) {
    const uint32_t x = k0 / KS;
    k = k0;
    ks = k0 % KS;
    tt = x % t_tiles;
    nt = x / t_tiles;
    tile(p);
  }
  __device__ void next(const QgParams &p, uint32_t KS, uint32_t t_tiles) {
    ++k;
    if (++ks < KS) {
      G += step;
      return;
    }
    ks = 0;
    if (++tt == t_tiles) {
      tt = 0;
      ++nt;
    }
    tile(p);
  }
};
__device__ __forceinline__ void cpa4(uint32_t dst, const void *src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
// the unit's bytes into slot R (layout per type: see deq_from_slot); type
// index 0 Q4_K, 1 Q6_K, 2 Q8_0, 3 Q4_0
__device__ __forceinline__ uint32_t pf_type_index(uint32_t type) {
  return type == kQ4_K ? 0u : type == kQ6_K ? 1u : type == kQ8_0 ? 2u : 3u;
}
__device__ __forceinline__ void fetch_unit(const PfCursorAny &fc, uint32_t R, uint32_t lane) {
  const uint8_t *G = fc.G;
  const uint32_t w = fc.w, i = fc.i, th = fc.th, s = i >> 2, nt16 = min(64u, w - 64 * i) / 16;
  switch (fc.type) {
    case kQ4_K:  // [0, 512) code words (16 B per lane), [512, 640) headers of rows 8th .. 8th + 7
      cpa16(R + 16 * lane, G + 512 * i + 16 * lane);
      if (lane < 8) cpa16(R + 512 + 16 * lane, G + 8 * w + (16 * s + 8 * th + lane) * 16);
      break;
    case kQ6_K:  // [0, 256) low words, [256, 384) high words, [384, 416) the 16 rows' d, [416, 448) sub-scales
      cpa8(R + 8 * lane, G + 512 * i + 4 * nt16 * lane + 8 * th);
      cpa4(R + 256 + 4 * lane, G + 8 * w + 256 * i + 8 * lane + 4 * th);
      if (lane < 2) cpa16(R + 384 + 16 * lane, G + 13 * w + 32 * s + 16 * lane);
      else if (lane < 4) cpa16(R + 416 + 16 * (lane - 2), G + 12 * w + 16 * (4 * i + 2 * th) + 16 * (lane - 2));
      break;
    case kQ8_0:  // as the single-type ring
      cpa16(R + 16 * lane, G + 1024 * i + 8 * nt16 * lane + 16 * th);
      if (lane < 2) cpa16(R + 512 + 16 * lane, G + 16 * w + 32 * (2 * i + th) + 16 * lane);
      break;
    default:
      cpa8(R + 8 * lane, G + 512 * i + 4 * nt16 * lane + 8 * th);
      if (lane < 2) cpa16(R + 512 + 16 * lane, G + 8 * w + 32 * (2 * i + th) + 16 * lane);
      break;
  }
}
// dequantise the unit in slot R (type index ti, slice index & 3 = i3)
__device__ __forceinline__ void deq_from_slot(uint32_t R, uint32_t ti, uint32_t i3, uint32_t th, uint32_t lane,
                                              uint32_t a, uint32_t n0, uint32_t k0, uint32_t o0, uint32_t o1) {
  const uint32_t c = lane & 3;
  if (ti == 0) {
    const uint4 qv = lds128(R + 16 * lane);
    const uint4 hr[2] = {lds128(R + 512 + 32 * c), lds128(R + 512 + 32 * c + 16)};
    deq_q4k_vals(qv, hr, i3, th, lane, a, n0, k0);
  } else if (ti == 1) {
    const uint2 qv = lds64(R + 8 * lane);
    const uint32_t hw = lds32(R + 256 + 4 * lane);
    const uint32_t rr[4] = {2 * c, 2 * c + 1, 2 * c + 8, 2 * c + 9};
    float sa[4];
    uint32_t scb[2][4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sa[j] = h2f((uint16_t)lds16(R + 384 + 2 * rr[j]));
#pragma unroll
      for (uint32_t tt = 0; tt < 2; ++tt) scb[tt][j] = lds8(R + 416 + 16 * tt + rr[j]);
    }
    deq_q6k_vals(qv, hw, sa, scb, th, lane, a, n0, k0);
  } else {
    const uint32_t d01 = lds32(R + 512 + 4 * c), d23 = lds32(R + 512 + 4 * c + 16);
    if (ti == 2) {
      deq_pairs_q0<kQ8_0>(lds128(R + 16 * lane), d01, d23, th, a + o0, a + o1);
    } else {
      const uint2 v = lds64(R + 8 * lane);
      deq_pairs_q0<kQ4_0>(make_uint4(v.x, v.y, 0u, 0u), d01, d23, th, a + o0, a + o1);
    }
  }
}

// PT: 0 = the dequant warps load the weights directly; kQ8_0 / kQ4_0 = every
// chunk has that type and the weights go through the prefetch ring
template <uint32_t BN, int PT>
__global__ void __launch_bounds__(kQThreads, 1) k_qgemm(const QgParams p, const __grid_constant__ CUtensorMap xmap) {
  constexpr bool PF = PT != 0;  // kQ8_0 / kQ4_0 (single-type ring) or kPfAny
  using C = QCfg<BN, PF>;
  extern __shared__ __align__(1024) uint8_t qsm_raw[];
  const uint32_t raw = smem_u32(qsm_raw), pad = (1024u - (raw & 1023u)) & 1023u;
  uint8_t *base = qsm_raw + pad;
  const uint32_t sbase = raw + pad;
  QBars &b = *reinterpret_cast<QBars *>(base + C::kBarOff);
  const uint32_t tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t G16 = p.K / 16, ksteps = (G16 + 3) / 4, t_tiles = (p.T + BN - 1) / BN;
  if (tid == 0) {
    for (uint32_t s = 0; s < C::kStages; ++s) {
      mbar_init(&b.full_a[s], kDeq);
      mbar_init(&b.full_b[s], 1);
      mbar_init(&b.empty[s], 1);
    }
    for (uint32_t a = 0; a < C::kAccBufs; ++a) {
      mbar_init(&b.acc_full[a], 1);
      mbar_init(&b.acc_empty[a], 4);
    }
    mbar_init(&b.done, 1);
    b.abort = 0u;
    fence_mbar_init();
  }
  if (warp == 1) {  // tensor memory: two accumulators of BN columns
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&b.tmem)),
                 "r"(C::kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = b.tmem;
  // programmatic dependent launch: the weight dequantisation (static data)
  // may start while the previous kernel finishes; the X loads and the output
  // stores wait for it (warp 0 and the epilogue warps call pdl_wait)
  pdl_launch_dependents();

  if (warp == 0) {
    // ---- X tiles by TMA ----
    pdl_wait();
    if (lane == 0) {
      uint32_t s = 0, ph = 1, pending = 0, last_ph = 0;  // pending: stages with a load issued (bit mask)
      SegIter it(blockIdx.x, gridDim.x, p.n_tiles, t_tiles, ksteps);
      Seg sg;
      while (it.next(sg)) {
        const uint32_t tt = sg.tt;
        for (uint32_t ks = sg.ks0; ks < sg.ks1; ++ks) {
          if (!qwait(&b.empty[s], ph, b)) goto tma_out;
          mbar_arrive_expect_tx(&b.full_b[s], C::kBTile);
#pragma unroll
          for (uint32_t h = 0; h < C::kHalves; ++h)
            tma_load_2d(base + s * C::kStage + kATile + h * (C::kN * kBK * 2), &xmap, (int32_t)(ks * kBK),
                        (int32_t)(tt * BN + h * C::kN), &b.full_b[s]);
          pending |= 1u << s;
          last_ph = (last_ph & ~(1u << s)) | ((ph ^ 1u) << s);  // consumer parity of this load
          if (++s == C::kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
      }
    tma_out:
      // no copy may still be writing shared memory when the CTA exits
      for (uint32_t x = 0; x < C::kStages; ++x)
        if (pending & (1u << x)) mbar_wait_sleep(&b.full_b[x], (last_ph >> x) & 1u);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ---- MMA issue ----
    uint32_t s = 0, ph = 0, acc = 0, aph = 1;
    bool issued = false;
    SegIter it(blockIdx.x, gridDim.x, p.n_tiles, t_tiles, ksteps);
    Seg wo;
    while (it.next(wo)) {
      if (!qwait_warp(&b.acc_empty[acc], aph, b)) break;
      tc_fence_after();
      const uint32_t dt = tmem + acc * BN;
      bool ok = true;
      for (uint32_t ks = wo.ks0; ks < wo.ks1; ++ks) {
        if (!qwait_warp(&b.full_a[s], ph, b) || !qwait_warp(&b.full_b[s], ph, b)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a0 = sbase + s * C::kStage, b0 = a0 + kATile;
#pragma unroll
          for (uint32_t kk = 0; kk < kBK / 16; ++kk)
#pragma unroll
            for (uint32_t h = 0; h < C::kHalves; ++h)
              umma_f16(dt + h * C::kN, sw128_desc(a0 + 32 * kk), sw128_desc(b0 + h * (C::kN * kBK * 2) + 32 * kk),
                       C::kIdesc, (ks != wo.ks0) || kk);
          umma_commit(&b.empty[s]);
        }
        __syncwarp();
        issued = true;
        if (++s == C::kStages) {
          s = 0;
          ph ^= 1u;
        }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&b.acc_full[acc]);
      __syncwarp();
      if (++acc == C::kAccBufs) {
        acc = 0;
        aph ^= 1u;
      }
    }
    // drain: every MMA this CTA issued completes before the memory is released
    if (issued) {
      if (lane == 0) umma_commit(&b.done);
      __syncwarp();
      if (!mbar_wait_sleep(&b.done, 0)) atomicExch(&b.abort, 1u);
    }
  } else if (warp < kEpi0) {
    // ---- dequantisation: unit (group gi, slice si, block th) of every stage ----
    const uint32_t d = warp - 2, gi = d >> 2, si = (d >> 1) & 1, th = d & 1;
    uint32_t s = 0, ph = 1;
    if constexpr (PT == kPfAny) {
      // The unit bytes of k-step j + kPf - 1 are copied (cp.async, one group
      // per k-step) while k-step j is dequantised; per slot the fetch records
      // 1 dequantise / 2 zero rows past K / 0 nothing, the type index and
      // the slice index & 3 (8 bits per slot).
      static_assert((C::kPf & (C::kPf - 1)) == 0 && C::kPf <= 4, "ring depth");
      const uint64_t Wk = (uint64_t)p.n_tiles * t_tiles * ksteps;
      const uint32_t k0 = sk_start(blockIdx.x, Wk, gridDim.x), kend = sk_start(blockIdx.x + 1, Wk, gridDim.x);
      const uint32_t pf0 = sbase + C::kPfOff + d * kPfWarp;
      uint32_t o0, o1;
      q0_store_offsets(lane, 64 * si, 16 * gi, o0, o1);
      PfCursorAny fc(p, k0, ksteps, t_tiles, gi, si, th, lane);
      uint32_t fslot = 0, cslot = 0, flags = 0;
      auto fetch = [&]() {
        uint32_t f = 0;
        if (fc.k < kend) {
          if (fc.active) {
            if (4 * fc.ks + gi < G16) {
              fetch_unit(fc, pf0 + fslot * C::kPfStage, lane);
              f = 1u | (pf_type_index(fc.type) << 2) | ((fc.i & 3u) << 4);
            } else {
              f = 2;
            }
          }
          fc.next(p, ksteps, t_tiles);
        }
        cpa_commit();
        flags = (flags & ~(0xFFu << (8 * fslot))) | (f << (8 * fslot));
        fslot = (fslot + 1) & (C::kPf - 1);
      };
#pragma unroll 1
      for (uint32_t j = 0; j + 1 < C::kPf; ++j) fetch();
      for (uint32_t n = kend - k0; n; --n) {
        fetch();
        cpa_wait<C::kPf - 1>();  // this lane's copies for the k-step have landed
        __syncwarp();            // ... and every other lane's
        if (!qwait_warp(&b.empty[s], ph, b)) break;
        const uint32_t f = (flags >> (8 * cslot)) & 0xFFu, a = sbase + s * C::kStage;
        if ((f & 3u) == 1u)
          deq_from_slot(pf0 + cslot * C::kPfStage, (f >> 2) & 3u, (f >> 4) & 3u, th, lane, a, 64 * si, 16 * gi, o0, o1);
        else if ((f & 3u) == 2u)
          zero_unit(th, lane, a, 64 * si, 16 * gi);
        fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(&b.full_a[s]);
        if (++s == C::kStages) {
          s = 0;
          ph ^= 1u;
        }
        cslot = (cslot + 1) & (C::kPf - 1);
      }
      cpa_wait<0>();  // no copy may still be writing shared memory when the CTA exits
    } else if constexpr (PF) {
      // The weight bytes of k-step j + kPf - 1 are copied while k-step j is
      // dequantised (one cp.async group per k-step, empty where the unit has
      // no weights), so each warp has kPf - 1 k-steps of loads in flight.
      // The fetch records per slot what the k-step needs: 1 dequantise, 2
      // zero rows past K, 0 nothing (block outside the tile).
      static_assert((C::kPf & (C::kPf - 1)) == 0, "ring depth a power of two");
      constexpr bool Q8 = PT == kQ8_0;
      const uint64_t Wk = (uint64_t)p.n_tiles * t_tiles * ksteps;
      const uint32_t k0 = sk_start(blockIdx.x, Wk, gridDim.x), kend = sk_start(blockIdx.x + 1, Wk, gridDim.x);
      const uint32_t pf0 = sbase + C::kPfOff + d * kPfWarp;
      const uint32_t rq = pf0 + (Q8 ? 16 : 8) * lane, rs = pf0 + 512 + 4 * (lane & 3);  // this lane's reads
      uint32_t o0, o1;
      q0_store_offsets(lane, 64 * si, 16 * gi, o0, o1);
      PfCursor<PT> fc(p, k0, ksteps, t_tiles, gi, si, th, lane);
      uint32_t fslot = 0, cslot = 0, flags = 0;
      auto fetch = [&]() {
        uint32_t f = 0;
        if (fc.k < kend) {
          if (fc.active) {
            if (4 * fc.ks + gi < G16) {
              const uint32_t R = pf0 + fslot * C::kPfStage;
              if (Q8) cpa16(R + 16 * lane, fc.code);
              else cpa8(R + 8 * lane, fc.code);
              if (lane < 2) cpa16(R + 512 + 16 * lane, fc.sc);
              f = 1;
            } else {
              f = 2;
            }
          }
          fc.next(p, ksteps, t_tiles);
        }
        cpa_commit();
        flags = (flags & ~(3u << (2 * fslot))) | (f << (2 * fslot));
        fslot = (fslot + 1) & (C::kPf - 1);
      };
#pragma unroll 1
      for (uint32_t j = 0; j + 1 < C::kPf; ++j) fetch();
      for (uint32_t n = kend - k0; n; --n) {
        fetch();
        cpa_wait<C::kPf - 1>();  // this lane's copies for the k-step have landed
        __syncwarp();            // ... and every other lane's
        if (!qwait_warp(&b.empty[s], ph, b)) break;
        const uint32_t f = (flags >> (2 * cslot)) & 3u, a = sbase + s * C::kStage;
        if (f == 1u) {
          const uint32_t so = cslot * C::kPfStage;
          const uint32_t d01 = lds32(rs + so), d23 = lds32(rs + so + 16);
          uint4 q;
          if (Q8) {
            q = lds128(rq + so);
          } else {
            const uint2 v = lds64(rq + so);
            q = make_uint4(v.x, v.y, 0u, 0u);
          }
          deq_pairs_q0<PT>(q, d01, d23, th, a + o0, a + o1);
        } else if (f == 2u) {
          zero_unit(th, lane, a, 64 * si, 16 * gi);
        }
        fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
        __syncwarp();
        if (lane == 0) mbar_arrive(&b.full_a[s]);
        if (++s == C::kStages) {
          s = 0;
          ph ^= 1u;
        }
        cslot = (cslot + 1) & (C::kPf - 1);
      }
      cpa_wait<0>();  // no copy may still be writing shared memory when the CTA exits
    } else {
      SegIter it(blockIdx.x, gridDim.x, p.n_tiles, t_tiles, ksteps);
      Seg wo;
      while (it.next(wo)) {
        const QgTile tl = p.tiles[wo.nt];
        const ChunkDesc cd = p.chunks[tl.chunk];
        const uint32_t i = tl.col0 / 64 + si, n0 = 64 * si;
        // the block exists: inside the tile's columns and the slice's tiles
        const bool active = n0 < tl.ncols && 2 * th < min(64u, cd.width - 64 * i) / 16;
        bool ok = true;
        for (uint32_t ks = wo.ks0; ks < wo.ks1; ++ks) {
          const uint32_t grp = 4 * ks + gi;
          if (!qwait_warp(&b.empty[s], ph, b)) {
            ok = false;
            break;
          }
          const uint32_t a = sbase + s * C::kStage;
          if (active) {
            if (grp < G16) {
              const uint8_t *G = p.w + cd.offset + (uint64_t)grp * cd.gbytes;
              uint4 q;
              uint32_t d01, d23;
              switch (cd.type) {
                case kQ4_K: deq_unit_q4k_rows(G, cd.width, i, th, lane, a, n0, 16 * gi); break;
                case kQ6_K: deq_unit_q6k(G, cd.width, i, th, lane, a, n0, 16 * gi); break;
                case kQ8_0:
                  load_q0<kQ8_0>(G, cd.width, i, th, lane, q, d01, d23);
                  deq_unit_q0<kQ8_0>(q, d01, d23, th, lane, a, n0, 16 * gi);
                  break;
                default:
                  load_q0<kQ4_0>(G, cd.width, i, th, lane, q, d01, d23);
                  deq_unit_q0<kQ4_0>(q, d01, d23, th, lane, a, n0, 16 * gi);
                  break;
              }
            } else {
              zero_unit(th, lane, a, n0, 16 * gi);
            }
          }
          fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
          __syncwarp();
          if (lane == 0) mbar_arrive(&b.full_a[s]);
          if (++s == C::kStages) {
            s = 0;
            ph ^= 1u;
          }
        }
        if (!ok) break;
      }
    }
  } else {
    // ---- epilogue warpgroup: TMEM lanes 32*(warp%4) .. +32 ----
    const uint32_t q4 = warp & 3, m = 32 * q4 + lane;
    uint32_t acc = 0, aph = 0;
    pdl_wait();
    if (p.zero) {  // this CTA's share of the buffer the launch clears (the epilogue warps are idle until the first tile)
      const uint64_t n4 = p.n_zero / 4, per = (n4 + gridDim.x - 1) / gridDim.x;
      const uint64_t z0 = min(n4, (uint64_t)blockIdx.x * per), z1 = min(n4, z0 + per);
      for (uint64_t i = z0 + (tid - kEpi0 * 32); i < z1; i += 128)
        reinterpret_cast<float4 *>(p.zero)[i] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
    SegIter it(blockIdx.x, gridDim.x, p.n_tiles, t_tiles, ksteps);
    Seg wo;
    while (it.next(wo)) {
      if (!qwait_warp(&b.acc_full[acc], aph, b)) break;
      tc_fence_after();
      const QgTile tl = p.tiles[wo.nt];
      const uint32_t t0 = wo.tt * BN, col_out = p.chunks[tl.chunk].out_col + tl.col0;
      const bool mine = m < tl.ncols;
      // a whole tile goes to the output; a piece of a split tile to the
      // CTA's partial slot ([token][column] within the tile)
      // per tile one of three stores: the output (+= for a residual
      // launch), a piece into the CTA's partial slot, or (red launches) a
      // piece added into the output by red.add
      const int mode = wo.whole ? (p.epi == kQgResid ? 1 : 0) : (p.red ? 3 : 2);
      float *slot = p.part + (size_t)(2 * blockIdx.x + (wo.first ? 0 : 1)) * kBM * BN;
      float *obase = mode == 2 ? slot + m : p.out + (size_t)t0 * p.ldo + col_out + m;
      const size_t ostride = mode == 2 ? kBM : p.ldo;
      const uint32_t tn = p.T > t0 ? min(BN, p.T - t0) : 0u;  // valid tokens of the tile
      for (uint32_t c0 = 0; c0 < BN; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + ((32 * q4) << 16) + acc * BN + c0, v);
        if (mine) {
          float *o = obase + (size_t)c0 * ostride;
          if (mode == 1) {
#pragma unroll
            for (uint32_t j = 0; j < 32; ++j)
              if (c0 + j < tn) o[(size_t)j * ostride] += __uint_as_float(v[j]);
          } else if (mode == 3) {
#pragma unroll
            for (uint32_t j = 0; j < 32; ++j)
              if (c0 + j < tn) atomicAdd(o + (size_t)j * ostride, __uint_as_float(v[j]));
          } else {
#pragma unroll
            for (uint32_t j = 0; j < 32; ++j)
              if (c0 + j < tn) o[(size_t)j * ostride] = __uint_as_float(v[j]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&b.acc_empty[acc]);
      if (++acc == C::kAccBufs) {
        acc = 0;
        aph ^= 1u;
      }
    }
  }
  __syncthreads();
  if (tid == 0 && b.abort && p.err) atomicOr(p.err, kErrWaitTimeout);
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::kTmemCols));
  }
}

// Stream-K fixup: blocks (b - 1, y) look at the range boundary sk_start(b);
// the first boundary inside a tile adds that tile's pieces (the CTA that
// reached into it from its start or earlier, then each CTA starting inside
// it) in CTA order and writes (or, for a residual launch, adds) the output.
constexpr uint32_t kFixupSlots = 512;  // pieces of one tile: at most k-steps per tile + 1 (the host checks)

__global__ void k_qg_fixup(const QgParams p, uint32_t BN, uint32_t G) {
  pdl_enter();
  const uint32_t KS = (p.K / 16 + 3) / 4, t_tiles = (p.T + BN - 1) / BN;
  const uint64_t W = (uint64_t)p.n_tiles * t_tiles * KS;
  const uint32_t bnd = blockIdx.x + 1;  // blockIdx.y: which 1024 elements of the tile
  auto kstart = [&](uint32_t c) { return (uint64_t)sk_start(c, W, G); };
  const uint64_t kb = kstart(bnd);
  if (kb % KS == 0) return;  // a tile edge: no tile is split here
  const uint32_t x = (uint32_t)(kb / KS);
  const uint64_t x0 = (uint64_t)x * KS;
  if (kstart(bnd - 1) > x0) return;  // an earlier boundary inside this tile does it
  const uint32_t tt = x % t_tiles, nt = x / t_tiles;
  const QgTile tl = p.tiles[nt];
  const uint32_t col_out = p.chunks[tl.chunk].out_col + tl.col0;
  // the pieces' slots, in CTA order, once per block
  __shared__ uint32_t slots[kFixupSlots];
  __shared__ uint32_t n_slots;
  if (threadIdx.x == 0) {
    uint32_t n = 0;
    slots[n++] = 2 * (bnd - 1) + (kstart(bnd - 1) < x0 ? 1 : 0);
    for (uint32_t c = bnd; c < G && kstart(c) < x0 + KS && n < kFixupSlots; ++c) slots[n++] = 2 * c;
    n_slots = n;
  }
  __syncthreads();
  const uint32_t n = n_slots;
  // this block's 1024 elements of the tile, four consecutive columns per thread
  const uint32_t idx = blockIdx.y * 1024 + 4 * threadIdx.x, t = idx / kBM, m = idx % kBM;
  if (idx >= BN * kBM || m >= tl.ncols || tt * BN + t >= p.T) return;
  float4 *o = reinterpret_cast<float4 *>(p.out + (size_t)(tt * BN + t) * p.ldo + col_out + m);
  float4 v = p.epi == kQgResid ? *o : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  for (uint32_t j = 0; j < n; ++j) {
    const float4 a = __ldcg(reinterpret_cast<const float4 *>(p.part + (size_t)slots[j] * kBM * BN + idx));
    v.x += a.x;
    v.y += a.y;
    v.z += a.z;
    v.w += a.w;
  }
  *o = v;
}

template <uint32_t BN>
int launch_bn(const QgParams &p, const void *tmap, uint32_t grid, cudaStream_t st) {
  const CUtensorMap *m = reinterpret_cast<const CUtensorMap *>(tmap);
  if (p.prefetch == kQ8_0)
    return launch_pdl(k_qgemm<BN, kQ8_0>, dim3(grid), dim3(kQThreads), QCfg<BN, true>::kSmem, st, p, *m);
  if (p.prefetch == kQ4_0)
    return launch_pdl(k_qgemm<BN, kQ4_0>, dim3(grid), dim3(kQThreads), QCfg<BN, true>::kSmem, st, p, *m);
  if (p.prefetch == kPfAny)
    return launch_pdl(k_qgemm<BN, kPfAny>, dim3(grid), dim3(kQThreads), QCfg<BN, true>::kSmem, st, p, *m);
  return launch_pdl(k_qgemm<BN, 0>, dim3(grid), dim3(kQThreads), QCfg<BN, false>::kSmem, st, p, *m);
}
template <uint32_t BN, int PT>
bool set_smem() {
  return cudaFuncSetAttribute(k_qgemm<BN, PT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              QCfg<BN, PT != 0>::kSmem) == cudaSuccess;
}

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

}  // namespace

int qgemm_init() {
  if (!set_smem<64, 0>() || !set_smem<128, 0>() || !set_smem<256, 0>() || !set_smem<512, 0>() ||
      !set_smem<64, kQ8_0>() || !set_smem<128, kQ8_0>() || !set_smem<256, kQ8_0>() || !set_smem<512, kQ8_0>() ||
      !set_smem<64, kQ4_0>() || !set_smem<128, kQ4_0>() || !set_smem<256, kQ4_0>() || !set_smem<512, kQ4_0>() ||
      !set_smem<64, kPfAny>() || !set_smem<128, kPfAny>() || !set_smem<256, kPfAny>() || !set_smem<512, kPfAny>())
    return -1;
  if (!g_encode) {
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || !fn)
      return -1;
    g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  }
  return 0;
}

// f16 activations X[T_rows][K] (row stride K*2 bytes): tiles of 64 rows x bn
// tokens with the 128-byte swizzle; rows beyond T_rows read as zero
int qgemm_make_xmap(QgXMap *map, const void *x_f16, uint32_t K, uint32_t T_rows, uint32_t bn) {
  if (!g_encode || !map || !x_f16 || K % 8 || !T_rows || (bn != 64 && bn != 128 && bn != 256)) return -1;
  if (reinterpret_cast<uintptr_t>(x_f16) % 16) return -1;
  const cuuint64_t dims[2] = {K, T_rows};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {kBK, bn};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = g_encode(reinterpret_cast<CUtensorMap *>(map->bytes), CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                              const_cast<void *>(x_f16), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                              CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  map->bn = bn;
  return r == CUDA_SUCCESS ? 0 : -1;
}

uint64_t qgemm_part_floats(uint32_t bn, uint32_t n_sm) { return (uint64_t)2 * n_sm * kBM * bn; }

int launch_qgemm(const QgParams &p_in, const QgXMap &map, uint32_t n_sm, cudaStream_t st) {
  if (!p_in.T || !p_in.n_tiles || p_in.K % 16 || !p_in.w || !p_in.out || p_in.ldo % 4) return -1;  // fixup: float4 rows
  // red.add of split pieces only for 64-token tiles: a piece is 8K values
  // there (decode batches), but 64K in a 512-token pair, where the atomics
  // cost more than the fixup launch (measured: 2048-token prefill -16%)
  QgParams p0 = p_in;
  if (map.bn > 64) p0.red = 0;
  // more than one 256-token tile: token-tile pairs (one dequantised weight
  // stage per 512 tokens) over the same 256-row TMA boxes
  const uint32_t bn = (map.bn == 256 && p0.T > 256) ? 512 : map.bn;
  const uint32_t t_tiles = (p0.T + bn - 1) / bn, ksteps = (p0.K / 16 + 3) / 4;
  const uint64_t W = (uint64_t)p0.n_tiles * t_tiles * ksteps;
  const uint32_t grid = (uint32_t)std::max<uint64_t>(1, std::min<uint64_t>(n_sm, W / kMinSk));
  if (!p0.part || p0.part_floats < qgemm_part_floats(bn, grid) || ksteps + 1 > kFixupSlots) return -1;
  int rc;
  switch (bn) {
    case 64: rc = launch_bn<64>(p0, map.bytes, grid, st); break;
    case 128: rc = launch_bn<128>(p0, map.bytes, grid, st); break;
    case 256: rc = launch_bn<256>(p0, map.bytes, grid, st); break;
    case 512: rc = launch_bn<512>(p0, map.bytes, grid, st); break;
    default: return -1;
  }
  if (rc || grid < 2 || p0.red) return rc;
  return launch_pdl(k_qg_fixup, dim3(grid - 1, bn * kBM / 1024), dim3(256), 0, st, p0, bn, grid);
}

}  // namespace fa
