// Stream-K dequant-GEMV for batch-1 decode: y[N] = x[K] . W[K][N] with W in
// the chunked row-group layout (fa_layout.hpp) — the reference's
// tensor::matmul orientation (src/tensor.rs:244-258), quant blocks along N.
//
// One persistent CTA per SM streams a contiguous, byte-balanced range of the
// weight's 8-row groups (possibly spanning chunks).  A producer warp moves
// each stage (weight groups + the matching x / norm-weight slices) with 1-D
// bulk TMA copies into a 4-slot shared-memory ring; the weight copies of the
// first slots are issued before griddepcontrol.wait, so with programmatic
// dependent launch this kernel's weight stream starts while the previous
// kernel drains.  Eight consumer warps dequantise with byte-permute "magic
// float" tricks and packed FFMA2 (lane j owns 32 columns of one row per
// step).  When a CTA finishes its rows of a chunk it publishes the chunk
// partial; the last CTA to arrive (atomic counter) sums the partials in a
// fixed order (deterministic) and runs the fused epilogue: residual add +
// sum of squares, RoPE + KV append, SwiGLU, or logits + argmax.
#include <cuda_runtime.h>

#include "fa_device.cuh"
#include "fa_kernels.hpp"
#include "gemv_epi.cuh"

namespace fa {

namespace {

constexpr int kConsumerWarps = 16;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kStages = 4;
constexpr uint32_t kHeaderBytes = 128;

__device__ __forceinline__ uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

// 0.5 + q/32 for the 4-bit code held (shifted left by 3) in byte b of v
__device__ __forceinline__ float magic_hi(uint32_t v, uint32_t sel) { return __uint_as_float(__byte_perm(v, 0x3F000000u, sel)); }

// ---------------------------------------------------------------------------
// per-type row kernels: accumulate one row (x) of a lane's 32 columns.
// Every kind keeps acc such that y_e = scale * acc[e] - corr[e / 16], with
// acc held as 16 float2 pairs (columns 2p, 2p+1) fed to packed FFMA2.
// ---------------------------------------------------------------------------
struct Acc {
  float2 a[16];
  float c0, c1;
};

// per-lane constants of a chunk (lane j of the row owns columns 32j..32j+31)
struct LaneK {
  uint32_t j;      // 32-column lane index within the chunk
  uint32_t sb;     // sub-block within its 256-column super-block (K-quants)
  uint32_t fw;     // Q4_K: word (0..2) of the 96-bit scale field block
  uint32_t fs;     // Q4_K: bit shift of the 12-bit field inside words fw, fw+1
};

__device__ __forceinline__ void ffma2v(float2 &acc, float xs, float f0, float f1) {
  acc = __ffma2_rn(make_float2(xs, xs), make_float2(f0, f1), acc);
}

// 4-bit codes in the lane format (byte i: col i low nibble, col i+16 high)
// -> acc += xs * (0.5 + q/32) for the 16 low and 16 high columns
__device__ __forceinline__ void acc_nibbles(const uint4 c, float xs_lo, float xs_hi, Acc &A) {
  const uint32_t wv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
  for (int t = 0; t < 4; ++t) {
    const uint32_t lo3 = (wv[t] * 8u) & 0x78787878u, hi3 = __umulhi(wv[t], 0x80000000u) & 0x78787878u;
    ffma2v(A.a[2 * t + 0], xs_lo, magic_hi(lo3, 0x7044), magic_hi(lo3, 0x7144));
    ffma2v(A.a[2 * t + 1], xs_lo, magic_hi(lo3, 0x7244), magic_hi(lo3, 0x7344));
    ffma2v(A.a[8 + 2 * t + 0], xs_hi, magic_hi(hi3, 0x7044), magic_hi(hi3, 0x7144));
    ffma2v(A.a[8 + 2 * t + 1], xs_hi, magic_hi(hi3, 0x7244), magic_hi(hi3, 0x7344));
  }
}

template <int T>
struct RowOp;

// Q4_K: value = (d*sc)*q - dmin*m ; F = 0.5 + q/32 -> y = 32*acc - sum(16*xs + x*dmin*m).
// The device header keeps d, dmin and re-lays the 12 scale bytes as eight
// 12-bit fields (sc | m << 6) so a lane reaches its own with one funnel shift.
template <>
struct RowOp<kQ4_K> {
  static constexpr float kScale = 32.0f;
  __device__ __forceinline__ static void run(const uint8_t *G, uint32_t w, uint32_t r, const LaneK &lk, float x,
                                             Acc &A) {
    const uint4 c = *reinterpret_cast<const uint4 *>(G + r * (w / 2) + 16 * lk.j);
    const uint4 h = *reinterpret_cast<const uint4 *>(G + 4 * w + (r * (w / 256) + (lk.j >> 3)) * 16);
    const uint32_t lo = lk.fw == 0 ? h.y : (lk.fw == 1 ? h.z : h.w);
    const uint32_t hi = lk.fw == 0 ? h.z : h.w;
    const uint32_t f = __funnelshift_r(lo, hi, lk.fs);
    const float sc = __uint_as_float((f & 63u) | 0x4B000000u) - 8388608.0f;
    const float m = __uint_as_float(((f >> 6) & 63u) | 0x4B000000u) - 8388608.0f;
    const float2 dd = __half22float2(*reinterpret_cast<const __half2 *>(&h.x));
    const float xs = x * (dd.x * sc);
    const float xm = x * (dd.y * m);
    A.c0 += fmaf(16.0f, xs, xm);
    acc_nibbles(c, xs, xs, A);
  }
};

// Q4_0: value = d*(q-8) -> y = 32*acc - 24*sum(x*d)
template <>
struct RowOp<kQ4_0> {
  static constexpr float kScale = 32.0f;
  __device__ __forceinline__ static void run(const uint8_t *G, uint32_t w, uint32_t r, const LaneK &lk, float x,
                                             Acc &A) {
    const uint4 c = *reinterpret_cast<const uint4 *>(G + r * (w / 2) + 16 * lk.j);
    const float d = h2f(*reinterpret_cast<const uint16_t *>(G + 4 * w + (r * (w / 32) + lk.j) * 2));
    const float xd = x * d;
    A.c0 = fmaf(24.0f, xd, A.c0);
    acc_nibbles(c, xd, xd, A);
  }
};

// Q4_1: value = d*q + m ; F = 0.5 + q/32 -> y = 32*acc - sum(16*x*d - x*m)
template <>
struct RowOp<kQ4_1> {
  static constexpr float kScale = 32.0f;
  __device__ __forceinline__ static void run(const uint8_t *G, uint32_t w, uint32_t r, const LaneK &lk, float x,
                                             Acc &A) {
    const uint4 c = *reinterpret_cast<const uint4 *>(G + r * (w / 2) + 16 * lk.j);
    const uint8_t *dp = G + 4 * w + (r * (w / 32) + lk.j) * 2;
    const float d = h2f(*reinterpret_cast<const uint16_t *>(dp)), m = h2f(*reinterpret_cast<const uint16_t *>(dp + w / 2));
    const float xd = x * d;
    A.c0 += fmaf(16.0f, xd, -x * m);
    acc_nibbles(c, xd, xd, A);
  }
};

// Q5_0: value = d*(q-16), q = nibble | fifth bit << 4 ; F = 0.5 + q/64 (the
// 5-bit code at bits 2-6 of the byte) -> y = 64*acc - 48*sum(x*d)
template <>
struct RowOp<kQ5_0> {
  static constexpr float kScale = 64.0f;
  // bits 0-3 of v -> bit 6 of bytes 0-3
  __device__ __forceinline__ static uint32_t spread4(uint32_t v) { return ((v * 0x00204081u) & 0x01010101u) << 6; }
  __device__ __forceinline__ static void run(const uint8_t *G, uint32_t w, uint32_t r, const LaneK &lk, float x,
                                             Acc &A) {
    const uint4 c = *reinterpret_cast<const uint4 *>(G + r * (w / 2) + 16 * lk.j);
    const uint32_t qh = *reinterpret_cast<const uint32_t *>(G + 4 * w + (r * (w / 32) + lk.j) * 4);
    const float d = h2f(*reinterpret_cast<const uint16_t *>(G + 5 * w + (r * (w / 32) + lk.j) * 2));
    const float xd = x * d;
    A.c0 = fmaf(48.0f, xd, A.c0);
    const uint32_t wv[4] = {c.x, c.y, c.z, c.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t lo = ((wv[t] << 2) & 0x3C3C3C3Cu) | spread4((qh >> (4 * t)) & 0xFu);
      const uint32_t hi = ((wv[t] >> 2) & 0x3C3C3C3Cu) | spread4((qh >> (16 + 4 * t)) & 0xFu);
      ffma2v(A.a[2 * t + 0], xd, magic_hi(lo, 0x7044), magic_hi(lo, 0x7144));
      ffma2v(A.a[2 * t + 1], xd, magic_hi(lo, 0x7244), magic_hi(lo, 0x7344));
      ffma2v(A.a[8 + 2 * t + 0], xd, magic_hi(hi, 0x7044), magic_hi(hi, 0x7144));
      ffma2v(A.a[8 + 2 * t + 1], xd, magic_hi(hi, 0x7244), magic_hi(hi, 0x7344));
    }
  }
};

// Q6_K: value = (d*sc)*(q-32) ; F = 0.5 + q/128 -> y = 128*acc - 96*sum(xs)
template <>
struct RowOp<kQ6_K> {
  static constexpr float kScale = 128.0f;
  __device__ __forceinline__ static void run(const uint8_t *G, uint32_t w, uint32_t r, const LaneK &lk, float x,
                                             Acc &A) {
    const uint32_t j = lk.j;
    const uint4 ql = *reinterpret_cast<const uint4 *>(G + r * (w / 2) + 16 * j);
    const uint2 qh = *reinterpret_cast<const uint2 *>(G + 4 * w + r * (w / 4) + 8 * j);
    const uint32_t scw = *reinterpret_cast<const uint16_t *>(G + 6 * w + r * (w / 16) + 2 * j);
    const float d = h2f(*reinterpret_cast<const uint16_t *>(G + 6 * w + w / 2 + (r * (w / 256) + (j >> 3)) * 2));
    const int sc0 = (int)(int8_t)(scw & 0xFFu), sc1 = (int)(int8_t)(scw >> 8);  // exact int -> float below
    const float s0 = __int_as_float(0x4B400000 + sc0) - 12582912.0f, s1 = __int_as_float(0x4B400000 + sc1) - 12582912.0f;
    const float xd = x * d;
    const float xs0 = xd * s0, xs1 = xd * s1;
    A.c0 = fmaf(96.0f, xs0, A.c0);
    A.c1 = fmaf(96.0f, xs1, A.c1);
    const uint32_t wv[4] = {ql.x, ql.y, ql.z, ql.w};
    const uint32_t Q[2] = {qh.x, qh.y};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t q = Q[t & 1];
      // low-nibble columns 4t..4t+3: high bits at shift 2*(t>>1); high-nibble columns 16+4t..: shift 4+2*(t>>1)
      const uint32_t vl = ((wv[t] << 1) & 0x1E1E1E1Eu) | ((t < 2 ? (q << 5) : (q << 3)) & 0x60606060u);
      const uint32_t vh = ((wv[t] >> 3) & 0x1E1E1E1Eu) | ((t < 2 ? (q << 1) : (q >> 1)) & 0x60606060u);
      ffma2v(A.a[2 * t + 0], xs0, magic_hi(vl, 0x7044), magic_hi(vl, 0x7144));
      ffma2v(A.a[2 * t + 1], xs0, magic_hi(vl, 0x7244), magic_hi(vl, 0x7344));
      ffma2v(A.a[8 + 2 * t + 0], xs1, magic_hi(vh, 0x7044), magic_hi(vh, 0x7144));
      ffma2v(A.a[8 + 2 * t + 1], xs1, magic_hi(vh, 0x7244), magic_hi(vh, 0x7344));
    }
  }
};

// Q8_0: value = d*q, u = q+128 ; F = 1 + u/256 -> y = 256*acc - 384*sum(x*d)
template <>
struct RowOp<kQ8_0> {
  static constexpr float kScale = 256.0f;
  __device__ __forceinline__ static void run(const uint8_t *G, uint32_t w, uint32_t r, const LaneK &lk, float x,
                                             Acc &A) {
    const uint4 c0 = *reinterpret_cast<const uint4 *>(G + r * w + 32 * lk.j);
    const uint4 c1 = *reinterpret_cast<const uint4 *>(G + r * w + 32 * lk.j + 16);
    const float d = h2f(*reinterpret_cast<const uint16_t *>(G + 8 * w + (r * (w / 32) + lk.j) * 2));
    const float xd = x * d;
    A.c0 = fmaf(384.0f, xd, A.c0);
    const uint32_t wv[8] = {c0.x, c0.y, c0.z, c0.w, c1.x, c1.y, c1.z, c1.w};
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const uint32_t u = wv[t] ^ 0x80808080u;
      ffma2v(A.a[2 * t + 0], xd, __uint_as_float(((u << 15) & 0x007F8000u) | 0x3F800000u),
             __uint_as_float(((u << 7) & 0x007F8000u) | 0x3F800000u));
      ffma2v(A.a[2 * t + 1], xd, __uint_as_float(((u >> 1) & 0x007F8000u) | 0x3F800000u),
             __uint_as_float(((u >> 9) & 0x007F8000u) | 0x3F800000u));
    }
  }
};

template <>
struct RowOp<kF16> {
  static constexpr float kScale = 1.0f;
  __device__ __forceinline__ static void run(const uint8_t *G, uint32_t w, uint32_t r, const LaneK &lk, float x,
                                             Acc &A) {
    const uint4 *p = reinterpret_cast<const uint4 *>(G + r * 2 * w + 64 * lk.j);
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint4 v = p[t];
      const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&wv[q]));
        A.a[4 * t + q] = __ffma2_rn(make_float2(x, x), f, A.a[4 * t + q]);
      }
    }
  }
};

template <>
struct RowOp<kF32> {
  static constexpr float kScale = 1.0f;
  __device__ __forceinline__ static void run(const uint8_t *G, uint32_t w, uint32_t r, const LaneK &lk, float x,
                                             Acc &A) {
    const float4 *p = reinterpret_cast<const float4 *>(G + r * 4 * w + 128 * lk.j);
#pragma unroll
    for (int t = 0; t < 8; ++t) {
      const float4 v = p[t];
      A.a[2 * t + 0] = __ffma2_rn(make_float2(x, x), make_float2(v.x, v.y), A.a[2 * t + 0]);
      A.a[2 * t + 1] = __ffma2_rn(make_float2(x, x), make_float2(v.z, v.w), A.a[2 * t + 1]);
    }
  }
};

struct Smem {
  uint64_t *full, *empty;
  uint32_t *flag;
  float *red;        // 32 floats of block-reduction scratch
  uint8_t *stages;   // kStages x stage_bytes
  float *xs;         // kStages x x_slot
  float *nw;         // kStages x x_slot (norm weights, rmsnorm prologue)
  float *warp_part;  // kConsumerWarps x CW
};

__device__ __forceinline__ Smem carve(uint8_t *smem, const GemvParams &p) {
  Smem s;
  s.full = reinterpret_cast<uint64_t *>(smem);
  s.empty = s.full + kStages;
  s.flag = reinterpret_cast<uint32_t *>(smem + 64);
  s.red = reinterpret_cast<float *>(smem + kHeaderBytes);  // 128 floats
  uint32_t off = kHeaderBytes + 512;
  s.stages = smem + off;
  off += kStages * p.stage_bytes;
  s.xs = reinterpret_cast<float *>(smem + off);
  off += kStages * p.x_slot * 4;
  s.nw = reinterpret_cast<float *>(smem + off);
  off += kStages * p.x_slot * 4;
  s.warp_part = reinterpret_cast<float *>(smem + off);
  return s;
}

__device__ __forceinline__ void consumer_bar() { epi::consumer_bar<kConsumerWarps>(); }

// stage enumeration shared by producer and consumers: a stage holds up to NG
// groups of one chunk; (c, g) walks the CTA's [start, end) range.
struct StageIt {
  uint32_t c, g, ng, gend;
  bool last_of_chunk;
};
__device__ __forceinline__ uint32_t stage_ng(const GemvParams &p, const ChunkDesc &cd) {
  return max(1u, min(p.stage_bytes / cd.gbytes, p.x_slot / 8));
}
__device__ __forceinline__ bool stage_first(const GemvParams &p, const CtaRange &R, StageIt &it) {
  it.c = R.c0;
  it.g = R.g0;
  const uint32_t gtot = p.K8 / 8;
  if (it.c > R.c1 || (it.c == R.c1 && it.g >= R.g1)) return false;
  it.gend = it.c == R.c1 ? R.g1 : gtot;
  it.ng = min(stage_ng(p, p.chunks[it.c]), it.gend - it.g);
  it.last_of_chunk = it.g + it.ng == it.gend;
  return true;
}
__device__ __forceinline__ bool stage_next(const GemvParams &p, const CtaRange &R, StageIt &it) {
  const uint32_t gtot = p.K8 / 8;
  it.g += it.ng;
  if (it.g >= it.gend) {
    it.c += 1;
    it.g = 0;
  }
  if (it.c > R.c1 || (it.c == R.c1 && it.g >= R.g1)) return false;
  it.gend = it.c == R.c1 ? R.g1 : gtot;
  it.ng = min(stage_ng(p, p.chunks[it.c]), it.gend - it.g);
  it.last_of_chunk = it.g + it.ng == it.gend;
  return true;
}

template <int T>
__device__ __forceinline__ void stage_rows(const GemvParams &p, const uint8_t *base, const float *xrow, const float *nrow,
                                           float inv, uint32_t ngs, uint32_t w, uint32_t gb, uint32_t G, uint32_t gl,
                                           uint32_t warp, const LaneK &lk, Acc &A) {
  const uint32_t steps = ngs * 8 / G;
  const bool norm = p.pro == kProRmsNorm;
  uint32_t step = warp;
  for (; step + kConsumerWarps < steps; step += 2 * kConsumerWarps) {
    const uint32_t r0 = step * G + gl, r1 = (step + kConsumerWarps) * G + gl;
    float x0 = xrow[r0], x1 = xrow[r1];
    if (norm) {
      x0 = __fmul_rn(__fmul_rn(x0, inv), nrow[r0]);
      x1 = __fmul_rn(__fmul_rn(x1, inv), nrow[r1]);
    }
    RowOp<T>::run(base + (r0 >> 3) * gb, w, r0 & 7u, lk, x0, A);
    RowOp<T>::run(base + (r1 >> 3) * gb, w, r1 & 7u, lk, x1, A);
  }
  if (step < steps) {
    const uint32_t r0 = step * G + gl;
    float x0 = xrow[r0];
    if (norm) x0 = __fmul_rn(__fmul_rn(x0, inv), nrow[r0]);
    RowOp<T>::run(base + (r0 >> 3) * gb, w, r0 & 7u, lk, x0, A);
  }
}

template <int T>
__device__ __forceinline__ void finalize(const Acc &A, float vals[32]) {
  constexpr bool two_corr = T == kQ6_K;
#pragma unroll
  for (int e = 0; e < 16; ++e) {
    const float c = (two_corr && e >= 8) ? A.c1 : A.c0;
    vals[2 * e] = RowOp<T>::kScale * A.a[e].x - c;
    vals[2 * e + 1] = RowOp<T>::kScale * A.a[e].y - c;
  }
}

// publish this CTA's partial of chunk c; the last contributor reduces and
// runs the epilogue
template <int T>
__device__ __forceinline__ void flush(const GemvParams &p, const Smem &sm, const ChunkDesc &cd, uint32_t c,
                                      const Acc &A, uint32_t warp, uint32_t lane, uint32_t tid) {
  float vals[32];
  finalize<T>(A, vals);
  const uint32_t lanes_per_row = p.CW / 32;
  for (uint32_t o = lanes_per_row; o < 32; o <<= 1) {
#pragma unroll
    for (int e = 0; e < 32; ++e) vals[e] += __shfl_xor_sync(0xFFFFFFFFu, vals[e], o);
  }
  if (lane < lanes_per_row) {
#pragma unroll
    for (int e = 0; e < 32; ++e) sm.warp_part[warp * p.CW + lane * 32 + e] = vals[e];
  }
  consumer_bar();
  const uint32_t slot = blockIdx.x * p.max_chunks_per_cta + (c - p.ranges[blockIdx.x].c0);
  float *dst = p.part + (size_t)slot * p.CW;
  for (uint32_t col = tid; col < cd.width; col += kConsumerWarps * 32) {
    float s = 0.0f;
#pragma unroll
    for (int wv = 0; wv < kConsumerWarps; ++wv) s += sm.warp_part[wv * p.CW + col];
    __stcg(dst + col, s);
  }
  __threadfence();
  consumer_bar();
  if (tid == 0) {
    const uint32_t old = atomicAdd(p.counters + c, 1u);
    *sm.flag = (old + 1 == cd.n_contrib) ? 1u : 0u;
  }
  consumer_bar();
  if (*sm.flag) {
    __threadfence();
    epi::epilogue<kConsumerWarps>(p, sm.red, sm.warp_part, p.contrib + cd.contrib_off, cd, c, tid, warp, lane);
    if (tid == 0) p.counters[c] = 0;  // ready for the next launch
  }
  consumer_bar();
}

template <int T>
__device__ __forceinline__ void zero(Acc &A) {
#pragma unroll
  for (int e = 0; e < 16; ++e) A.a[e] = make_float2(0.0f, 0.0f);
  A.c0 = A.c1 = 0.0f;
}

}  // namespace

__global__ void __launch_bounds__(kThreads, 1) k_gemv(const GemvParams p) {
  extern __shared__ __align__(128) uint8_t smem[];
  const Smem sm = carve(smem, p);
  const uint32_t tid = threadIdx.x, warp = tid / 32, lane = tid % 32;
  const CtaRange R = p.ranges[blockIdx.x];
  const bool norm = p.pro == kProRmsNorm;

  if (tid == 0) {
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&sm.full[i], 1);
      mbar_init(&sm.empty[i], kConsumerWarps);
    }
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  bool ok = true;
  if (warp == kConsumerWarps) {
    // ---------------- producer ----------------
    if (lane == 0) {
      StageIt it;
      uint32_t s = 0;
      bool more = stage_first(p, R, it);
      // weights of the first slots before waiting on the previous kernel
      for (; more && s < kStages; ++s) {
        const ChunkDesc &cd = p.chunks[it.c];
        const uint32_t wb = it.ng * cd.gbytes, xb = it.ng * 32 * (norm ? 2 : 1);
        mbar_arrive_expect_tx(&sm.full[s], wb + xb);
        bulk_g2s(sm.stages + s * p.stage_bytes, p.w + cd.offset + (uint64_t)it.g * cd.gbytes, wb, &sm.full[s]);
        more = stage_next(p, R, it);
      }
      pdl_wait();
      {  // activations of those slots
        StageIt jt;
        bool m2 = stage_first(p, R, jt);
        for (uint32_t t = 0; m2 && t < s; ++t) {
          const uint32_t k = jt.g * 8;
          bulk_g2s(sm.xs + t * p.x_slot, p.in + k, jt.ng * 32, &sm.full[t]);
          if (norm) bulk_g2s(sm.nw + t * p.x_slot, p.norm_w + k, jt.ng * 32, &sm.full[t]);
          m2 = stage_next(p, R, jt);
        }
      }
      for (; more; ++s) {
        const uint32_t slot = s % kStages;
        if (!mbar_wait(&sm.empty[slot], ((s / kStages) - 1) & 1u)) {
          ok = false;
          break;
        }
        fence_proxy_async_smem();
        const ChunkDesc &cd = p.chunks[it.c];
        const uint32_t wb = it.ng * cd.gbytes, xb = it.ng * 32 * (norm ? 2 : 1);
        mbar_arrive_expect_tx(&sm.full[slot], wb + xb);
        bulk_g2s(sm.stages + slot * p.stage_bytes, p.w + cd.offset + (uint64_t)it.g * cd.gbytes, wb, &sm.full[slot]);
        const uint32_t k = it.g * 8;
        bulk_g2s(sm.xs + slot * p.x_slot, p.in + k, it.ng * 32, &sm.full[slot]);
        if (norm) bulk_g2s(sm.nw + slot * p.x_slot, p.norm_w + k, it.ng * 32, &sm.full[slot]);
        more = stage_next(p, R, it);
      }
    } else {
      pdl_wait();
    }
  } else {
    // ---------------- consumers ----------------
    pdl_wait();
    if (norm) {
      if (warp == 0) {
        float s = 0.0f;
        for (uint32_t i = lane; i < p.n_ssq; i += 32) s += p.ssq[i];
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
        if (lane == 0) sm.red[96] = 1.0f / sqrtf(s / (float)p.K + p.eps);
      }
      consumer_bar();
    }
    const float inv = norm ? sm.red[96] : 1.0f;
    const uint32_t lanes_per_row = p.CW / 32, G = 32 / lanes_per_row, gl = lane / lanes_per_row;
    LaneK lk;
    lk.j = lane % lanes_per_row;
    lk.sb = lk.j & 7;
    lk.fw = (12 * lk.sb) / 32;
    lk.fs = (12 * lk.sb) % 32;
    Acc A;
    zero<0>(A);
    StageIt it;
    uint32_t s = 0;
    for (bool more = stage_first(p, R, it); more; more = stage_next(p, R, it), ++s) {
      const uint32_t slot = s % kStages;
      if (!mbar_wait(&sm.full[slot], (s / kStages) & 1u)) {
        ok = false;
        break;
      }
      const ChunkDesc cd = p.chunks[it.c];
      const bool active = lk.j < cd.width / 32u;
      const uint8_t *base = sm.stages + slot * p.stage_bytes;
      const float *xrow = sm.xs + slot * p.x_slot, *nrow = sm.nw + slot * p.x_slot;
      if (active) {
        switch (cd.type) {
          case kQ4_K: stage_rows<kQ4_K>(p, base, xrow, nrow, inv, it.ng, cd.width, cd.gbytes, G, gl, warp, lk, A); break;
          case kQ6_K: stage_rows<kQ6_K>(p, base, xrow, nrow, inv, it.ng, cd.width, cd.gbytes, G, gl, warp, lk, A); break;
          case kQ8_0: stage_rows<kQ8_0>(p, base, xrow, nrow, inv, it.ng, cd.width, cd.gbytes, G, gl, warp, lk, A); break;
          case kQ4_0: stage_rows<kQ4_0>(p, base, xrow, nrow, inv, it.ng, cd.width, cd.gbytes, G, gl, warp, lk, A); break;
          case kQ4_1: stage_rows<kQ4_1>(p, base, xrow, nrow, inv, it.ng, cd.width, cd.gbytes, G, gl, warp, lk, A); break;
          case kQ5_0: stage_rows<kQ5_0>(p, base, xrow, nrow, inv, it.ng, cd.width, cd.gbytes, G, gl, warp, lk, A); break;
          case kF16: stage_rows<kF16>(p, base, xrow, nrow, inv, it.ng, cd.width, cd.gbytes, G, gl, warp, lk, A); break;
          default: stage_rows<kF32>(p, base, xrow, nrow, inv, it.ng, cd.width, cd.gbytes, G, gl, warp, lk, A); break;
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&sm.empty[slot]);
      if (it.last_of_chunk) {
        switch (cd.type) {
          case kQ4_K: flush<kQ4_K>(p, sm, cd, it.c, A, warp, lane, tid); break;
          case kQ6_K: flush<kQ6_K>(p, sm, cd, it.c, A, warp, lane, tid); break;
          case kQ8_0: flush<kQ8_0>(p, sm, cd, it.c, A, warp, lane, tid); break;
          case kQ4_0: flush<kQ4_0>(p, sm, cd, it.c, A, warp, lane, tid); break;
          case kQ4_1: flush<kQ4_1>(p, sm, cd, it.c, A, warp, lane, tid); break;
          case kQ5_0: flush<kQ5_0>(p, sm, cd, it.c, A, warp, lane, tid); break;
          case kF16: flush<kF16>(p, sm, cd, it.c, A, warp, lane, tid); break;
          default: flush<kF32>(p, sm, cd, it.c, A, warp, lane, tid); break;
        }
        zero<0>(A);
      }
    }
  }
  if (!ok && p.state) atomicOr(&p.state->err, kErrWaitTimeout);
}

size_t gemv_smem_bytes(const GemvParams &p) {
  return kHeaderBytes + 512 + (size_t)kStages * p.stage_bytes + (size_t)kStages * p.x_slot * 8 +
         (size_t)kConsumerWarps * p.CW * 4;
}

int gemv_init() {
  if (cudaFuncSetAttribute(k_gemv, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess) return -1;
  return 0;
}

int launch_gemv(const GemvParams &p, bool pdl, cudaStream_t st) {
  if (p.mma) return launch_gemv_mma(p, pdl, st);
  // the red.add epilogue, the SwiGLU prologue and buffer clearing exist on
  // the tensor-core path only
  if (p.epi == kEpiRed || p.pro == kProSwiglu || p.zero) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.n_ctas);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = gemv_smem_bytes(p);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, k_gemv, p) == cudaSuccess ? 0 : -1;
}

}  // namespace fa
