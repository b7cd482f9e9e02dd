// Sampler::sample (src/sampling.rs:110-152) on the device, one CTA of 1024
// threads per sequence row.  The reference's f32 arithmetic is kept step for
// step (no FMA contraction, the reference's summation orders):
//
//   adjust   repetition penalty (l > 0 ? l / pen : l * pen on seen ids),
//            frequency / presence penalty (l - fp*freq, then - pp), / T
//            (src/sampling.rs:175-219, :123-129)                       parallel
//   softmax  max fold, e = exp(l - max), sum in index order, e / sum
//            (src/sampling.rs:222-231)                      sum sequential
//   top-k    keep the k largest by (p desc, index asc): the stable sort of
//            src/sampling.rs:234-248, found by radix select
//   top-p    total in index order, cumulative p / total in sorted order,
//            zero from the first rank whose cumulative sum exceeds 0.999
//            (src/sampling.rs:251-280)
//   pick     T == 0 or all filtered <= 0: first index of the maximum
//            (src/sampling.rs:297-310); else r -= p in index order, first
//            i with r <= 0 (src/sampling.rs:283-294), r from Philox4x32-10
//            (seed of the row, counter = samples drawn so far)
//
// Sequential f32 sums (softmax total, top-p cumulative, the categorical walk)
// run on one warp in order.  A chunk of 32 terms that are each below half
// the gap to the running value's neighbour leaves it unchanged (every add
// rounds back), so such chunks are skipped; the result is the same float.
//
// exp is evaluated in double precision and rounded once to f32, i.e. the
// correctly rounded expf (up to double rounding of a 2^-52-close case);
// glibc's expf, which the reference calls, is within 0.502 ulp, so the two
// can differ in the last bit for a small fraction of arguments.
//
// Top-k above kSampleFastK and top-p without top-k sort the row's composite
// keys (~float_key(p) << 32 | index) with a bitonic sort in global scratch
// (shared-memory tiles for the inner stages).
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include "fa_device.cuh"
#include "fa_kernels.hpp"

namespace fa {
namespace {

constexpr uint32_t kST = 1024, kSW = 32;  // threads, warps
constexpr uint32_t kTile = 4096;          // bitonic tile (u64 keys) in shared memory
constexpr uint32_t kFull = 0xFFFFFFFFu;

struct SSmem {
  uint32_t whist[kSW][256];
  uint32_t hist[256];
  uint32_t cidx[kSampleFastK];
  float cp[kSampleFastK];
  unsigned long long tile[kTile];
  float redf[kSW];
  unsigned long long redk[kSW];
  uint32_t seq_tot[2][kSW], seq_qex[2][kSW];  // ordered scans (double-buffered)
  float seq_s;
  uint32_t seq_at;
  uint32_t seq_first[2][kSW];
  float seq_t[2][kSW];
  uint32_t wcnt[3][kSW];
  float sum, total;
  uint32_t prefix, remaining, cut, tok;
};

// ---- Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11): published round
// multipliers and Weyl key increments; uniform = top 24 bits of word 0 ----
__device__ __forceinline__ float philox_uniform(uint64_t seed, uint64_t step) {
  uint32_t c0 = (uint32_t)step, c1 = (uint32_t)(step >> 32), c2 = 0u, c3 = 0u;
  uint32_t k0 = (uint32_t)seed, k1 = (uint32_t)(seed >> 32);
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    const uint32_t lo0 = 0xD2511F53u * c0, hi0 = __umulhi(0xD2511F53u, c0);
    const uint32_t lo1 = 0xCD9E8D57u * c2, hi1 = __umulhi(0xCD9E8D57u, c2);
    const uint32_t n0 = hi1 ^ c1 ^ k0, n2 = hi0 ^ c3 ^ k1;
    c0 = n0;
    c1 = lo1;
    c2 = n2;
    c3 = lo0;
    k0 += 0x9E3779B9u;
    k1 += 0xBB67AE85u;
  }
  return (float)(c0 >> 8) * (1.0f / 16777216.0f);
}

// term t of a sequence handed to the ordered scans below
struct RowTerm {
  const float *v;
  __device__ float operator()(uint32_t i) const { return __ldcg(v + i); }
};
struct SortedTerm {  // p[index of rank i] / total
  const float *v;
  const unsigned long long *keys;
  float total;
  __device__ float operator()(uint32_t i) const {
    return __fdiv_rn(__ldcg(v + (uint32_t)(__ldcg(keys + i) & 0xFFFFFFFFull)), total);
  }
};

// ---- ordered f32 scans, block-parallel and bit-exact ----
// The reference accumulates in index order, s(i+1) = fl(s(i) + t(i)).  While
// s stays inside one binade [2^e, 2^(e+1)) every partial sum is a multiple of
// that binade's spacing g, and fl(s + t) = s + g * rn(t / g) exactly unless
// t / g lies exactly halfway between integers (the tie goes to the even
// multiple, which depends on s) or the rounded sum leaves the binade.  So the
// scan runs as an integer prefix sum of q(i) = rn(t(i) / g) over a tile of
// the sequence; at the first index where the prefix would leave the binade,
// where a tie occurs, or where t is not a finite non-negative float, the
// partial sum is formed exactly (its bit pattern plus the integer prefix) and
// that one step is taken in f32 as the reference does; the scan then resumes
// after it with the new binade.  The walk mode runs the reference's
// categorical draw r(i+1) = fl(r(i) - p(i)) the same way, downwards.
enum : int { kSeqSum = 0, kSeqStop = 1, kSeqWalk = 2 };
constexpr uint32_t kMlp = 8;     // loads in flight per thread in the streaming passes
constexpr uint32_t kMlpW = 4;    // warp-wide iterations loaded ahead in the top-k passes
constexpr uint32_t kSeqPer = 8;
constexpr uint32_t kSeqSat = 1u << 30;  // saturation of the scan's integer prefixes
constexpr uint32_t kSeqHead = 2048;     // leading terms one lane adds in order
__device__ __forceinline__ uint32_t sat_add(uint32_t a, uint32_t b) { return min(a + b, kSeqSat); }  // terms per thread per tile (after the first tile)

// q = rn(t / g) for g = 2^(ue - 150) (ue = max(biased exponent, 1) of the
// accumulator), t finite and >= 0; tie: t / g is exactly halfway
__device__ __forceinline__ uint32_t grid_units(uint32_t tb, uint32_t ue, bool &tie) {
  const uint32_t et = tb >> 23;
  const uint32_t m = et ? (tb & 0x7FFFFFu) | 0x800000u : tb;
  const uint32_t e = et ? et : 1u;
  tie = false;
  if (e >= ue) return e - ue >= 8 ? 0x80000000u : m << (e - ue);  // >= 2^31 ends the binade anyway
  const uint32_t sh = ue - e;
  if (sh >= 32) return 0u;
  const uint32_t rem = m & ((1u << sh) - 1u), half = 1u << (sh - 1);
  tie = rem == half;
  return (m >> sh) + (rem > half ? 1u : 0u);
}

struct SeqOut {
  float s;      // final accumulator (kSeqWalk: r)
  uint32_t at;  // kSeqStop: first i with s > stop; kSeqWalk: first i with r <= 0; n if none
};

// Whole block.  kSeqSum: s = fl(..fl(s0 + t(0)).. + t(n-1)); kSeqStop: the
// same scan ended at the first i where s > stop; kSeqWalk: r = s0 > 0 minus
// the terms in order, ended at the first i where r <= 0.
template <int MODE, class Term>
__device__ SeqOut block_seq(Term term, uint32_t n, float s0, float stop, SSmem &sm) {
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float s = s0;
  uint32_t par = 0;
  // The first kSeqHead terms are added in order by one lane from shared
  // memory: early on the running sum is small against the terms, so binade
  // crossings and ties (each a rescan of the rest of a tile) come every few
  // terms there, while a plain f32 chain costs a few cycles per term.
  const uint32_t hn = min(n, kSeqHead);
  if (hn) {
    float *hs = reinterpret_cast<float *>(sm.tile);
    for (uint32_t i = tid; i < hn; i += kST) hs[i] = term(i);
    __syncthreads();
    if (tid == 0) {
      float r = s0;
      uint32_t at = n;
      for (uint32_t i = 0; i < hn; ++i) {
        r = MODE == kSeqWalk ? __fsub_rn(r, hs[i]) : __fadd_rn(r, hs[i]);
        if ((MODE == kSeqStop && r > stop) || (MODE == kSeqWalk && r <= 0.0f)) {
          at = i;
          break;
        }
      }
      sm.seq_s = r;
      sm.seq_at = at;
    }
    __syncthreads();
    s = sm.seq_s;
    const uint32_t at = sm.seq_at;
    __syncthreads();  // the staging area and seq_s/seq_at are free again
    if (at != n) return {s, at};
  }
  for (uint32_t t0 = hn, per = kSeqPer; t0 < n; t0 += kST * per) {
    const uint32_t tend = min(n, t0 + kST * per), j0 = t0 + tid * per;
    float x[kSeqPer];
#pragma unroll
    for (uint32_t e = 0; e < kSeqPer; ++e) x[e] = e < per && j0 + e < tend ? term(j0 + e) : 0.0f;
    uint32_t i = t0;
    while (i < tend) {
      const uint32_t sb = __float_as_uint(s);
      if (s != s) return {s, n};  // NaN stays NaN (and is never > stop or <= 0)
      // kind 0: on the binade grid; 1: s == 0 (next step at the first nonzero
      // term); 2: s == +inf (next step at the first NaN term)
      int kind = 0;
      uint32_t ue = 1, room = 0;
      if (MODE != kSeqWalk && s == 0.0f) {
        kind = 1;
      } else if (MODE != kSeqWalk && sb == 0x7F800000u) {
        kind = 2;
      } else {
        const uint32_t es = sb >> 23, m = es ? (sb & 0x7FFFFFu) | 0x800000u : sb;
        ue = es ? es : 1u;
        room = MODE == kSeqWalk ? (es >= 2 ? m - 0x800000u : m) : 0x1000000u - m;
      }
      uint32_t q[kSeqPer];
      bool st[kSeqPer];
      uint32_t tot = 0;
#pragma unroll
      for (uint32_t e = 0; e < kSeqPer; ++e) {
        const uint32_t j = j0 + e, tb = __float_as_uint(x[e]);
        const bool valid = e < per && j >= i && j < tend;
        q[e] = 0u;
        st[e] = false;
        if (valid) {
          if (kind == 1) {
            st[e] = x[e] != 0.0f;
          } else if (kind == 2) {
            st[e] = x[e] != x[e];
          } else if ((tb >> 23) >= 255u) {  // negative, inf or NaN: the f32 step decides
            st[e] = true;
          } else {
            bool tie;
            q[e] = grid_units(tb, ue, tie);
            st[e] = tie;
          }
        }
        q[e] = min(q[e], kSeqSat);
        tot = sat_add(tot, q[e]);
      }
      // block exclusive prefix of the per-thread totals, saturating at
      // kSeqSat: a saturated prefix is only ever compared with room (< 2^25),
      // and min(prefix, kSeqSat) keeps every such comparison exact
      uint32_t inc = tot;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t u = __shfl_up_sync(kFull, inc, o);
        if ((int)lane >= o) inc = sat_add(inc, u);
      }
      const uint32_t t_ex = __shfl_up_sync(kFull, inc, 1);
      if (lane == 31) sm.seq_tot[par][warp] = inc;
      __syncthreads();
      uint32_t winc = sm.seq_tot[par][lane];
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t u = __shfl_up_sync(kFull, winc, o);
        if ((int)lane >= o) winc = sat_add(winc, u);
      }
      const uint32_t block_tot = __shfl_sync(kFull, winc, 31);
      const uint32_t w_ex = __shfl_up_sync(kFull, winc, 1);
      const uint32_t wexcl = __shfl_sync(kFull, lane ? w_ex : 0u, warp);
      uint32_t Q = sat_add(wexcl, lane ? t_ex : 0u);  // exclusive prefix at this thread's first term
      uint32_t first = ~0u;
      uint32_t qex = 0;
      float tf = 0.0f;
#pragma unroll
      for (uint32_t e = 0; e < kSeqPer; ++e) {
        const uint32_t Qi = sat_add(Q, q[e]);
        bool stp = st[e];
        if (kind == 0 && !stp && e < per && (j0 + e) >= i && (j0 + e) < tend) {
          stp = Qi >= room;
          if (MODE == kSeqStop && !stp) stp = __uint_as_float(sb + (uint32_t)Qi) > stop;
        }
        if (stp && first == ~0u) {
          first = j0 + e;
          qex = Q;
          tf = x[e];
        }
        Q = Qi;
      }
      const uint32_t bal = __ballot_sync(kFull, first != ~0u);
      if (bal) {
        if (lane == (uint32_t)(__ffs(bal) - 1)) {
          sm.seq_first[par][warp] = first;
          sm.seq_qex[par][warp] = qex;
          sm.seq_t[par][warp] = tf;
        }
      } else if (lane == 0) {
        sm.seq_first[par][warp] = ~0u;
      }
      __syncthreads();
      const uint32_t f = sm.seq_first[par][lane];
      const uint32_t fmin = __reduce_min_sync(kFull, f);
      if (fmin == ~0u) {  // no step of its own in the rest of the tile
        if (kind == 0) s = __uint_as_float(MODE == kSeqWalk ? sb - (uint32_t)block_tot : sb + (uint32_t)block_tot);
        i = tend;
      } else {
        const uint32_t w = __ffs(__ballot_sync(kFull, f == fmin)) - 1;
        const uint32_t qx = sm.seq_qex[par][w];
        const float t = sm.seq_t[par][w];
        float base = s;
        if (kind == 0) base = __uint_as_float(MODE == kSeqWalk ? sb - (uint32_t)qx : sb + (uint32_t)qx);
        s = MODE == kSeqWalk ? __fsub_rn(base, t) : __fadd_rn(base, t);
        if (MODE == kSeqStop && s > stop) return {s, fmin};
        if (MODE == kSeqWalk && s <= 0.0f) return {s, fmin};
        i = fmin + 1;
      }
      par ^= 1u;
    }
  }
  return {s, n};
}

__device__ __forceinline__ void cmpx(unsigned long long &a, unsigned long long &b, bool up) {
  if ((a > b) == up) {
    const unsigned long long t = a;
    a = b;
    b = t;
  }
}

// bitonic stages (k, j from jmax down to 1) of the n-key tile at global
// offset t0 (direction from the global index); whole block
__device__ void tile_stages(unsigned long long *tile, uint32_t n, uint32_t t0, uint32_t k, uint32_t jmax) {
  for (uint32_t j = jmax; j > 0; j >>= 1) {
    for (uint32_t q = threadIdx.x; q < n / 2; q += kST) {
      const uint32_t i = 2 * q - (q & (j - 1)), l = i + j;
      cmpx(tile[i], tile[l], ((t0 + i) & k) == 0);
    }
    __syncthreads();
  }
}

// ascending bitonic sort of N (power of two) keys in global memory
__device__ void bitonic_global(unsigned long long *a, uint32_t N, unsigned long long *tile) {
  const uint32_t T = N < kTile ? N : kTile;
  for (uint32_t t0 = 0; t0 < N; t0 += T) {
    for (uint32_t i = threadIdx.x; i < T; i += kST) tile[i] = __ldcg(a + t0 + i);
    __syncthreads();
    for (uint32_t k = 2; k <= T; k <<= 1) tile_stages(tile, T, t0, k, k >> 1);
    for (uint32_t i = threadIdx.x; i < T; i += kST) __stcg(a + t0 + i, tile[i]);
    __syncthreads();
  }
  for (uint32_t k = 2 * T; k <= N; k <<= 1) {
    for (uint32_t j = k >> 1; j >= T; j >>= 1) {
      for (uint32_t q = threadIdx.x; q < N / 2; q += kST) {
        const uint32_t i = 2 * q - (q & (j - 1)), l = i + j;
        unsigned long long x = __ldcg(a + i), y = __ldcg(a + l);
        cmpx(x, y, (i & k) == 0);
        __stcg(a + i, x);
        __stcg(a + l, y);
      }
      __syncthreads();
    }
    for (uint32_t t0 = 0; t0 < N; t0 += T) {
      for (uint32_t i = threadIdx.x; i < T; i += kST) tile[i] = __ldcg(a + t0 + i);
      __syncthreads();
      tile_stages(tile, T, t0, k, T >> 1);
      for (uint32_t i = threadIdx.x; i < T; i += kST) __stcg(a + t0 + i, tile[i]);
      __syncthreads();
    }
  }
}

__device__ __forceinline__ unsigned long long sort_key(float p, uint32_t i) {
  return ((unsigned long long)(~float_key(p)) << 32) | i;  // ascending = p desc, index asc
}

__device__ float block_max(float v, SSmem &sm) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(kFull, v, o));
  if ((threadIdx.x & 31) == 0) sm.redf[threadIdx.x >> 5] = v;
  __syncthreads();
  float m = sm.redf[0];
  for (uint32_t w = 1; w < kSW; ++w) m = fmaxf(m, sm.redf[w]);
  __syncthreads();
  return m;
}

__device__ unsigned long long block_max_u64(unsigned long long v, SSmem &sm) {
#pragma unroll
  for (int o = 16; o; o >>= 1) {
    const unsigned long long u = __shfl_xor_sync(kFull, v, o);
    v = u > v ? u : v;
  }
  if ((threadIdx.x & 31) == 0) sm.redk[threadIdx.x >> 5] = v;
  __syncthreads();
  unsigned long long m = sm.redk[0];
  for (uint32_t w = 1; w < kSW; ++w) m = sm.redk[w] > m ? sm.redk[w] : m;
  __syncthreads();
  return m;
}

// exclusive prefix over the 32 warps' counts sm.wcnt[c] (in place), by warp 0
__device__ void warp_counts_scan(SSmem &sm, int c, uint32_t lane) {
  uint32_t v = sm.wcnt[c][lane], inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t u = __shfl_up_sync(kFull, inc, o);
    if ((int)lane >= o) inc += u;
  }
  sm.wcnt[c][lane] = inc - v;
}

// Top-k candidates of row pr[0, n) into sm.cidx / sm.cp in index order
// (k <= kSampleFastK): radix select of the k-th largest float_key(p), then
// every key above it and the lowest-index ties up to k.
__device__ void select_top_k(const float *pr, uint32_t n, uint32_t k, SSmem &sm) {
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  uint32_t prefix = 0, mask = 0, remaining = k;
  for (int d = 3; d >= 0; --d) {
    for (uint32_t i = tid; i < kSW * 256; i += kST) (&sm.whist[0][0])[i] = 0u;
    __syncthreads();
    for (uint32_t base0 = warp * 32; base0 < n; base0 += kST * kMlpW) {
      uint32_t keys[kMlpW];  // kMlpW iterations' loads in flight
#pragma unroll
      for (uint32_t u = 0; u < kMlpW; ++u) {
        const uint32_t i = base0 + u * kST + lane;
        keys[u] = i < n ? float_key(__ldcg(pr + i)) : 0u;
      }
#pragma unroll
      for (uint32_t u = 0; u < kMlpW; ++u) {
        const uint32_t i = base0 + u * kST + lane, key = keys[u];
        const bool in = i < n && (key & mask) == prefix;
        if (!__any_sync(kFull, in)) continue;  // after the first pass most warps hold no candidate
        const uint32_t b = (key >> (8 * d)) & 255u;
        const uint32_t peers = __match_any_sync(kFull, in ? b : 256u + lane);
        if (in && lane == (uint32_t)(__ffs(peers) - 1)) sm.whist[warp][b] += __popc(peers);
      }
    }
    __syncthreads();
    if (tid < 256) {
      uint32_t c = 0;
      for (uint32_t w = 0; w < kSW; ++w) c += sm.whist[w][tid];
      sm.hist[tid] = c;
    }
    __syncthreads();
    if (tid == 0) {
      uint32_t above = 0;
      for (int b = 255; b >= 0; --b) {
        if (above + sm.hist[b] >= remaining) {
          sm.remaining = remaining - above;
          sm.prefix = prefix | ((uint32_t)b << (8 * d));
          break;
        }
        above += sm.hist[b];
      }
    }
    __syncthreads();
    prefix = sm.prefix;
    remaining = sm.remaining;
    mask |= 255u << (8 * d);
  }
  const uint32_t thr = prefix, need = remaining;  // need >= 1 ties of key thr are kept
  // warp w owns indices [lo, hi): counts of keys above / equal to thr
  const uint32_t R = (n + kST - 1) / kST * 32, lo = min(n, warp * R), hi = min(n, lo + R);
  uint32_t gt = 0, eq = 0;
  for (uint32_t base0 = lo; base0 < hi; base0 += 32 * kMlpW) {
    uint32_t keys[kMlpW];
#pragma unroll
    for (uint32_t u = 0; u < kMlpW; ++u) {
      const uint32_t i = base0 + 32 * u + lane;
      keys[u] = i < hi ? float_key(__ldcg(pr + i)) : 0u;
    }
#pragma unroll
    for (uint32_t u = 0; u < kMlpW; ++u) {
      const uint32_t i = base0 + 32 * u + lane;
      gt += __popc(__ballot_sync(kFull, i < hi && keys[u] > thr));
      eq += __popc(__ballot_sync(kFull, i < hi && keys[u] == thr));
    }
  }
  if (lane == 0) {
    sm.wcnt[0][warp] = gt;
    sm.wcnt[1][warp] = eq;
  }
  __syncthreads();
  if (warp == 0) warp_counts_scan(sm, 1, lane);  // ties before this warp
  __syncthreads();
  const uint32_t eq_before = sm.wcnt[1][warp];
  const uint32_t take = eq_before >= need ? 0u : min(eq, need - eq_before);
  if (lane == 0) sm.wcnt[2][warp] = gt + take;
  __syncthreads();
  if (warp == 0) warp_counts_scan(sm, 2, lane);  // output offset of this warp
  __syncthreads();
  uint32_t out = sm.wcnt[2][warp], eq_seen = 0;
  const uint32_t lt = (1u << lane) - 1u;
  for (uint32_t base0 = lo; base0 < hi; base0 += 32 * kMlpW) {
    float pvs[kMlpW];
#pragma unroll
    for (uint32_t u = 0; u < kMlpW; ++u) {
      const uint32_t i = base0 + 32 * u + lane;
      pvs[u] = i < hi ? __ldcg(pr + i) : 0.0f;
    }
#pragma unroll
    for (uint32_t u = 0; u < kMlpW; ++u) {  // in index order: ties are taken lowest index first
      const uint32_t i = base0 + 32 * u + lane;
      const float pv = pvs[u];
      const uint32_t key = float_key(pv);
      const uint32_t beq = __ballot_sync(kFull, i < hi && key == thr);
      const bool keep = i < hi && (key > thr || (key == thr && eq_seen + __popc(beq & lt) < take));
      const uint32_t bk = __ballot_sync(kFull, keep);
      if (keep) {
        const uint32_t o = out + __popc(bk & lt);
        sm.cidx[o] = i;
        sm.cp[o] = pv;
      }
      out += __popc(bk);
      eq_seen += __popc(beq);
    }
  }
  __syncthreads();
}

__global__ void __launch_bounds__(kST, 1) k_sample(const SamplerParams p) {
  pdl_enter();
  extern __shared__ __align__(16) uint8_t smem_raw[];
  SSmem &sm = *reinterpret_cast<SSmem *>(smem_raw);
  const uint32_t tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const uint32_t row = p.row0 + blockIdx.x;
  if (p.state) {  // decode loop: the logits of prompt steps are discarded
    const uint32_t done = p.state->step;
    if (done == 0 || done - 1 < p.sample_from) return;
  }
  const uint32_t n = p.n;
  const float *lg = p.logits + (size_t)blockIdx.x * p.ld;
  float *pr = p.probs + (size_t)row * p.vocab;
  const uint32_t *fq = p.freq + (size_t)row * p.vocab;
  const bool rep = p.rep != 1.0f, fpp = !(p.freq_pen == 0.0f && p.pres_pen == 0.0f);
  const bool temp = p.temperature > 0.0f && p.temperature != 1.0f;
  // The elementwise passes stream the row through L2 with kMlp independent
  // loads in flight per thread (one CTA per row would otherwise wait a full
  // memory latency per element it handles).
  // 1-3: adjusted logits and their maximum
  float mx = -INFINITY;
  for (uint32_t i0 = tid; i0 < n; i0 += kST * kMlp) {
    float lv[kMlp];
    uint32_t fv[kMlp];
#pragma unroll
    for (uint32_t j = 0; j < kMlp; ++j) {
      const uint32_t i = i0 + j * kST;
      lv[j] = i < n ? lg[i] : 0.0f;
      fv[j] = (rep || fpp) && i < n ? fq[i] : 0u;
    }
#pragma unroll
    for (uint32_t j = 0; j < kMlp; ++j) {
      const uint32_t i = i0 + j * kST;
      if (i >= n) break;
      float l = lv[j];
      const uint32_t f = fv[j];
      if (rep && f) l = l > 0.0f ? __fdiv_rn(l, p.rep) : __fmul_rn(l, p.rep);
      if (fpp && f) {
        l = __fsub_rn(l, __fmul_rn(p.freq_pen, (float)f));
        l = __fsub_rn(l, p.pres_pen);
      }
      if (temp) l = __fdiv_rn(l, p.temperature);
      __stcg(pr + i, l);
      mx = fmaxf(mx, l);
    }
  }
  mx = block_max(mx, sm);
  // 4: softmax
  for (uint32_t i0 = tid; i0 < n; i0 += kST * kMlp) {
    float v[kMlp];
#pragma unroll
    for (uint32_t j = 0; j < kMlp; ++j) v[j] = i0 + j * kST < n ? __ldcg(pr + i0 + j * kST) : 0.0f;
#pragma unroll
    for (uint32_t j = 0; j < kMlp; ++j)
      if (i0 + j * kST < n) __stcg(pr + i0 + j * kST, __double2float_rn(exp((double)__fsub_rn(v[j], mx))));
  }
  __syncthreads();
  const float sum = block_seq<kSeqSum>(RowTerm{pr}, n, 0.0f, 0.0f, sm).s;
  if (sum != 0.0f)
    for (uint32_t i0 = tid; i0 < n; i0 += kST * kMlp) {
      float v[kMlp];
#pragma unroll
      for (uint32_t j = 0; j < kMlp; ++j) v[j] = i0 + j * kST < n ? __ldcg(pr + i0 + j * kST) : 0.0f;
#pragma unroll
      for (uint32_t j = 0; j < kMlp; ++j)
        if (i0 + j * kST < n) __stcg(pr + i0 + j * kST, __fdiv_rn(v[j], sum));
    }
  __syncthreads();
  const bool topk = p.top_k > 0 && p.top_k < n, topp = p.top_p > 0.0f && p.top_p < 1.0f;
  const bool greedy = p.temperature == 0.0f;
  uint32_t tok = 0;
  if (topk && p.top_k <= kSampleFastK) {
    // ---- fast path: k candidates in index order ----
    select_top_k(pr, n, p.top_k, sm);
    const uint32_t m = p.top_k;
    if (topp) {
      if (tid == 0) {  // total in index order (the other entries are zero)
        float t = 0.0f;
        for (uint32_t j = 0; j < m; ++j) t = __fadd_rn(t, sm.cp[j]);
        sm.total = t;
      }
      __syncthreads();
      const float total = sm.total;
      if (total > 0.0f) {
        uint32_t P2 = 2;
        while (P2 < m) P2 <<= 1;
        for (uint32_t j = tid; j < P2; j += kST) sm.tile[j] = j < m ? sort_key(sm.cp[j], j) : ~0ull;
        __syncthreads();
        for (uint32_t k = 2; k <= P2; k <<= 1) tile_stages(sm.tile, P2, 0, k, k >> 1);
        if (tid == 0) {
          float cum = 0.0f;
          uint32_t cut = m;
          for (uint32_t r = 0; r < m; ++r) {
            cum = __fadd_rn(cum, __fdiv_rn(sm.cp[sm.tile[r] & 0xFFFFFFFFull], total));
            if (cum > 0.999f) {
              cut = r;
              break;
            }
          }
          sm.cut = cut;
        }
        __syncthreads();
        for (uint32_t r = sm.cut + tid; r < m; r += kST) sm.cp[sm.tile[r] & 0xFFFFFFFFull] = 0.0f;
        __syncthreads();
      }
    }
    if (tid == 0) {
      float best = 0.0f;
      uint32_t bj = ~0u;
      for (uint32_t j = 0; j < m; ++j)
        if (sm.cp[j] > best) {
          best = sm.cp[j];
          bj = j;
        }
      const uint32_t amax = bj == ~0u ? 0u : sm.cidx[bj];  // all zero: the first index
      if (greedy || bj == ~0u) {
        tok = amax;
      } else {
        float r = philox_uniform(p.seeds[row], p.counters[row]);
        tok = amax;
        if (!(r > 0.0f)) {
          tok = 0;
        } else {
          for (uint32_t j = 0; j < m; ++j) {
            r = __fsub_rn(r, sm.cp[j]);
            if (r <= 0.0f) {
              tok = sm.cidx[j];
              break;
            }
          }
        }
      }
      sm.tok = tok;
    }
  } else {
    // ---- whole-row path ----
    if (topk || topp) {
      unsigned long long *keys = p.keys + (size_t)row * p.pow2;
      for (uint32_t i = tid; i < p.pow2; i += kST) __stcg(keys + i, i < n ? sort_key(__ldcg(pr + i), i) : ~0ull);
      __syncthreads();
      bitonic_global(keys, p.pow2, sm.tile);
      if (topk)
        for (uint32_t r = p.top_k + tid; r < n; r += kST) __stcg(pr + (uint32_t)(__ldcg(keys + r) & 0xFFFFFFFFull), 0.0f);
      __syncthreads();
      if (topp) {
        const float t = block_seq<kSeqSum>(RowTerm{pr}, n, 0.0f, 0.0f, sm).s;
        const uint32_t cut = t > 0.0f ? block_seq<kSeqStop>(SortedTerm{pr, keys, t}, n, 0.0f, 0.999f, sm).at : n;
        for (uint32_t r = cut + tid; r < n; r += kST) __stcg(pr + (uint32_t)(__ldcg(keys + r) & 0xFFFFFFFFull), 0.0f);
        __syncthreads();
      }
    }
    // first index of the maximum
    unsigned long long best = 0ull;
    for (uint32_t i = tid; i < n; i += kST) {
      const unsigned long long kk = ((unsigned long long)float_key(__ldcg(pr + i)) << 32) | (unsigned long long)(~i);
      best = kk > best ? kk : best;
    }
    best = block_max_u64(best, sm);
    const uint32_t amax = ~(uint32_t)(best & 0xFFFFFFFFull);
    const bool all_zero = !(key_float((uint32_t)(best >> 32)) > 0.0f);
    if (greedy || all_zero) {
      if (tid == 0) sm.tok = amax;
    } else {
      const float r = philox_uniform(p.seeds[row], p.counters[row]);
      uint32_t t = r > 0.0f ? block_seq<kSeqWalk>(RowTerm{pr}, n, r, 0.0f, sm).at : 0u;
      if (t >= n) t = amax;
      if (tid == 0) sm.tok = t;
    }
  }
  __syncthreads();
  if (tid == 0) {
    tok = sm.tok;
    if (p.ids) p.ids[row] = tok;
    p.counters[row] += 1;
    if (p.state) {
      const uint32_t s = p.state->step - 1;
      p.state->token = tok;
      if (p.gen_ids && s < p.max_ids) p.gen_ids[s] = tok;
    }
    if (p.observe && tok < p.vocab) p.freq[(size_t)row * p.vocab + tok] += 1;
  }
}

__global__ void k_sampler_observe(uint32_t *freq, uint32_t vocab, uint32_t seq, uint32_t token) {
  freq[(size_t)seq * vocab + token] += 1;
}

}  // namespace

int sampler_init() {
  return cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(SSmem)) == cudaSuccess
             ? 0
             : -1;
}

int launch_sample(const SamplerParams &p, uint32_t rows, cudaStream_t st) {
  if (!rows || !p.n || p.n > p.vocab) return -1;
  if (sample_needs_sort(p) && (!p.keys || p.pow2 < p.n)) return -1;
  return launch_pdl(k_sample, dim3(rows), dim3(kST), sizeof(SSmem), st, p);
}

int launch_sampler_observe(uint32_t *freq, uint32_t vocab, uint32_t seq, uint32_t token, cudaStream_t st) {
  k_sampler_observe<<<1, 1, 0, st>>>(freq, vocab, seq, token);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace fa
