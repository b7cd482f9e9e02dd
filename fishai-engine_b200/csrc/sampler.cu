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

// half the gap from s >= 0 to the next float above / from r > 0 to the next
// float below (NaN for inf; 0 where the half gap underflows)
__device__ __forceinline__ float half_gap_up(float s) {
  return __fmul_rn(__fsub_rn(__int_as_float(__float_as_int(s) + 1), s), 0.5f);
}
__device__ __forceinline__ float half_gap_down(float r) {
  return __fmul_rn(__fsub_rn(r, __int_as_float(__float_as_int(r) - 1)), 0.5f);
}

// term t of a sequence handed to the warp scans below
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

// s = fl(..fl(fl(s + t(0)) + t(1)).. + t(n-1)) for terms >= 0, by one warp;
// with stop > 0 the scan ends at the first i where s > stop and *at = i.
// The terms of the next 256 are loaded while the current 256 are added.
template <class Term>
__device__ float warp_seq_sum(Term t, uint32_t n, float s, uint32_t lane, float stop, uint32_t *at) {
  float nx[8];
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const uint32_t i = 32 * b + lane;
    nx[b] = i < n ? t(i) : 0.0f;
  }
  for (uint32_t c0 = 0; c0 < n; c0 += 256) {
    float x[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      x[b] = nx[b];
      const uint32_t i = c0 + 256 + 32 * b + lane;
      nx[b] = i < n ? t(i) : 0.0f;
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      if (c0 + 32 * b >= n) break;
      const float h = half_gap_up(s);
      if (__any_sync(kFull, !(x[b] < h))) {
        for (int j = 0; j < 32; ++j) {
          s = __fadd_rn(s, __shfl_sync(kFull, x[b], j));
          if (stop > 0.0f && s > stop) {
            *at = c0 + 32 * b + j;
            return s;
          }
        }
      }
    }
  }
  return s;
}

// categorical_sample's walk: first i with fl(r - p0 - .. - pi) <= 0 (in
// order), n if none; r > 0
__device__ uint32_t warp_seq_categorical(const float *v, uint32_t n, float r, uint32_t lane) {
  float nx[8];
#pragma unroll
  for (int b = 0; b < 8; ++b) {
    const uint32_t i = 32 * b + lane;
    nx[b] = i < n ? __ldcg(v + i) : 0.0f;
  }
  for (uint32_t c0 = 0; c0 < n; c0 += 256) {
    float x[8];
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      x[b] = nx[b];
      const uint32_t i = c0 + 256 + 32 * b + lane;
      nx[b] = i < n ? __ldcg(v + i) : 0.0f;
    }
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      if (c0 + 32 * b >= n) break;
      const float h = half_gap_down(r);
      if (__any_sync(kFull, !(x[b] < h))) {
        for (int j = 0; j < 32; ++j) {
          r = __fsub_rn(r, __shfl_sync(kFull, x[b], j));
          if (r <= 0.0f) return c0 + 32 * b + j;
        }
      }
    }
  }
  return n;
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
    for (uint32_t base = warp * 32; base < n; base += kST) {
      const uint32_t i = base + lane;
      const uint32_t key = i < n ? float_key(__ldcg(pr + i)) : 0u;
      const bool in = i < n && (key & mask) == prefix;
      const uint32_t b = (key >> (8 * d)) & 255u;
      const uint32_t peers = __match_any_sync(kFull, in ? b : 256u + lane);
      if (in && lane == (uint32_t)(__ffs(peers) - 1)) sm.whist[warp][b] += __popc(peers);
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
  for (uint32_t base = lo; base < hi; base += 32) {
    const uint32_t i = base + lane;
    const uint32_t key = i < hi ? float_key(__ldcg(pr + i)) : 0u;
    gt += __popc(__ballot_sync(kFull, i < hi && key > thr));
    eq += __popc(__ballot_sync(kFull, i < hi && key == thr));
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
  for (uint32_t base = lo; base < hi; base += 32) {
    const uint32_t i = base + lane;
    const float pv = i < hi ? __ldcg(pr + i) : 0.0f;
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
  __syncthreads();
}

__global__ void __launch_bounds__(kST, 1) k_sample(const SamplerParams p) {
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
  // 1-3: adjusted logits and their maximum
  float mx = -INFINITY;
  for (uint32_t i = tid; i < n; i += kST) {
    float l = lg[i];
    const uint32_t f = (rep || fpp) ? fq[i] : 0u;
    if (rep && f) l = l > 0.0f ? __fdiv_rn(l, p.rep) : __fmul_rn(l, p.rep);
    if (fpp && f) {
      l = __fsub_rn(l, __fmul_rn(p.freq_pen, (float)f));
      l = __fsub_rn(l, p.pres_pen);
    }
    if (temp) l = __fdiv_rn(l, p.temperature);
    __stcg(pr + i, l);
    mx = fmaxf(mx, l);
  }
  mx = block_max(mx, sm);
  // 4: softmax
  for (uint32_t i = tid; i < n; i += kST) __stcg(pr + i, __double2float_rn(exp((double)__fsub_rn(__ldcg(pr + i), mx))));
  __syncthreads();
  if (warp == 0) {
    uint32_t at = 0;
    const float s = warp_seq_sum(RowTerm{pr}, n, 0.0f, lane, 0.0f, &at);
    if (lane == 0) sm.sum = s;
  }
  __syncthreads();
  const float sum = sm.sum;
  if (sum != 0.0f)
    for (uint32_t i = tid; i < n; i += kST) __stcg(pr + i, __fdiv_rn(__ldcg(pr + i), sum));
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
        if (warp == 0) {
          uint32_t at = 0;
          const float t = warp_seq_sum(RowTerm{pr}, n, 0.0f, lane, 0.0f, &at);
          uint32_t cut = n;
          if (t > 0.0f) warp_seq_sum(SortedTerm{pr, keys, t}, n, 0.0f, lane, 0.999f, &cut);
          if (lane == 0) sm.cut = t > 0.0f ? cut : n;
        }
        __syncthreads();
        for (uint32_t r = sm.cut + tid; r < n; r += kST) __stcg(pr + (uint32_t)(__ldcg(keys + r) & 0xFFFFFFFFull), 0.0f);
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
    } else if (warp == 0) {
      const float r = philox_uniform(p.seeds[row], p.counters[row]);
      uint32_t t = r > 0.0f ? warp_seq_categorical(pr, n, r, lane) : 0u;
      if (t >= n) t = amax;
      if (lane == 0) sm.tok = t;
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
  k_sample<<<rows, kST, sizeof(SSmem), st>>>(p);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int launch_sampler_observe(uint32_t *freq, uint32_t vocab, uint32_t seq, uint32_t token, cudaStream_t st) {
  k_sampler_observe<<<1, 1, 0, st>>>(freq, vocab, seq, token);
  return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

}  // namespace fa
