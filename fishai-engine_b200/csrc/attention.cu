// Decode attention over the paged KV cache (split-K "flash decode").
//
// Reference: scaled_dot_product_attention with the cache expanded per query
// head (src/model.rs:374-394, src/tensor.rs:451-551): s = (q.k)*scale,
// softmax over every cached position, o = sum p*v; GQA query head h reads kv
// head h / (H/KVH) (expand_kv_heads, src/model.rs:500-526) — no copy here,
// the kv head is indexed directly.  Grid (splits, KVH); a CTA handles all
// query heads of one kv head over one contiguous slice of positions, keeps
// an online softmax per head and writes (max, sum, unnormalised o) partials
// that the o-projection GEMV combines in its prologue.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include "fa_dequant.cuh"
#include "fa_device.cuh"
#include "fa_kernels.hpp"

namespace fa {

namespace {
constexpr int kWarps = 4;
constexpr int kMaxRep = 8;   // query heads per kv head

template <bool F16>
__device__ __forceinline__ float kv_load(const void *base, uint64_t idx) {
  if (F16) return __half2float(reinterpret_cast<const __half *>(base)[idx]);
  return reinterpret_cast<const float *>(base)[idx];
}

template <bool F16, int REP, int DPL>
__device__ void attn_body(const AttnParams &p) {
  const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const uint32_t split = blockIdx.x, kvh = blockIdx.y;
  const uint32_t hd = p.kv.head_dim, KVH = p.kv.n_kv;
  constexpr uint32_t rep = REP, dpl = DPL;
  const uint32_t row = blockIdx.z;
  const uint32_t T = p.kc ? p.t_fixed : p.state->len + 1;
  const float *qrow = p.q + (uint64_t)row * p.n_heads * hd;
  float *part = p.part + (uint64_t)row * p.n_heads * p.splits * (2 + hd);
  uint32_t *counters = p.counters + (uint64_t)row * KVH;
  float *outrow = p.out + (uint64_t)row * p.n_heads * hd;
  uint32_t L = (T + p.splits - 1) / p.splits;
  L = (L + 15) / 16 * 16;
  const uint32_t t0 = split * L, t1 = min(T, t0 + L);
  __shared__ float sm_m[kWarps][REP], sm_l[kWarps][REP];
  __shared__ float sm_o[kWarps][REP][DPL * 32];

  float q[REP][DPL];
  for (uint32_t r = 0; r < rep; ++r)
    for (uint32_t i = 0; i < dpl; ++i) {
      const uint32_t d = lane + 32 * i;
      q[r][i] = d < hd ? qrow[(kvh * rep + r) * hd + d] : 0.0f;
    }
  float m[REP], l[REP], o[REP][DPL];
#pragma unroll
  for (uint32_t r = 0; r < REP; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.0f;
#pragma unroll
    for (uint32_t i = 0; i < DPL; ++i) o[r][i] = 0.0f;
  }
  const void *base = p.kc ? nullptr
                         : reinterpret_cast<const uint8_t *>(p.kv.base) + (uint64_t)p.layer * p.kv.layer_stride * (F16 ? 2 : 4);
  const uint32_t *pt = p.kc ? nullptr : p.kv.page_table + (uint64_t)p.seq * p.kv.max_pages;
  for (uint32_t t = t0 + warp; t < t1; t += kWarps) {
    float kk[DPL], vv[DPL];
    if (p.kc) {
      const uint64_t rb = ((uint64_t)t * KVH + kvh) * hd;
      for (uint32_t i = 0; i < dpl; ++i) {
        const uint32_t d = lane + 32 * i;
        kk[i] = d < hd ? p.kc[rb + d] : 0.0f;
        vv[i] = d < hd ? p.vc[rb + d] : 0.0f;
      }
    } else {
      const uint32_t page = pt[t / 16], slot = t % 16;
      for (uint32_t i = 0; i < dpl; ++i) {
        const uint32_t d = lane + 32 * i;
        kk[i] = d < hd ? kv_load<F16>(base, kv_index(page, 0, kvh, slot, d, KVH, hd)) : 0.0f;
        vv[i] = d < hd ? kv_load<F16>(base, kv_index(page, 1, kvh, slot, d, KVH, hd)) : 0.0f;
      }
    }
    for (uint32_t r = 0; r < rep; ++r) {
      float s = 0.0f;
      for (uint32_t i = 0; i < dpl; ++i) s = fmaf(q[r][i], kk[i], s);
#pragma unroll
      for (int off = 16; off; off >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, off);
      s *= p.scale;
      const float mn = fmaxf(m[r], s);
      const float a = expf(m[r] - mn), b = expf(s - mn);
      l[r] = fmaf(l[r], a, b);
      for (uint32_t i = 0; i < dpl; ++i) o[r][i] = fmaf(o[r][i], a, b * vv[i]);
      m[r] = mn;
    }
  }
  // merge the warps (fixed order)
  for (uint32_t r = 0; r < rep; ++r) {
    if (lane == 0) {
      sm_m[warp][r] = m[r];
      sm_l[warp][r] = l[r];
    }
    for (uint32_t i = 0; i < dpl; ++i) {
      const uint32_t d = lane + 32 * i;
      if (d < hd) sm_o[warp][r][d] = o[r][i];
    }
  }
  __syncthreads();
  for (uint32_t idx = threadIdx.x; idx < rep * (hd + 2); idx += blockDim.x) {
    const uint32_t r = idx / (hd + 2), c = idx % (hd + 2);
    float M = -INFINITY;
    for (int wv = 0; wv < kWarps; ++wv) M = fmaxf(M, sm_m[wv][r]);
    float out;
    if (c == 0) {
      out = M;
    } else {
      float acc = 0.0f;
      for (int wv = 0; wv < kWarps; ++wv) {
        const float mw = sm_m[wv][r];
        if (mw == -INFINITY) continue;
        const float e = expf(mw - M);
        acc = fmaf(c == 1 ? sm_l[wv][r] : sm_o[wv][r][c - 2], e, acc);
      }
      out = acc;
    }
    const uint32_t h = kvh * rep + r;
    part[((uint64_t)h * p.splits + split) * (2 + hd) + c] = out;
  }
  // the last split CTA of this kv head combines all splits (fixed order)
  __threadfence();
  __syncthreads();
  __shared__ uint32_t last;
  if (threadIdx.x == 0) last = atomicAdd(counters + kvh, 1u) + 1 == p.splits;
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (uint32_t idx = threadIdx.x; idx < rep * hd; idx += blockDim.x) {
    const uint32_t r = idx / hd, dd = idx % hd, h = kvh * rep + r;
    const float *P = part + (uint64_t)h * p.splits * (2 + hd);
    float M = -INFINITY;
    for (uint32_t s = 0; s < p.splits; ++s) M = fmaxf(M, __ldcg(P + s * (2 + hd)));
    float Lsum = 0.0f, o = 0.0f;
    for (uint32_t s = 0; s < p.splits; ++s) {
      const float m = __ldcg(P + s * (2 + hd));
      if (m == -INFINITY) continue;
      const float e = expf(m - M);
      Lsum = fmaf(__ldcg(P + s * (2 + hd) + 1), e, Lsum);
      o = fmaf(__ldcg(P + s * (2 + hd) + 2 + dd), e, o);
    }
    outrow[h * hd + dd] = o / Lsum;
  }
  if (threadIdx.x == 0) counters[kvh] = 0;
}

template <bool F16, int REP, int DPL>
__global__ void __launch_bounds__(kWarps * 32) k_attention(const AttnParams p) {
  pdl_launch_dependents();
  pdl_wait();
  attn_body<F16, REP, DPL>(p);
}

template <int REP>
void *pick_dpl(uint32_t hd, bool f16) {
  if (hd <= 32) return f16 ? (void *)k_attention<true, REP, 1> : (void *)k_attention<false, REP, 1>;
  if (hd <= 64) return f16 ? (void *)k_attention<true, REP, 2> : (void *)k_attention<false, REP, 2>;
  return f16 ? (void *)k_attention<true, REP, 4> : (void *)k_attention<false, REP, 4>;
}
}  // namespace

int launch_attention(const AttnParams &p, bool pdl, cudaStream_t st) {
  const uint32_t rep = p.n_heads / p.kv.n_kv;
  if (p.kv.head_dim > 128 || rep > kMaxRep || p.n_heads % p.kv.n_kv) return -1;
  const bool f16 = p.kv.f16 != 0;
  void *fn = rep == 1 ? pick_dpl<1>(p.kv.head_dim, f16)
             : rep == 2 ? pick_dpl<2>(p.kv.head_dim, f16)
             : rep == 4 ? pick_dpl<4>(p.kv.head_dim, f16)
             : rep == 8 ? pick_dpl<8>(p.kv.head_dim, f16) : nullptr;
  if (!fn) return -1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(p.splits, p.kv.n_kv, p.q_rows ? p.q_rows : 1);
  cfg.blockDim = dim3(kWarps * 32);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  void *args[] = {(void *)&p};
  return cudaLaunchKernelExC(&cfg, fn, args) == cudaSuccess ? 0 : -1;
}

// ---------------------------------------------------------------------------
// embedding gather (src/model.rs:338-343) + sum-of-squares partials
// ---------------------------------------------------------------------------

namespace {
__global__ void k_embed(const EmbedParams p) {
  pdl_launch_dependents();
  pdl_wait();
  const uint32_t fed = p.state->fed;
  uint32_t tok = (p.feed && fed < p.state->n_feed) ? p.feed[fed] : p.state->token;
  if (tok >= p.vocab) {
    if (threadIdx.x == 0 && blockIdx.x == 0) atomicOr(&p.state->err, kErrBadToken);
    tok = 0;
  }
  if (threadIdx.x == 0 && blockIdx.x == 0) p.state->argmax_key = 0ull;
  const uint32_t per = (p.d + gridDim.x - 1) / gridDim.x;
  const uint32_t c0 = blockIdx.x * per, c1 = min(p.d, c0 + per);
  float s = 0.0f;
  for (uint32_t i = c0 + threadIdx.x; i < c1; i += blockDim.x) {
    const float v = dequant_native_elem(p.type, p.emb, (uint64_t)tok * p.d + i);
    p.x[i] = v;
    s = fmaf(v, v, s);
  }
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
  __shared__ float red[32];
  if (threadIdx.x % 32 == 0) red[threadIdx.x / 32] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.0f;
    for (uint32_t i = 0; i < blockDim.x / 32; ++i) t += red[i];
    p.ssq_out[blockIdx.x] = t;
  }
}

__global__ void k_step_end(SeqState *st, uint32_t *ids, uint32_t max_ids) {
  pdl_launch_dependents();
  pdl_wait();
  const unsigned long long key = st->argmax_key;
  const uint32_t tok = ~(uint32_t)(key & 0xFFFFFFFFull);
  st->token = tok;
  if (ids && st->step < max_ids) ids[st->step] = tok;
  st->step += 1;
  st->pos += 1;
  st->len += 1;
  if (st->fed < st->n_feed) st->fed += 1;
}

// tied head: one warp per vocabulary row, dot(xn, E[j]) over d
__global__ void k_tied_head(const TiedHeadParams p) {
  pdl_launch_dependents();
  pdl_wait();
  extern __shared__ float xn[];
  __shared__ float inv_s;
  if (threadIdx.x < 32) {
    float s = 0.0f;
    for (uint32_t i = threadIdx.x; i < p.n_ssq; i += 32) s += p.ssq[i];
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (threadIdx.x == 0) inv_s = 1.0f / sqrtf(s / (float)p.d + p.eps);
  }
  __syncthreads();
  for (uint32_t i = threadIdx.x; i < p.d; i += blockDim.x) xn[i] = __fmul_rn(__fmul_rn(p.x[i], inv_s), p.norm_w[i]);
  __syncthreads();
  const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x % 32, nw = blockDim.x / 32;
  unsigned long long best = 0ull;
  for (uint32_t j = blockIdx.x * nw + warp; j < p.vocab; j += gridDim.x * nw) {
    float s = 0.0f;
    for (uint32_t i = lane; i < p.d; i += 32) s = fmaf(xn[i], dequant_native_elem(p.type, p.emb, (uint64_t)j * p.d + i), s);
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xFFFFFFFFu, s, o);
    if (p.logits && lane == 0) p.logits[j] = s;
    const unsigned long long key = ((unsigned long long)float_key(s) << 32) | (unsigned long long)(~j);
    best = key > best ? key : best;
  }
  if (lane == 0 && best) atomicMax(&p.state->argmax_key, best);
}
}  // namespace

static cudaLaunchConfig_t make_cfg(dim3 g, dim3 b, size_t smem, cudaStream_t st, bool pdl, cudaLaunchAttribute *attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = g;
  cfg.blockDim = b;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

int launch_embed(const EmbedParams &p, bool pdl, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(p.n_ssq), dim3(256), 0, st, pdl, attr);
  return cudaLaunchKernelEx(&cfg, k_embed, p) == cudaSuccess ? 0 : -1;
}

int launch_step_end(SeqState *state, uint32_t *ids, uint32_t max_ids, bool pdl, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(1), dim3(1), 0, st, pdl, attr);
  return cudaLaunchKernelEx(&cfg, k_step_end, state, ids, max_ids) == cudaSuccess ? 0 : -1;
}

int launch_tied_head(const TiedHeadParams &p, bool pdl, cudaStream_t st) {
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(148 * 4), dim3(256), p.d * sizeof(float), st, pdl, attr);
  return cudaLaunchKernelEx(&cfg, k_tied_head, p) == cudaSuccess ? 0 : -1;
}

}  // namespace fa
